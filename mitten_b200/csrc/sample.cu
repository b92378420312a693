// Token sampling on the device, bit-exact with the reference's sample_token
// (inference-engine/src/scheduler.rs:186-223), so an engine never copies a
// [rows, vocab] f32 logits block to the host:
//   temperature <= 0  first strict maximum (NaN never wins; an all -inf row
//                     gives 0), scheduler.rs:187-199;
//   temperature > 0   hash = fold over the first 100 logits' bit patterns
//                     (hash * 31 + bits, wrapping u64), rand = (hash % 1000) /
//                     1000 in f32; e_i = exp(l_i / t) in f32; sum = e_0 + e_1
//                     + ... in index order; the first i whose running sum of
//                     e_j / sum reaches rand, else the last index
//                     (scheduler.rs:201-222).
// The f32 operations are the reference's, in its order: IEEE division and
// addition (__fdiv_rn / __fadd_rn, never contracted or reassociated), and
// exp rounded correctly to f32 from the double-precision exp.  Rust's
// f32::exp calls libm's expf (glibc: at most 0.502 ulp), which is correctly
// rounded except for results within about 0.002 ulp of a rounding midpoint;
// only there can an e_i differ, by one ulp.  The two sums are sequential
// chains, as in the reference: one thread runs them over shared-memory
// chunks that the rest of the block computes and stages ahead of it.
#include "common.cuh"

namespace mtn {
namespace {

constexpr int kSampleThreads = 512;
constexpr int kChunk = 4096;  // floats per shared-memory stage of the two sequential sums

__device__ __forceinline__ float exp_f32(float x) { return __double2float_rn(exp(static_cast<double>(x))); }

__global__ void __launch_bounds__(kSampleThreads) sample_rows_kernel(const float* __restrict__ logits, int64_t vocab,
                                                                     const float* __restrict__ temps,
                                                                     float* __restrict__ ws, int32_t* __restrict__ out) {
  const int64_t r = blockIdx.x;
  const float* row = logits + r * vocab;
  const float t = temps[r];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (!(t > 0.0f)) {
    // Greedy: first strict max (x > best skips NaN, as the reference's loop does).
    float best = -INFINITY;
    int64_t idx = INT64_MAX;
    for (int64_t i = tid; i < vocab; i += kSampleThreads) {
      const float x = row[i];
      if (x > best) {
        best = x;
        idx = i;
      }
    }
    __shared__ float sv[kSampleThreads / 32];
    __shared__ int64_t si[kSampleThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) {
        best = ov;
        idx = oi;
      }
    }
    if (lane == 0) {
      sv[warp] = best;
      si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
      best = lane < kSampleThreads / 32 ? sv[lane] : -INFINITY;
      idx = lane < kSampleThreads / 32 ? si[lane] : INT64_MAX;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
          best = ov;
          idx = oi;
        }
      }
      if (lane == 0) out[r] = (best == -INFINITY || idx == INT64_MAX) ? 0 : static_cast<int32_t>(idx);
    }
    return;
  }
  // e_i = exp(l_i / t), every element in parallel, into this row's scratch.
  float* e = ws + r * vocab;
  for (int64_t i = tid; i < vocab; i += kSampleThreads) e[i] = exp_f32(__fdiv_rn(row[i], t));
  __syncthreads();
  __shared__ float buf[2][kChunk];
  __shared__ float sum_s;
  __shared__ int done_s;
  uint64_t hash = 0;
  float rand_val = 0.0f;
  if (tid == 0) {
    const int64_t nh = vocab < 100 ? vocab : 100;
    for (int64_t i = 0; i < nh; ++i) hash = hash * 31u + static_cast<uint64_t>(__float_as_uint(row[i]));
    rand_val = __fdiv_rn(static_cast<float>(hash % 1000u), 1000.0f);
    done_s = 0;
  }
  const int64_t nc = (vocab + kChunk - 1) / kChunk;
  // Both chains run in thread 0 over shared-memory chunks, while the other
  // threads stage the next chunk: pass 0 stages e_i and sums them in index
  // order; pass 1 stages e_i / sum and accumulates the running sum until it
  // reaches rand_val.
  float sum = 0.0f, cum = 0.0f;
  int64_t pick = vocab - 1;
  for (int pass = 0; pass < 2; ++pass) {
    const float div = pass ? sum_s : 1.0f;
    auto stage = [&](int64_t c) {
      const int64_t base = c * kChunk;
      for (int k = tid; k < kChunk; k += kSampleThreads) {
        const int64_t i = base + k;
        float x = 0.0f;
        if (i < vocab) x = pass ? __fdiv_rn(e[i], div) : e[i];
        buf[c & 1][k] = x;
      }
    };
    stage(0);
    __syncthreads();
    for (int64_t c = 0; c < nc; ++c) {
      if (c + 1 < nc) stage(c + 1);
      if (tid == 0 && !(pass == 1 && done_s)) {
        const float* b = buf[c & 1];
        const int n = static_cast<int>(min(static_cast<int64_t>(kChunk), vocab - c * kChunk));
        if (pass == 0) {
          int k = 0;
          for (; k + 8 <= n; k += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = b[k + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) sum = __fadd_rn(sum, v[j]);
          }
          for (; k < n; ++k) sum = __fadd_rn(sum, b[k]);
        } else {
          int k = 0;
          for (; k + 8 <= n; k += 8) {
            float v[8], run[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = b[k + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              cum = __fadd_rn(cum, v[j]);
              run[j] = cum;
            }
            int hit = -1;
#pragma unroll
            for (int j = 7; j >= 0; --j)
              if (rand_val <= run[j]) hit = j;  // the first crossing of the eight
            if (hit >= 0) {
              pick = c * kChunk + k + hit;
              done_s = 1;
              break;
            }
          }
          for (; !done_s && k < n; ++k) {
            cum = __fadd_rn(cum, b[k]);
            if (rand_val <= cum) {
              pick = c * kChunk + k;
              done_s = 1;
            }
          }
        }
      }
      __syncthreads();
      if (pass == 1 && done_s) break;  // every thread reads the flag after the barrier
    }
    if (pass == 0) {
      if (tid == 0) sum_s = sum;
      __syncthreads();
    }
  }
  if (tid != 0) return;
  out[r] = static_cast<int32_t>(pick);
}

}  // namespace
}  // namespace mtn

extern "C" {

size_t mtn_sample_rows_workspace_bytes(int64_t n_rows, int64_t vocab) {
  if (n_rows <= 0 || vocab <= 0) return 0;
  return static_cast<size_t>(n_rows) * static_cast<size_t>(vocab) * 4;
}

int mtn_sample_rows(const float* logits, const float* temperatures, int64_t n_rows, int64_t vocab, int32_t* out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  MTN_CHECK_ARG(n_rows >= 0 && n_rows <= INT32_MAX && vocab > 0 && vocab <= INT32_MAX, "mtn_sample_rows: bad sizes");
  if (n_rows == 0) return MTN_OK;
  MTN_CHECK_ARG(logits && temperatures && out, "mtn_sample_rows: null pointer");
  const size_t need = mtn_sample_rows_workspace_bytes(n_rows, vocab);
  MTN_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                "mtn_sample_rows: workspace of %zu bytes < %zu needed", workspace_bytes, need);
  mtn::sample_rows_kernel<<<static_cast<unsigned>(n_rows), mtn::kSampleThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, vocab, temperatures, static_cast<float*>(workspace), out);
  return mtn::check_launch("sample_rows_kernel");
}

}  // extern "C"
