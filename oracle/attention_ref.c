/*
 * TEST INFRASTRUCTURE -- CPU oracle for the paged-KV hot path.  Only the
 * test suite, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
 * this file; the product path never links it.
 *
 * f32 restatement of the reference's attention (tianhaoz95/mitten,
 * inference-model-qwen/src/model.rs), in the reference's own data layout:
 * a contiguous per-request cache KVCacheState::Attention [Hkv][T][D]
 * (inference-model-common/src/lib.rs:5-13) whose row 0 is the all-zero row
 * seeded by init_cache (model.rs:207-220).
 *
 * Parity status: the reference's arithmetic runs inside Burn 0.16.1's
 * NdArray backend (burn-ndarray 0.16.1 -> ndarray 0.16.1 +
 * matrixmultiply 0.3.10, Cargo.lock), which is not vendored and cannot be
 * built here (no Rust toolchain).  No reference test pins any attention
 * value, so attention numerics are "parity unpinned" at the Burn boundary;
 * this file restates the published op sequence and the tests hold the CUDA
 * kernels to it within the 2e-2 max-abs tolerance the spec states.
 *
 * Functions:
 *   ref_attention      one GatedAttention core over a contiguous cache
 *                      (model.rs:394-416 + generate_causal_mask :542-555).
 *   ref_catgrown_step  the reference's decode step as it executes on the
 *                      CPU path: Tensor::cat growth of the cache
 *                      (model.rs:390-392), n_rep x `repeat` of K/V
 *                      (model.rs:398-408), a materialised -1e10 mask
 *                      (model.rs:410-411), q.k^T*scale, softmax, P.V
 *                      (model.rs:413-416).  Used as the timed CPU baseline.
 *   ref_sample_token   sample_token (scheduler.rs:186-223) of one logits row.
 *   ref_rne_bf16       f32 -> bf16 round-to-nearest-even (IEEE), the rounding
 *                      the device path applies when K/V are stored as bf16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Burn's softmax over the last dim: exp(x - max) / sum(exp(x - max)). */
static void softmax_row(float* x, int64_t n) {
  float m = -INFINITY;
  for (int64_t j = 0; j < n; ++j) m = x[j] > m ? x[j] : m;
  float s = 0.0f;
  for (int64_t j = 0; j < n; ++j) {
    x[j] = expf(x[j] - m);
    s += x[j];
  }
  for (int64_t j = 0; j < n; ++j) x[j] /= s;
}

/*
 * q    [S][Hq][D]   queries of this call (after q_norm + RoPE), f32
 * kc   [Hkv][T][D]  contiguous cache AFTER appending the S new rows
 * vc   [Hkv][T][D]
 * out  [S][Hq][D]   attention output before the sigmoid gate
 * Query i of S attends to keys j <= T - S + i (model.rs:545-551); head h
 * reads kv head h / (Hq / Hkv) (model.rs:398-408).
 */
void ref_attention(const float* q, const float* kc, const float* vc, int64_t T, int64_t S, int64_t Hq, int64_t Hkv,
                   int64_t D, float scale, float* out) {
  const int64_t n_rep = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t h = 0; h < Hq; ++h) {
    for (int64_t i = 0; i < S; ++i) {
      const int64_t g = h / n_rep;
      const float* qi = q + (i * Hq + h) * D;
      const float* kg = kc + g * T * D;
      const float* vg = vc + g * T * D;
      float* sc = (float*)malloc(sizeof(float) * (size_t)T);
      const int64_t cur = T - S + i;
      for (int64_t j = 0; j < T; ++j) {
        float acc = 0.0f;
        for (int64_t d = 0; d < D; ++d) acc += qi[d] * kg[j * D + d];
        sc[j] = acc * scale + (j > cur ? -1e10f : 0.0f);
      }
      softmax_row(sc, T);
      float* oi = out + (i * Hq + h) * D;
      for (int64_t d = 0; d < D; ++d) oi[d] = 0.0f;
      for (int64_t j = 0; j < T; ++j) {
        const float p = sc[j];
        for (int64_t d = 0; d < D; ++d) oi[d] += p * vg[j * D + d];
      }
      free(sc);
    }
  }
}

/*
 * One decode step of the reference CPU path for a batch of requests, each
 * with its own contiguous cache (served one request at a time, as
 * BurnBackend::forward does, burn_backend.rs:44-71).
 *   caches[r]   in/out: [Hkv][T_r][D] on entry; reallocated to T_r + 1 rows
 *   lens[r]     in/out: T_r (phantom row included)
 *   knew/vnew   [n_req][Hkv][D] rows appended this step
 *   q           [n_req][Hq][D]
 *   out         [n_req][Hq][D]
 * Work is spread over requests x query heads with OpenMP (the reference
 * itself runs ndarray/rayon under the Burn backend).
 */
void ref_catgrown_step(float** kcaches, float** vcaches, int64_t* lens, const float* knew, const float* vnew,
                       const float* q, int64_t n_req, int64_t Hq, int64_t Hkv, int64_t D, float scale, float* out) {
  const int64_t n_rep = Hq / Hkv;
  /* Tensor::cat: a fresh [Hkv][T+1][D] buffer holding old rows + new row. */
#pragma omp parallel for schedule(dynamic)
  for (int64_t r = 0; r < n_req; ++r) {
    const int64_t T = lens[r];
    float* nk = (float*)malloc(sizeof(float) * (size_t)(Hkv * (T + 1) * D));
    float* nv = (float*)malloc(sizeof(float) * (size_t)(Hkv * (T + 1) * D));
    for (int64_t g = 0; g < Hkv; ++g) {
      memcpy(nk + g * (T + 1) * D, kcaches[r] + g * T * D, sizeof(float) * (size_t)(T * D));
      memcpy(nv + g * (T + 1) * D, vcaches[r] + g * T * D, sizeof(float) * (size_t)(T * D));
      memcpy(nk + (g * (T + 1) + T) * D, knew + (r * Hkv + g) * D, sizeof(float) * (size_t)D);
      memcpy(nv + (g * (T + 1) + T) * D, vnew + (r * Hkv + g) * D, sizeof(float) * (size_t)D);
    }
    free(kcaches[r]);
    free(vcaches[r]);
    kcaches[r] = nk;
    vcaches[r] = nv;
    lens[r] = T + 1;
  }
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t r = 0; r < n_req; ++r) {
    for (int64_t h = 0; h < Hq; ++h) {
      const int64_t T = lens[r];
      const int64_t g = h / n_rep;
      /* repeat(): this head's private copy of its KV head's rows. */
      float* ke = (float*)malloc(sizeof(float) * (size_t)(T * D));
      float* ve = (float*)malloc(sizeof(float) * (size_t)(T * D));
      memcpy(ke, kcaches[r] + g * T * D, sizeof(float) * (size_t)(T * D));
      memcpy(ve, vcaches[r] + g * T * D, sizeof(float) * (size_t)(T * D));
      /* materialised mask row for the single query (seq = 1): all zeros. */
      float* mask = (float*)calloc((size_t)T, sizeof(float));
      float* sc = (float*)malloc(sizeof(float) * (size_t)T);
      const float* qi = q + (r * Hq + h) * D;
      for (int64_t j = 0; j < T; ++j) {
        float acc = 0.0f;
        for (int64_t d = 0; d < D; ++d) acc += qi[d] * ke[j * D + d];
        sc[j] = acc * scale + mask[j];
      }
      softmax_row(sc, T);
      float* oi = out + (r * Hq + h) * D;
      for (int64_t d = 0; d < D; ++d) oi[d] = 0.0f;
      for (int64_t j = 0; j < T; ++j)
        for (int64_t d = 0; d < D; ++d) oi[d] += sc[j] * ve[j * D + d];
      free(ke);
      free(ve);
      free(mask);
      free(sc);
    }
  }
}

/* IEEE round-to-nearest-even f32 -> bf16 (NaN kept quiet). */
uint16_t ref_rne_bf16_one(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

void ref_rne_bf16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ref_rne_bf16_one(x[i]);
}

int ref_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* sample_token (inference-engine/src/scheduler.rs:186-223) on one logits row,
 * in the reference's f32 operations and order.  temperature <= 0: index of
 * the first strict maximum (val > max_val; NaN never wins).  Otherwise:
 * hash = fold over the first 100 logits of hash * 31 + bits (wrapping u64),
 * rand = (hash % 1000) / 1000 in f32, e_i = expf(l_i / t) (libm's expf, which
 * Rust's f32::exp calls), sum = e_0 + e_1 + ... left to right, then the first
 * i whose running sum of e_i / sum reaches rand, else the last index.
 * scratch: vocab floats.  Built without -ffast-math, so no sum is
 * reassociated. */
int64_t ref_sample_token(const float* row, int64_t vocab, float temperature, float* scratch) {
  if (temperature <= 0.0f) {
    float max_val = -INFINITY;
    int64_t max_idx = 0;
    for (int64_t i = 0; i < vocab; ++i) {
      if (row[i] > max_val) {
        max_val = row[i];
        max_idx = i;
      }
    }
    return max_idx;
  }
  uint64_t hash = 0;
  for (int64_t i = 0; i < vocab && i < 100; ++i) {
    uint32_t bits;
    memcpy(&bits, &row[i], 4);
    hash = hash * 31u + (uint64_t)bits;
  }
  const float rand_val = (float)(hash % 1000u) / 1000.0f;
  for (int64_t i = 0; i < vocab; ++i) scratch[i] = expf(row[i] / temperature);
  float sum = 0.0f;
  for (int64_t i = 0; i < vocab; ++i) sum += scratch[i];
  float cum = 0.0f;
  for (int64_t i = 0; i < vocab; ++i) {
    cum += scratch[i] / sum;
    if (rand_val <= cum) return i;
  }
  return vocab - 1;
}
