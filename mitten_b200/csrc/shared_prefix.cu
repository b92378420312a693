// Decode over a prefix shared by every sequence of the batch (radix-cache
// prefix pages, config 3's 1024-token prompt head), computed once instead of
// once per sequence.
//
// The reference attends over each request's own contiguous cache
// (qwen model.rs:394-416); with refcounted prefix pages the same keys sit in
// every sequence's block table, and a plain paged decode reads them once per
// sequence.  Softmax attention splits exactly over any partition of the keys
// (each part's normalised output and its log-sum-exp recombine to the
// whole), so a step here is three launches on the caller's stream:
//   1. prefix part: the prefill kernel in its non-causal mode, every
//      sequence's query token one row of a single pseudo-sequence whose keys
//      are the shared pages -- K/V of the prefix read once per query head;
//   2. suffix part: the decode kernel over each sequence's own pages (with
//      the step's fused K/V append);
//   3. combine: out = (O_p 2^lse_p + O_s 2^lse_s) / (2^lse_p + 2^lse_s).
// The phantom zero row, when asked for, is counted once, in the prefix part.
#include <algorithm>

#include "common.cuh"

namespace mtn {
namespace {

struct SpLayout {
  size_t dec = 0, off_pf = 0, pf = 0, off_op = 0, off_os = 0, off_lp = 0, off_ls = 0, bytes = 0;
};

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

SpLayout sp_layout(int32_t n_seqs, int32_t hq, int32_t hkv, int32_t d) {
  SpLayout w;
  w.dec = up256(mtn_paged_decode_workspace_bytes(n_seqs, hq, hkv, d));
  if (w.dec == 0) return w;
  w.off_pf = w.dec;
  w.pf = up256(mtn_paged_prefill_workspace_bytes(1, n_seqs, hq, hkv, d));
  const size_t o_bytes = up256(static_cast<size_t>(n_seqs) * hq * d * 4);
  const size_t l_bytes = up256(static_cast<size_t>(n_seqs) * hq * 4);
  w.off_op = w.off_pf + w.pf;
  w.off_os = w.off_op + o_bytes;
  w.off_lp = w.off_os + o_bytes;
  w.off_ls = w.off_lp + l_bytes;
  w.bytes = w.off_ls + l_bytes;
  return w;
}

// out[r][:] = (o1[r] w1 + o2[r] w2) / (w1 + w2) with w = 2^(lse - max lse);
// a part whose lse is -inf (no key) has weight 0.  Four elements per thread.
__global__ void lse_combine_kernel(const float4* __restrict__ o1, const float* __restrict__ l1,
                                   const float4* __restrict__ o2, const float* __restrict__ l2, void* out,
                                   int out_f32, int64_t rows, int d4) {
  pdl_enter();  // launched as a dependent of the decode part
  const int64_t n = rows * d4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / d4;
    const float a = l1[r], b = l2[r];
    const float m = fmaxf(a, b);
    const float wa = a == -INFINITY ? 0.0f : exp2f(a - m);
    const float wb = b == -INFINITY ? 0.0f : exp2f(b - m);
    const float inv = wa + wb > 0.0f ? 1.0f / (wa + wb) : 0.0f;
    const float4 x = o1[i], y = o2[i];
    const float4 z = make_float4((x.x * wa + y.x * wb) * inv, (x.y * wa + y.y * wb) * inv,
                                 (x.z * wa + y.z * wb) * inv, (x.w * wa + y.w * wb) * inv);
    if (out_f32) {
      static_cast<float4*>(out)[i] = z;
    } else {
      static_cast<uint2*>(out)[i] = make_uint2(f2_to_bf2(z.x, z.y), f2_to_bf2(z.z, z.w));
    }
  }
}

}  // namespace
}  // namespace mtn

extern "C" {

size_t mtn_paged_decode_shared_prefix_workspace_bytes(int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                                      int32_t head_dim) {
  if (n_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0) return 0;
  return mtn::sp_layout(n_seqs, num_q_heads, num_kv_heads, head_dim).bytes;
}

int mtn_paged_decode_shared_prefix(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype,
                                   void* o, int32_t o_dtype, const void* k_new, const void* v_new,
                                   int32_t new_dtype, int32_t n_seqs, int32_t num_q_heads,
                                   const int32_t* prefix_pages, int32_t n_prefix_pages, const int32_t* kv_indptr,
                                   const int32_t* kv_indices, const int32_t* seq_lens, float scale, uint32_t flags,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  int st = mtn::validate_layout(pool, layer, "mtn_paged_decode_shared_prefix");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_seqs >= 0, "mtn_paged_decode_shared_prefix: n_seqs < 0");
  if (n_seqs == 0) return MTN_OK;
  MTN_CHECK_ARG(q && o && kv_indptr && kv_indices && seq_lens, "mtn_paged_decode_shared_prefix: null pointer");
  MTN_CHECK_ARG(prefix_pages != nullptr && n_prefix_pages > 0,
                "mtn_paged_decode_shared_prefix: the shared prefix needs at least one page");
  MTN_CHECK_ARG(o_dtype == MTN_DTYPE_BF16 || o_dtype == MTN_DTYPE_F32, "mtn_paged_decode_shared_prefix: bad o dtype");
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(o) & 15) == 0, "mtn_paged_decode_shared_prefix: o must be 16-byte aligned");
  MTN_CHECK_ARG(num_q_heads > 0 && num_q_heads <= 65535, "mtn_paged_decode_shared_prefix: bad num_q_heads");
  MTN_CHECK_ARG(!(flags & MTN_ATTN_SPLIT_BF16),
                "mtn_paged_decode_shared_prefix: MTN_ATTN_SPLIT_BF16 is not supported (bf16 operands only)");
  MTN_CHECK_ARG(n_seqs <= (1 << 24), "mtn_paged_decode_shared_prefix: n_seqs %d too large", n_seqs);
  const int64_t prefix_len = static_cast<int64_t>(n_prefix_pages) * pool->page_size;
  MTN_CHECK_ARG(prefix_len < (int64_t(1) << 31), "mtn_paged_decode_shared_prefix: prefix too long");
  const int D = pool->head_dim;
  const mtn::SpLayout wl = mtn::sp_layout(n_seqs, num_q_heads, pool->num_kv_heads, D);
  MTN_CHECK_ARG(wl.bytes > 0, "mtn_paged_decode_shared_prefix: unsupported shape (head_dim %d)", D);
  MTN_CHECK_ARG(workspace != nullptr && workspace_bytes >= wl.bytes,
                "mtn_paged_decode_shared_prefix: workspace of %zu bytes < %zu needed", workspace_bytes, wl.bytes);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                "mtn_paged_decode_shared_prefix: workspace must be 256-byte aligned");
  uint8_t* w = static_cast<uint8_t*>(workspace);
  float* o_p = reinterpret_cast<float*>(w + wl.off_op);
  float* o_s = reinterpret_cast<float*>(w + wl.off_os);
  float* l_p = reinterpret_cast<float*>(w + wl.off_lp);
  float* l_s = reinterpret_cast<float*>(w + wl.off_ls);
  auto s = static_cast<cudaStream_t>(stream);
  // 1. prefix part (phantom row counted here, once): one pseudo-sequence of
  //    n_seqs query rows over the prefix pages
  st = mtn::paged_prefill_impl(pool, layer, q, q_dtype, o_p, MTN_DTYPE_F32, 1, n_seqs, num_q_heads, nullptr, nullptr,
                               prefix_pages, nullptr, n_seqs, scale, flags & ~MTN_ATTN_PREFILL_ONE_TILE,
                               wl.pf ? w + wl.off_pf : nullptr, wl.pf, stream, 1, l_p, n_prefix_pages);
  if (st != MTN_OK) return st;
  // 2. suffix part: each sequence's own pages, with the step's append
  st = mtn::paged_decode_impl(pool, layer, q, q_dtype, o_s, MTN_DTYPE_F32, k_new, v_new, new_dtype, n_seqs,
                              num_q_heads, kv_indptr, kv_indices, seq_lens, scale,
                              flags & ~(MTN_ATTN_PHANTOM_ZERO_SLOT | MTN_ATTN_PREFILL_ONE_TILE), nullptr, w, wl.dec,
                              stream, l_s);
  if (st != MTN_OK) return st;
  // 3. combine
  const int64_t rows = static_cast<int64_t>(n_seqs) * num_q_heads;
  const int64_t n4 = rows * (D / 4);
  const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(mtn::sm_count()) * 16));
  return mtn::launch_pdl(mtn::lse_combine_kernel, dim3(grid), dim3(256), 0, s, "lse_combine_kernel",
                         reinterpret_cast<const float4*>(o_p), static_cast<const float*>(l_p),
                         reinterpret_cast<const float4*>(o_s), static_cast<const float*>(l_s), o,
                         static_cast<int>(o_dtype == MTN_DTYPE_F32), rows, D / 4);
}

}  // extern "C"
