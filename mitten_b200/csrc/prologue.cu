// Fused attention prologue for the paged-KV path: the per-head q/k work
// between the projection GEMMs and attention, in one launch.  Replaces, for
// every token row of a batch,
//   q = RoPE(RMSNorm_(1+w)(q_proj head))   (qwen model.rs:372-384)
//   k = RoPE(RMSNorm_(1+w)(k_proj head)), v = v_proj head, stored into the
//       pool at the token's slot          (model.rs:380-392, the paged cat)
// RMSNorm: x / sqrt(mean(x^2) + eps) * (1 + w), omitted when no weight is
// given (Gemma has no q/k norm).  RoPE: rotate-half over the first
// rotary_dim elements, angle = position * inv_freq[i] in f32, cos/sin of
// that angle; the products and the sum are rounded separately, as an
// elementwise evaluation of x1*c - x2*s and x2*c + x1*s does.
//
// One warp per (token, head) row; lane l holds elements l + 32 k, so the
// rotate-half partner of element i (i + rotary_dim / 2) sits in the same
// lane when rotary_dim / 2 is a multiple of 32.
#include "common.cuh"

namespace mtn {
namespace {

constexpr int kPrologueThreads = 256;

template <int D, bool kBf16In>
__device__ __forceinline__ void load_row(const void* src, int64_t off, float (&x)[D / 32], int lane) {
#pragma unroll
  for (int k = 0; k < D / 32; ++k) {
    const int64_t i = off + lane + 32 * k;
    x[k] = kBf16In ? __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]) : static_cast<const float*>(src)[i];
  }
}

// RMSNorm (1 + w) then RoPE of one row held as x[k] = element lane + 32 k.
template <int D>
__device__ __forceinline__ void norm_rope(float (&x)[D / 32], const float* w1, float eps, float pos,
                                          const float* inv_freq, int rd, int lane) {
  if (w1 != nullptr) {
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < D / 32; ++k) ss = fmaf(x[k], x[k], ss);
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int k = 0; k < D / 32; ++k) x[k] = x[k] * rstd * w1[lane + 32 * k];
  }
  const int half = rd / 2, kh = half / 32;  // partner of slot k is slot k + kh
#pragma unroll
  for (int k = 0; k < D / 32; ++k) {
    if (k >= kh) continue;  // handled with its partner
    const int i = lane + 32 * k;
    const float ang = __fmul_rn(pos, inv_freq[i]);
    const float c = cosf(ang), s = sinf(ang);
    const float x1 = x[k], x2 = x[k + kh];
    x[k] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    x[k + kh] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
}

struct PrologueParams {
  const void* q;  // [T][hq][qg][D]: per head q then (qg = 2) its gate
  const void* k;  // rows k_stride elements apart, [hkv][D] each
  const void* v;
  int64_t q_stride, k_stride, v_stride;  // elements between token rows
  int qg;
  int hq, hkv;
  const float* q_w1;  // [D] (1 + w) or null
  const float* k_w1;
  const float* inv_freq;  // [rd / 2]
  int rd;
  float eps;
  const int32_t* pos;  // [T]
  const int64_t* slots;  // [T] pool slot (page * page_size + offset), < 0: not stored
  int64_t n_tokens;
  float* q_out;  // [T][hq][D] f32
  __nv_bfloat16* pool;
  int64_t num_pages;
  int ps;
  int64_t k_base, v_base;  // element offsets of this layer's K and V blocks
  int* err;
};

template <int D, bool kBf16In>
__global__ void __launch_bounds__(kPrologueThreads) qkv_prologue_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t rows_per_tok = p.hq + p.hkv;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * kPrologueThreads + threadIdx.x) / 32;
  if (row >= p.n_tokens * rows_per_tok) return;
  const int64_t t = row / rows_per_tok;
  const int h = static_cast<int>(row - t * rows_per_tok);
  const float pos = static_cast<float>(p.pos[t]);
  float x[D / 32];
  if (h < p.hq) {
    load_row<D, kBf16In>(p.q, t * p.q_stride + static_cast<int64_t>(h) * p.qg * D, x, lane);
    norm_rope<D>(x, p.q_w1, p.eps, pos, p.inv_freq, p.rd, lane);
    float* o = p.q_out + (t * p.hq + h) * D;
#pragma unroll
    for (int k = 0; k < D / 32; ++k) o[lane + 32 * k] = x[k];
    return;
  }
  const int g = h - p.hq;
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  if (slot >= p.num_pages * p.ps) {
    if (lane == 0 && g == 0) record_error(p.err, kDevErrBadSlot, static_cast<int>(t));
    return;
  }
  load_row<D, kBf16In>(p.k, t * p.k_stride + static_cast<int64_t>(g) * D, x, lane);
  norm_rope<D>(x, p.k_w1, p.eps, pos, p.inv_freq, p.rd, lane);
  // pool [layer][K|V][page][hkv][ps][D]: row (page, g, offset)
  const int64_t page = slot / p.ps, off = slot - page * p.ps;
  const int64_t dst = ((page * p.hkv + g) * p.ps + off) * D;
#pragma unroll
  for (int k = 0; k < D / 32; ++k) p.pool[p.k_base + dst + lane + 32 * k] = __float2bfloat16_rn(x[k]);
  load_row<D, kBf16In>(p.v, t * p.v_stride + static_cast<int64_t>(g) * D, x, lane);
#pragma unroll
  for (int k = 0; k < D / 32; ++k) p.pool[p.v_base + dst + lane + 32 * k] = __float2bfloat16_rn(x[k]);
}

template <int D>
int launch_prologue(const PrologueParams& prm, bool bf16_in, cudaStream_t s) {
  const int64_t rows = prm.n_tokens * (prm.hq + prm.hkv);
  const int64_t blocks = (rows * 32 + kPrologueThreads - 1) / kPrologueThreads;
  if (blocks > 0x7fffffff) return set_error(MTN_EINVAL, "mtn_qkv_prologue: batch too large");
  if (bf16_in)
    qkv_prologue_kernel<D, true><<<static_cast<unsigned>(blocks), kPrologueThreads, 0, s>>>(prm);
  else
    qkv_prologue_kernel<D, false><<<static_cast<unsigned>(blocks), kPrologueThreads, 0, s>>>(prm);
  return check_launch("qkv_prologue_kernel");
}

}  // namespace
}  // namespace mtn

extern "C" {

int mtn_qkv_prologue(const mtn_kv_layout* pool, int32_t layer, const void* q, const void* k, const void* v,
                     int32_t src_dtype, int64_t q_stride, int64_t k_stride, int64_t v_stride, int32_t q_gated,
                     int32_t num_q_heads, const float* q_norm_w1, const float* k_norm_w1, float eps,
                     const float* inv_freq, int32_t rotary_dim, const int32_t* positions, const int64_t* slots,
                     int64_t n_tokens, float* q_out, void* stream) {
  int st = mtn::validate_layout(pool, layer, "mtn_qkv_prologue");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_tokens >= 0, "mtn_qkv_prologue: n_tokens < 0");
  if (n_tokens == 0) return MTN_OK;
  MTN_CHECK_ARG(q && k && v && inv_freq && positions && slots && q_out, "mtn_qkv_prologue: null pointer");
  MTN_CHECK_ARG(src_dtype == MTN_DTYPE_BF16 || src_dtype == MTN_DTYPE_F32, "mtn_qkv_prologue: bad dtype");
  const int D = pool->head_dim;
  MTN_CHECK_ARG(rotary_dim > 0 && rotary_dim <= D && rotary_dim % 64 == 0,
                "mtn_qkv_prologue: rotary_dim %d must be a multiple of 64 up to head_dim %d", rotary_dim, D);
  MTN_CHECK_ARG(num_q_heads > 0 && num_q_heads % pool->num_kv_heads == 0, "mtn_qkv_prologue: bad head counts");
  const int qg = q_gated ? 2 : 1;
  MTN_CHECK_ARG(q_stride >= static_cast<int64_t>(num_q_heads) * qg * D && k_stride >= pool->num_kv_heads * D &&
                    v_stride >= pool->num_kv_heads * D,
                "mtn_qkv_prologue: row strides shorter than a row");
  mtn::PrologueParams prm{};
  prm.q = q;
  prm.k = k;
  prm.v = v;
  prm.q_stride = q_stride;
  prm.k_stride = k_stride;
  prm.v_stride = v_stride;
  prm.qg = qg;
  prm.hq = num_q_heads;
  prm.hkv = pool->num_kv_heads;
  prm.q_w1 = q_norm_w1;
  prm.k_w1 = k_norm_w1;
  prm.inv_freq = inv_freq;
  prm.rd = rotary_dim;
  prm.eps = eps;
  prm.pos = positions;
  prm.slots = slots;
  prm.n_tokens = n_tokens;
  prm.q_out = q_out;
  prm.pool = static_cast<__nv_bfloat16*>(pool->base);
  prm.num_pages = pool->num_pages;
  prm.ps = pool->page_size;
  const int64_t block = pool->num_pages * pool->num_kv_heads * pool->page_size * static_cast<int64_t>(D);
  prm.k_base = (static_cast<int64_t>(layer) * 2 + 0) * block;
  prm.v_base = (static_cast<int64_t>(layer) * 2 + 1) * block;
  prm.err = mtn::device_error_ptr();
  const bool bf16 = src_dtype == MTN_DTYPE_BF16;
  auto s = static_cast<cudaStream_t>(stream);
  switch (D) {
    case 64: return mtn::launch_prologue<64>(prm, bf16, s);
    case 128: return mtn::launch_prologue<128>(prm, bf16, s);
    default: return mtn::launch_prologue<256>(prm, bf16, s);
  }
}

}  // extern "C"
