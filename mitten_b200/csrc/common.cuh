// Shared device helpers for the sm_100a paged-KV kernels: status plumbing,
// the device error word, mbarrier / bulk-copy wrappers (inline PTX), and
// bf16 <-> f32 packing.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mitten_kv.h"

namespace mtn {

// ---------------------------------------------------------------- host side

// Thread-local last-error message (mtn_last_error).
int set_error(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

#define MTN_CHECK_ARG(cond, ...)                          \
  do {                                                    \
    if (!(cond)) return ::mtn::set_error(MTN_EINVAL, __VA_ARGS__); \
  } while (0)

#define MTN_CUDA_TRY(expr, what)                          \
  do {                                                    \
    cudaError_t _e = (expr);                              \
    if (_e != cudaSuccess) return ::mtn::cuda_status(_e, what); \
  } while (0)

// Launch-result check after a <<<>>> launch.
int check_launch(const char* what);

// Launch with programmatic dependent launch allowed: the kernel may begin
// while the previous kernel of the stream finishes, if that kernel lets it
// (griddepcontrol.launch_dependents); kernels launched this way execute
// griddepcontrol.wait before touching memory another kernel may write.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
  if (e != cudaSuccess) return cuda_status(e, what);
  return check_launch(what);
}

// First statements of a kernel launched with launch_pdl: wait for the
// previous grid's memory, then let the next grid start its CTAs.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Device error word: [0] = first error code, [1] = detail.
int* device_error_ptr();  // device address for the current device

// Shared argument checks for a pool layout and layer index.
int validate_layout(const mtn_kv_layout* pool, int layer, const char* who);

// SM count of the current device (cached per device).
int sm_count();

// Internal forms of mtn_paged_prefill / mtn_paged_decode_with_plan for the
// shared-prefix decode: `lse` (or null) receives each (row, query head)'s
// log2-domain log-sum-exp; `noncausal` lets every prefill query see every
// key of its sequence.
int paged_prefill_impl(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                       int32_t o_dtype, int32_t n_seqs, int64_t total_q, int32_t num_q_heads,
                       const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
                       const int32_t* seq_lens, int32_t max_q_len, float scale, uint32_t flags, void* workspace,
                       size_t workspace_bytes, void* stream, int noncausal, float* lse, int nc_pages);
int paged_decode_impl(const mtn_kv_layout* pool, int32_t layer, const void* q, int32_t q_dtype, void* o,
                      int32_t o_dtype, const void* k_new, const void* v_new, int32_t new_dtype, int32_t n_seqs,
                      int32_t num_q_heads, const int32_t* kv_indptr, const int32_t* kv_indices,
                      const int32_t* seq_lens, float scale, uint32_t flags, const void* plan, void* workspace,
                      size_t workspace_bytes, void* stream, float* lse);

// Device error codes (written by kernels, read by mtn_device_error).
enum DevErr : int {
  kDevErrNone = 0,
  kDevErrBadPage = 1,       // page id outside [0, num_pages)
  kDevErrBadSeqLen = 2,     // seq_len negative or beyond its pages
  kDevErrBadSlot = 3,       // slot outside the pool
  kDevErrTimeout = 4,       // bounded wait ran out
  kDevErrBadPosition = 5,   // position beyond a sequence's pages
  kDevErrBadPlan = 6        // decode plan made for another grid (detail: its grid) or not a plan (-1)
};

// ---------------------------------------------------------------- device side

__device__ __forceinline__ void record_error(int* err, int code, int detail) {
  if (err != nullptr && atomicCAS(err, 0, code) == 0) {
    atomicExch(err + 1, detail);
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Plain arrival (no transaction bytes).
__device__ __forceinline__ void mbar_arrive_plain(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Non-blocking probe: has the phase with parity `parity` of `bar` completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` with a bounded budget of polls.  Returns
// false (and records kDevErrTimeout) if the budget runs out.  try_wait
// itself suspends for a hardware-defined interval per poll, so the budget
// bounds the total wait to well under a second.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int where) {
  constexpr uint32_t kMaxPolls = 1u << 22;
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_error(err, kDevErrTimeout, where);
  return false;
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map).  dst/src 16-byte
// aligned, bytes a multiple of 16.  Completion is signalled on `bar` as
// transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy shared -> global, tracked by bulk async-groups of the
// issuing thread (commit with bulk_commit_group, wait with bulk_wait_*).
__device__ __forceinline__ void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem), "r"(smem_u32(src_smem)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N of this thread's bulk groups still reading their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every bulk group of this thread complete (its global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Log2-domain log-sum-exp of a softmax row kept as a running max m and sum
// l = sum 2^(s - m) (scores s already scaled into log2 units), with the
// reference's all-zero phantom key (score 0) folded in when `phantom` is
// set: log2(2^m * l [+ 1]).  -inf for a row with no key at all.
__device__ __forceinline__ float row_lse(int phantom, float m, float l) {
  if (phantom) {
    const float mf = fmaxf(m, 0.0f);  // m == -inf (no real keys) gives mf = 0
    const float a = m == -INFINITY ? 0.0f : exp2f(m - mf);
    return mf + log2f(l * a + exp2f(-mf));
  }
  return l > 0.0f ? m + log2f(l) : -INFINITY;
}

// bf16x2 (packed in a 32-bit word, low half = element 0) -> two floats.
__device__ __forceinline__ float2 bf2_to_f2(uint32_t w) {
  float2 r;
  r.x = __uint_as_float(w << 16);
  r.y = __uint_as_float(w & 0xffff0000u);
  return r;
}

__device__ __forceinline__ float bf_to_f(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

__device__ __forceinline__ uint32_t f2_to_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16x2 of the rounding remainders (a - hi.lo, b - hi.hi) of two f32 values
// whose bf16 pair (round to nearest even) is `hi`: hi + lo carries about 16
// significant bits of each value.
__device__ __forceinline__ uint32_t bf2_residual(uint32_t hi, float a, float b) {
  const float2 h = bf2_to_f2(hi);
  return f2_to_bf2(a - h.x, b - h.y);
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// L2-coherent loads for data written by other CTAs of the same launch.
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

}  // namespace mtn
