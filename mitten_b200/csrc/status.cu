// Status codes, the thread-local last-error string, the per-device error
// word kernels write instead of trapping, and small C-ABI utilities.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace mtn {

namespace {
thread_local char g_last_error[512] = "";

// Error word on every device that loads the library: [0] code, [1] detail.
__device__ int g_dev_error[2];

constexpr int kMaxDevices = 64;
int* g_dev_error_addr[kMaxDevices] = {};
std::mutex g_dev_error_mu;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  return set_error(MTN_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, what);
  return MTN_OK;
}

int sm_count() {
  static int cached[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int* device_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_dev_error_mu);
  if (g_dev_error_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
    g_dev_error_addr[dev] = static_cast<int*>(p);
  }
  return g_dev_error_addr[dev];
}

}  // namespace mtn

namespace mtn {
namespace {
// A wait that nothing completes: thread 0 waits on a fresh mbarrier with
// the same bounded wait the kernels use; after ~1 s it records
// kDevErrTimeout (detail `where`) and the kernel returns normally.
__global__ void bounded_wait_selftest_kernel(int* err, int where) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::wait_bounded(&bar, 0, &abort_flag, err, where);
}
}  // namespace
}  // namespace mtn

extern "C" {

const char* mtn_last_error(void) { return mtn::g_last_error; }

const char* mtn_version(void) { return "mitten_b200 0.1.0 (sm_100a)"; }

int mtn_device_error(int device, int clear, int32_t* code, int32_t* detail) {
  int prev = 0;
  MTN_CUDA_TRY(cudaGetDevice(&prev), "cudaGetDevice");
  MTN_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  int* p = mtn::device_error_ptr();
  if (p == nullptr) {
    cudaSetDevice(prev);
    return mtn::set_error(MTN_ECUDA, "device error word unavailable on device %d", device);
  }
  int host[2] = {0, 0};
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(host, p, sizeof(host), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) {
    int zero[2] = {0, 0};
    e = cudaMemcpy(p, zero, sizeof(zero), cudaMemcpyHostToDevice);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return mtn::cuda_status(e, "mtn_device_error");
  if (code) *code = host[0];
  if (detail) *detail = host[1];
  return MTN_OK;
}

size_t mtn_kv_required_bytes(int64_t num_pages, int64_t page_size, int64_t num_layers, int64_t num_kv_heads,
                             int64_t head_dim, int64_t dtype_bytes) {
  // kv_pool.rs:58-68: 2 (K + V) * layers * pages * page_size * heads * dim * dtype.
  return static_cast<size_t>(2 * num_layers * num_pages * page_size * num_kv_heads * head_dim * dtype_bytes);
}

int64_t mtn_kv_page_offset(const mtn_kv_layout* pool, int32_t layer, int32_t kv, int64_t page) {
  if (pool == nullptr) return -1;
  const int64_t page_elems = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * pool->head_dim;
  return ((static_cast<int64_t>(layer) * 2 + kv) * pool->num_pages + page) * page_elems;
}

int mtn_kv_pool_alloc(int device, mtn_kv_layout* out) {
  MTN_CHECK_ARG(out != nullptr, "mtn_kv_pool_alloc: null layout");
  MTN_CHECK_ARG(out->num_pages > 0 && out->num_layers > 0 && out->page_size > 0 && out->num_kv_heads > 0,
                "mtn_kv_pool_alloc: non-positive dimension");
  MTN_CHECK_ARG(out->head_dim == 64 || out->head_dim == 128 || out->head_dim == 256,
                "mtn_kv_pool_alloc: head_dim %d not in {64,128,256}", out->head_dim);
  const size_t bytes =
      mtn_kv_required_bytes(out->num_pages, out->page_size, out->num_layers, out->num_kv_heads, out->head_dim, 2);
  int prev = 0;
  MTN_CUDA_TRY(cudaGetDevice(&prev), "cudaGetDevice");
  MTN_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    if (e == cudaErrorMemoryAllocation) return mtn::set_error(MTN_ENOMEM, "pool of %zu bytes: out of device memory", bytes);
    return mtn::cuda_status(e, "mtn_kv_pool_alloc");
  }
  out->base = p;
  return MTN_OK;
}

int mtn_selftest_bounded_wait(void* stream) {
  int* err = mtn::device_error_ptr();
  if (err == nullptr) return mtn::set_error(MTN_ECUDA, "mtn_selftest_bounded_wait: no device error word");
  mtn::bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err, 99);
  return mtn::check_launch("bounded_wait_selftest_kernel");
}

int mtn_kv_pool_free(mtn_kv_layout* pool) {
  MTN_CHECK_ARG(pool != nullptr, "mtn_kv_pool_free: null layout");
  if (pool->base) MTN_CUDA_TRY(cudaFree(pool->base), "cudaFree");
  pool->base = nullptr;
  return MTN_OK;
}

}  // extern "C"
