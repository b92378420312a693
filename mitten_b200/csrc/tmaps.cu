// Host-side TMA tensor maps.  The pool map views the whole KV pool as a 2-D
// bf16 tensor [layers*2*pages*kv_heads*page_size rows, head_dim]; a box is
// box_rows rows x 64 columns with 128B swizzle (one page of one kv head for
// prefill, one page of every kv head for decode).  Maps are cached per pool
// layout and box height so a decode step encodes nothing.  The paged map is a
// 4-D view of the same memory that brings one page of one kv head in a single
// box whatever the head dim (see pool_tensor_map_paged).
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "tmaps.hpp"

namespace mtn {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(f);
  });
  return fn;
}

struct PoolKey {
  uintptr_t base;
  int64_t pages;
  int32_t layers, ps, hkv, d, box_rows;
  bool operator==(const PoolKey& o) const {
    return base == o.base && pages == o.pages && layers == o.layers && ps == o.ps && hkv == o.hkv && d == o.d &&
           box_rows == o.box_rows;
  }
};

struct PoolKeyHash {
  size_t operator()(const PoolKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.base);
    h ^= std::hash<int64_t>()(k.pages) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= static_cast<size_t>(k.layers * 131 + k.ps * 7 + k.hkv * 3 + k.d + k.box_rows * 1009);
    return h;
  }
};

std::mutex g_mu;
std::unordered_map<PoolKey, CUtensorMap, PoolKeyHash> g_pool_maps;

}  // namespace

int64_t pool_rows(const mtn_kv_layout* pool) {
  return static_cast<int64_t>(pool->num_layers) * 2 * pool->num_pages * pool->num_kv_heads * pool->page_size;
}

int pool_tensor_map(const mtn_kv_layout* pool, CUtensorMap* out, int box_rows) {
  const int64_t rows = pool_rows(pool);
  if (rows >= (int64_t(1) << 31))
    return set_error(MTN_EINVAL, "pool has %lld rows; TMA coordinates need < 2^31", (long long)rows);
  if (box_rows <= 0) box_rows = pool->page_size;
  if (box_rows > 256 || box_rows % 8 != 0)
    return set_error(MTN_EINVAL, "TMA pool boxes of %d rows: need a multiple of 8 up to 256", box_rows);
  const PoolKey key{reinterpret_cast<uintptr_t>(pool->base), pool->num_pages, pool->num_layers, pool->page_size,
                    pool->num_kv_heads, pool->head_dim, box_rows};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pool_maps.find(key);
    if (it != g_pool_maps.end()) {
      *out = it->second;
      return MTN_OK;
    }
  }
  auto enc = encoder();
  if (enc == nullptr) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(pool->head_dim), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pool->head_dim) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, pool->base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled(pool) failed: %d", (int)r);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_pool_maps.size() > 256) g_pool_maps.clear();
  g_pool_maps[key] = m;
  *out = m;
  return MTN_OK;
}

int pool_tensor_map_paged(const mtn_kv_layout* pool, CUtensorMap* out) {
  const int64_t rows = pool_rows(pool);
  const int ps = pool->page_size, d = pool->head_dim;
  if (rows >= (int64_t(1) << 34))
    return set_error(MTN_EINVAL, "pool has %lld rows; TMA coordinates need rows / 8 < 2^31", (long long)rows);
  if (ps % 8 != 0 || ps > 2048 || d % 64 != 0 || d > 256)
    return set_error(MTN_EINVAL, "paged TMA map: page_size %d (multiple of 8) / head_dim %d (64..256)", ps, d);
  const PoolKey key{reinterpret_cast<uintptr_t>(pool->base), pool->num_pages, pool->num_layers, ps,
                    pool->num_kv_heads, d, -1};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pool_maps.find(key);
    if (it != g_pool_maps.end()) {
      *out = it->second;
      return MTN_OK;
    }
  }
  auto enc = encoder();
  if (enc == nullptr) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  // dim 0: 64 columns; dim 1: 8 consecutive rows; dim 2: the 64-column blocks of a row
  // (128 bytes apart); dim 3: 8-row groups.  Every address stays inside the pool.
  const cuuint64_t dims[4] = {64, 8, static_cast<cuuint64_t>(d / 64), static_cast<cuuint64_t>(rows / 8)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, 128, static_cast<cuuint64_t>(d) * 16};
  const cuuint32_t box[4] = {64, 8, static_cast<cuuint32_t>(d / 64), static_cast<cuuint32_t>(ps / 8)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  if (box[3] > 256) return set_error(MTN_EINVAL, "paged TMA map: page_size %d above 2048", ps);
  CUtensorMap m;
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, pool->base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled(paged pool) failed: %d", (int)r);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_pool_maps.size() > 256) g_pool_maps.clear();
  g_pool_maps[key] = m;
  *out = m;
  return MTN_OK;
}

int q_tensor_map(const void* q, int64_t total_q, int hq, int d, int box_rows, CUtensorMap* out) {
  auto enc = encoder();
  if (enc == nullptr) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(hq), static_cast<cuuint64_t>(total_q)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(hq) * d * 2};
  const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MTN_ECUDA, "cuTensorMapEncodeTiled(q) failed: %d", (int)r);
  return MTN_OK;
}

}  // namespace mtn
