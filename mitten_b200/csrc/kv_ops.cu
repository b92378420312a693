// Data-movement kernels of the paged-KV path:
//   - slot mapping  (Batch CSR -> per-token pool slot, batch.rs:7-36)
//   - KV append     (paged replacement of Tensor::cat, qwen model.rs:390-392)
//   - page copy     (copy-on-write / prefix fork; no reference counterpart)
//   - gather        (pages -> KVCacheState::Attention layout, model-common lib.rs:5-13)
//   - row argmax    (greedy sample_token, scheduler.rs:186-199)
// All are HBM-bound byte movers: 16-byte vector accesses, several loads in
// flight per thread before the matching stores, grids sized in multiples of
// the SM count.
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace mtn {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 1;     // vectors per thread per pass: measured best for these short, HBM-bound calls

int grid_for(int64_t work_items, int64_t items_per_block) {
  const int sms = sm_count();
  int64_t blocks = (work_items + items_per_block - 1) / items_per_block;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

// Largest r in [0, n) with offs[r] <= t (offs non-decreasing, offs[0] <= t).
__device__ __forceinline__ int upper_index(const int32_t* offs, int n, int64_t t) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ int upper_index64(const int64_t* offs, int n, int64_t t) {
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

__global__ void slot_mapping_kernel(const int32_t* __restrict__ qo_indptr, const int32_t* __restrict__ positions,
                                    const int32_t* __restrict__ kv_indptr, const int32_t* __restrict__ kv_indices,
                                    int n_seqs, int64_t n_tokens, int page_size, int64_t* __restrict__ slots,
                                    int* err) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n_tokens;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = upper_index(qo_indptr, n_seqs, t);
    const int pos = positions[t];
    const int pidx = pos >= 0 ? pos / page_size : -1;
    const int np = kv_indptr[r + 1] - kv_indptr[r];
    if (pos < 0 || pidx >= np) {
      slots[t] = -1;
      record_error(err, kDevErrBadPosition, static_cast<int>(t));
    } else {
      slots[t] = static_cast<int64_t>(kv_indices[kv_indptr[r] + pidx]) * page_size + (pos % page_size);
    }
  }
}

// One work item = 16 output bytes (8 bf16) of one (token, kv head) row of K
// and the same chunk of V.
template <typename SrcT>
__device__ __forceinline__ uint4 load_chunk(const SrcT* p);

template <>
__device__ __forceinline__ uint4 load_chunk<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

template <>
__device__ __forceinline__ uint4 load_chunk<float>(const float* p) {
  const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
  uint4 r;
  r.x = f2_to_bf2(a.x, a.y);
  r.y = f2_to_bf2(a.z, a.w);
  r.z = f2_to_bf2(b.x, b.y);
  r.w = f2_to_bf2(b.z, b.w);
  return r;
}

// Idx is the work-item index type: 32-bit when every index fits (the
// common case; a 64-bit division per 16 bytes would dominate the kernel).
// P2: hkv and head_dim / 8 are powers of two (lg_chunks, lg_per_tok their
// logs), so the work index splits with shifts instead of divisions.
template <typename SrcT, typename Idx, bool P2>
__global__ void __launch_bounds__(kThreads) kv_append_kernel(
    __nv_bfloat16* __restrict__ kdst, __nv_bfloat16* __restrict__ vdst, int64_t num_pages, int hkv, int ps,
    int d, const SrcT* __restrict__ k, const SrcT* __restrict__ v, int64_t src_stride,
    const int64_t* __restrict__ slots, int64_t n_tokens, int* err, int lg_chunks, int lg_per_tok) {
  pdl_enter();
  const int chunks = d >> 3;
  const Idx per_tok = static_cast<Idx>(hkv) * chunks;
  const Idx total = static_cast<Idx>(n_tokens) * per_tok;
  const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
  for (Idx base = blockIdx.x * static_cast<Idx>(blockDim.x) + threadIdx.x; base < total;
       base += stride * kUnroll) {
    uint4 kv[kUnroll], vv[kUnroll];
    int64_t dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const Idx i = base + u * stride;
      dst[u] = -1;
      if (i < total) {
        const Idx t = P2 ? (i >> lg_per_tok) : i / per_tok;
        const int rem = static_cast<int>(i - t * per_tok);
        const int h = P2 ? (rem >> lg_chunks) : rem / chunks;
        const int c = rem - h * chunks;
        const int64_t slot = slots[t];
        if (slot >= 0) {
          const int64_t page = slot / ps;
          const int off = static_cast<int>(slot - page * ps);
          if (page < num_pages) {
            const int64_t so = static_cast<int64_t>(t) * src_stride + static_cast<int64_t>(h) * d + c * 8;
            kv[u] = load_chunk<SrcT>(k + so);
            vv[u] = load_chunk<SrcT>(v + so);
            dst[u] = ((page * hkv + h) * ps + off) * static_cast<int64_t>(d) + c * 8;
          } else {
            record_error(err, kDevErrBadSlot, static_cast<int>(t));
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (dst[u] >= 0) {
        *reinterpret_cast<uint4*>(kdst + dst[u]) = kv[u];
        *reinterpret_cast<uint4*>(vdst + dst[u]) = vv[u];
      }
    }
  }
}

// One work item = 16 bytes of one (pair, layer, K|V) page block.
template <typename Idx>
__global__ void __launch_bounds__(kThreads) page_copy_kernel(__nv_bfloat16* __restrict__ pool, int64_t num_pages,
                                                             int num_layers, int64_t page_vecs,
                                                             const int32_t* __restrict__ src,
                                                             const int32_t* __restrict__ dst, int64_t n_pairs,
                                                             int* err) {
  pdl_enter();
  uint4* p4 = reinterpret_cast<uint4*>(pool);
  const Idx pv = static_cast<Idx>(page_vecs);
  const Idx units = static_cast<Idx>(n_pairs) * num_layers * 2;
  const Idx total = units * pv;
  const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
  for (Idx base = blockIdx.x * static_cast<Idx>(blockDim.x) + threadIdx.x; base < total;
       base += stride * kUnroll) {
    uint4 val[kUnroll];
    int64_t to[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const Idx i = base + u * stride;
      to[u] = -1;
      if (i < total) {
        const Idx unit = i / pv;
        const int64_t w = i - unit * pv;
        const Idx pair = unit / static_cast<Idx>(num_layers * 2);
        const int64_t lk = unit - pair * static_cast<Idx>(num_layers * 2);  // layer * 2 + kv
        const int64_t s = src[pair], t = dst[pair];
        if (s < 0 || s >= num_pages || t < 0 || t >= num_pages) {
          record_error(err, kDevErrBadPage, static_cast<int>(pair));
        } else if (s != t) {
          val[u] = p4[(lk * num_pages + s) * page_vecs + w];
          to[u] = (lk * num_pages + t) * page_vecs + w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (to[u] >= 0) p4[to[u]] = val[u];
    }
  }
}

// Page copy with 1-D bulk copies.  Every (pair, layer, K|V) unit is one
// contiguous slab of page_bytes at the source and the destination page.  A
// CTA (one warp) takes up to 32 consecutive units: its lanes fetch their
// units' page ids together, then lane 0 moves the slabs global -> shared ->
// global (cp.async.bulk both ways) through a ring of `slots` buffers, so up
// to `slots` slabs are in flight for a handful of instructions each.  A slot
// is reloaded once the store that read it two steps earlier has read its
// source (bulk_wait_read<2>), so loads run slots - 2 units ahead.
constexpr int kCopyMaxSlots = 8;
constexpr int kCopyLag = 2;
constexpr int kCopyUnitsPerCta = 32;
constexpr int64_t kCopyBulkMaxBytes = 16384;  // larger slabs take the vector kernel

__global__ void __launch_bounds__(32) page_copy_bulk_kernel(uint8_t* __restrict__ pool, int64_t num_pages,
                                                           int num_layers, int64_t page_bytes,
                                                           const int32_t* __restrict__ src,
                                                           const int32_t* __restrict__ dst, int64_t n_pairs,
                                                           int units_per_cta, int slots, int* err) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int64_t from_s[kCopyUnitsPerCta], to_s[kCopyUnitsPerCta];  // byte offsets, -1 = nothing to copy
  const int lane = threadIdx.x;
  const int64_t per_pair = static_cast<int64_t>(num_layers) * 2;
  const int64_t units = n_pairs * per_pair;
  const int64_t u0 = static_cast<int64_t>(blockIdx.x) * units_per_cta;
  const int n = static_cast<int>(u0 < units ? std::min<int64_t>(units_per_cta, units - u0) : 0);
  if (lane < n) {
    const int64_t u = u0 + lane;
    const int64_t pair = u / per_pair, lk = u - pair * per_pair;  // lk = layer * 2 + (K|V)
    const int64_t s = src[pair], t = dst[pair];
    from_s[lane] = -1;
    to_s[lane] = -1;
    if (s < 0 || s >= num_pages || t < 0 || t >= num_pages) {
      record_error(err, kDevErrBadPage, static_cast<int>(pair));
    } else if (s != t) {
      from_s[lane] = (lk * num_pages + s) * page_bytes;
      to_s[lane] = (lk * num_pages + t) * page_bytes;
    }
  }
  __syncwarp();
  if (lane != 0) return;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);  // [kCopyMaxSlots]
  uint8_t* buf = smem_raw + 128;
  for (int k = 0; k < slots; ++k) mbar_init(&full[k], 1);
  fence_barrier_init();
  auto load = [&](int i) {  // unit i of this CTA into slot i % slots
    const int k = i % slots;
    if (to_s[i] >= 0) {
      mbar_arrive_expect_tx(&full[k], static_cast<uint32_t>(page_bytes));
      bulk_g2s(buf + k * page_bytes, pool + from_s[i], static_cast<uint32_t>(page_bytes), &full[k]);
    } else {
      mbar_arrive_plain(&full[k]);  // nothing to copy: complete the slot's phase without bytes
    }
  };
  int loaded = 0;  // units whose load is issued
  for (; loaded < n && loaded < slots; ++loaded) load(loaded);
  for (int j = 0; j < n; ++j) {
    const int k = j % slots;
    if (!mbar_wait_bounded(&full[k], static_cast<uint32_t>((j / slots) & 1), err, 40)) {
      // Gave up (error recorded): wait, bounded, for the other loads still
      // in flight into this CTA's shared memory before leaving.
      for (int i = j + 1; i < loaded; ++i)
        mbar_wait_bounded(&full[i % slots], static_cast<uint32_t>((i / slots) & 1), err, 41);
      break;
    }
    if (to_s[j] >= 0) bulk_s2g(pool + to_s[j], buf + k * page_bytes, static_cast<uint32_t>(page_bytes));
    bulk_commit_group();  // one group per step, empty for skipped units, so the lag counts steps
    const int r = j - kCopyLag + slots;  // the unit that reuses slot (j - kCopyLag) % slots
    if (j >= kCopyLag && r < n) {
      bulk_wait_read<kCopyLag>();
      load(r);
      loaded = r + 1;
    }
  }
  bulk_wait_all();
}

// Pages between the pool and a flat buffer [n_pages][layers][2 (K, V)]
// [page_vecs x 16 bytes] (KV offload and prefill -> decode handoff):
// kUnpack false copies pool -> buffer, true buffer -> pool.  The buffer may
// be device memory, pinned host memory or a peer GPU's memory.
template <typename Idx, bool kUnpack>
__global__ void __launch_bounds__(kThreads) page_xfer_kernel(__nv_bfloat16* __restrict__ pool, int64_t num_pages,
                                                             int num_layers, int64_t page_vecs,
                                                             const int32_t* __restrict__ pages, int64_t n_pages,
                                                             uint4* __restrict__ buf, int* err) {
  uint4* p4 = reinterpret_cast<uint4*>(pool);
  const Idx pv = static_cast<Idx>(page_vecs);
  const Idx total = static_cast<Idx>(n_pages) * num_layers * 2 * pv;
  const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
  for (Idx base = blockIdx.x * static_cast<Idx>(blockDim.x) + threadIdx.x; base < total;
       base += stride * kUnroll) {
    uint4 val[kUnroll];
    int64_t at[kUnroll];  // pool vector of element u, -1 = skip
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const Idx i = base + u * stride;
      at[u] = -1;
      if (i < total) {
        const Idx unit = i / pv;
        const int64_t w = i - unit * pv;
        const Idx pair = unit / static_cast<Idx>(num_layers * 2);
        const int64_t lk = unit - pair * static_cast<Idx>(num_layers * 2);  // layer * 2 + kv
        const int64_t pg = pages[pair];
        if (pg < 0 || pg >= num_pages) {
          record_error(err, kDevErrBadPage, static_cast<int>(pair));
        } else {
          at[u] = (lk * num_pages + pg) * page_vecs + w;
          val[u] = kUnpack ? buf[i] : p4[at[u]];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (at[u] < 0) continue;
      if (kUnpack) p4[at[u]] = val[u];
      else buf[base + u * stride] = val[u];
    }
  }
}

// One work item = 16 bytes (8 elements) of one (token, kv head) row.
__global__ void __launch_bounds__(kThreads) gather_kernel(
    const __nv_bfloat16* __restrict__ kpool, const __nv_bfloat16* __restrict__ vpool, int64_t num_pages, int hkv,
    int ps, int d, const int32_t* __restrict__ kv_indptr, const int32_t* __restrict__ kv_indices,
    const int32_t* __restrict__ seq_lens, const int64_t* __restrict__ out_offsets, int n_seqs,
    __nv_bfloat16* __restrict__ out_k, __nv_bfloat16* __restrict__ out_v, int64_t total_tokens, int* err) {
  const int chunks = d >> 3;
  const int64_t per_tok = static_cast<int64_t>(hkv) * chunks;
  const int64_t total = total_tokens * per_tok;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / per_tok;
    const int rem = static_cast<int>(i - t * per_tok);
    const int h = rem / chunks;
    const int c = rem - h * chunks;
    const int r = upper_index64(out_offsets, n_seqs, t);
    const int64_t j = t - out_offsets[r];
    const int len = seq_lens[r];
    if (j >= len) continue;
    const int pidx = static_cast<int>(j / ps);
    if (pidx >= kv_indptr[r + 1] - kv_indptr[r]) {
      record_error(err, kDevErrBadSeqLen, r);
      continue;
    }
    const int64_t page = kv_indices[kv_indptr[r] + pidx];
    if (page < 0 || page >= num_pages) {
      record_error(err, kDevErrBadPage, r);
      continue;
    }
    const int64_t src = ((page * hkv + h) * ps + (j - static_cast<int64_t>(pidx) * ps)) * d + c * 8;
    const int64_t dst = (out_offsets[r] * hkv + static_cast<int64_t>(h) * len + j) * d + c * 8;
    *reinterpret_cast<uint4*>(out_k + dst) = *reinterpret_cast<const uint4*>(kpool + src);
    *reinterpret_cast<uint4*>(out_v + dst) = *reinterpret_cast<const uint4*>(vpool + src);
  }
}

// First strict maximum of each row, NaN never wins (scheduler.rs:188-199:
// `if val > max_val` starting from -inf at index 0).
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int64_t vocab,
                                                      int32_t* __restrict__ out) {
  const float* row = logits + blockIdx.x * vocab;
  float best = -INFINITY;
  int64_t idx = INT64_MAX;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float x = row[i];
    if (x > best) { best = x; idx = i; }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if (lane == 0) out[blockIdx.x] = (best == -INFINITY || idx == INT64_MAX) ? 0 : static_cast<int32_t>(idx);
  }
}

int check_layout(const mtn_kv_layout* pool, int layer, const char* who) {
  MTN_CHECK_ARG(pool != nullptr && pool->base != nullptr, "%s: null pool", who);
  MTN_CHECK_ARG(pool->num_pages > 0 && pool->num_layers > 0 && pool->page_size > 0 && pool->num_kv_heads > 0,
                "%s: non-positive pool dimension", who);
  MTN_CHECK_ARG(pool->head_dim == 64 || pool->head_dim == 128 || pool->head_dim == 256,
                "%s: head_dim %d not in {64,128,256}", who, pool->head_dim);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(pool->base) & 255) == 0, "%s: pool base not 256-byte aligned", who);
  MTN_CHECK_ARG(layer >= 0 && layer < pool->num_layers, "%s: layer %d outside [0,%d)", who, layer, pool->num_layers);
  return MTN_OK;
}

}  // namespace

int validate_layout(const mtn_kv_layout* pool, int layer, const char* who) { return check_layout(pool, layer, who); }

}  // namespace mtn

using mtn::set_error;

namespace mtn {
namespace {

template <bool kUnpack>
int pages_xfer(const mtn_kv_layout* pool, const int32_t* pages, int64_t n_pages, void* buf, void* stream,
               const char* who) {
  int st = check_layout(pool, 0, who);
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_pages >= 0, "%s: n_pages < 0", who);
  if (n_pages == 0) return MTN_OK;
  MTN_CHECK_ARG(pages && buf, "%s: null pointer", who);
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(buf) & 15) == 0, "%s: buffer must be 16-byte aligned", who);
  const int64_t page_vecs = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * pool->head_dim / 8;
  const int64_t work = n_pages * pool->num_layers * 2 * page_vecs;
  const int grid = grid_for(work, kThreads * kUnroll);
  const bool narrow = work + static_cast<int64_t>(grid) * kThreads * kUnroll < (int64_t(1) << 31);
  auto* base = static_cast<__nv_bfloat16*>(pool->base);
  auto* b4 = static_cast<uint4*>(buf);
  auto s = static_cast<cudaStream_t>(stream);
  if (narrow)
    page_xfer_kernel<uint32_t, kUnpack><<<grid, kThreads, 0, s>>>(
        base, pool->num_pages, pool->num_layers, page_vecs, pages, n_pages, b4, device_error_ptr());
  else
    page_xfer_kernel<int64_t, kUnpack><<<grid, kThreads, 0, s>>>(
        base, pool->num_pages, pool->num_layers, page_vecs, pages, n_pages, b4, device_error_ptr());
  return check_launch("page_xfer_kernel");
}

}  // namespace
}  // namespace mtn

extern "C" {

int mtn_build_slot_mapping(const int32_t* qo_indptr, const int32_t* positions, const int32_t* kv_indptr,
                           const int32_t* kv_indices, int32_t n_seqs, int64_t n_tokens, int32_t page_size,
                           int64_t* slots, void* stream) {
  MTN_CHECK_ARG(n_seqs >= 0 && n_tokens >= 0 && page_size > 0, "mtn_build_slot_mapping: bad sizes");
  if (n_tokens == 0) return MTN_OK;
  MTN_CHECK_ARG(n_seqs > 0, "mtn_build_slot_mapping: tokens without sequences");
  MTN_CHECK_ARG(qo_indptr && positions && kv_indptr && kv_indices && slots, "mtn_build_slot_mapping: null pointer");
  const int grid = mtn::grid_for(n_tokens, mtn::kThreads);
  mtn::slot_mapping_kernel<<<grid, mtn::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      qo_indptr, positions, kv_indptr, kv_indices, n_seqs, n_tokens, page_size, slots, mtn::device_error_ptr());
  return mtn::check_launch("slot_mapping_kernel");
}

int mtn_kv_append(const mtn_kv_layout* pool, int32_t layer, const void* k, const void* v, int32_t src_dtype,
                  int64_t src_stride, const int64_t* slots, int64_t n_tokens, void* stream) {
  int st = mtn::check_layout(pool, layer, "mtn_kv_append");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_tokens >= 0, "mtn_kv_append: n_tokens < 0");
  if (n_tokens == 0) return MTN_OK;
  MTN_CHECK_ARG(k && v && slots, "mtn_kv_append: null pointer");
  const int64_t row = static_cast<int64_t>(pool->num_kv_heads) * pool->head_dim;
  MTN_CHECK_ARG(src_stride >= row, "mtn_kv_append: src_stride %lld < heads*dim %lld", (long long)src_stride,
                (long long)row);
  MTN_CHECK_ARG(src_dtype == MTN_DTYPE_BF16 || src_dtype == MTN_DTYPE_F32, "mtn_kv_append: bad src dtype");
  const int esz = src_dtype == MTN_DTYPE_BF16 ? 2 : 4;
  MTN_CHECK_ARG((reinterpret_cast<uintptr_t>(k) % 16) == 0 && (reinterpret_cast<uintptr_t>(v) % 16) == 0 &&
                    (src_stride * esz) % 16 == 0,
                "mtn_kv_append: k/v rows must be 16-byte aligned");
  const int64_t page_elems = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * pool->head_dim;
  auto* base = static_cast<__nv_bfloat16*>(pool->base);
  __nv_bfloat16* kd = base + (static_cast<int64_t>(layer) * 2 + 0) * pool->num_pages * page_elems;
  __nv_bfloat16* vd = base + (static_cast<int64_t>(layer) * 2 + 1) * pool->num_pages * page_elems;
  const int64_t work = n_tokens * pool->num_kv_heads * (pool->head_dim / 8);
  const int grid = mtn::grid_for(work, mtn::kThreads * mtn::kUnroll);
  auto s = static_cast<cudaStream_t>(stream);
  // 32-bit work indices while every index (plus one grid stride) stays below 2^31.
  const bool narrow = work + static_cast<int64_t>(grid) * mtn::kThreads * mtn::kUnroll < (int64_t(1) << 31);
  const int chunks = pool->head_dim / 8;
  const int per_tok = pool->num_kv_heads * chunks;
  const bool p2 = (chunks & (chunks - 1)) == 0 && (per_tok & (per_tok - 1)) == 0;
  const int lg_c = p2 ? __builtin_ctz(static_cast<unsigned>(chunks)) : 0;
  const int lg_t = p2 ? __builtin_ctz(static_cast<unsigned>(per_tok)) : 0;
#define MTN_APPEND_LAUNCH(SRC, IDX, P2F, KP, VP)                                                               \
  return mtn::launch_pdl(mtn::kv_append_kernel<SRC, IDX, P2F>, dim3(grid), dim3(mtn::kThreads), 0, s,           \
                         "kv_append_kernel", kd, vd, pool->num_pages, pool->num_kv_heads, pool->page_size,       \
                         pool->head_dim, KP, VP, src_stride, slots, n_tokens, mtn::device_error_ptr(), lg_c, lg_t)
  if (src_dtype == MTN_DTYPE_BF16) {
    auto kb = static_cast<const __nv_bfloat16*>(k);
    auto vb = static_cast<const __nv_bfloat16*>(v);
    if (narrow && p2) MTN_APPEND_LAUNCH(__nv_bfloat16, uint32_t, true, kb, vb);
    else if (narrow) MTN_APPEND_LAUNCH(__nv_bfloat16, uint32_t, false, kb, vb);
    else MTN_APPEND_LAUNCH(__nv_bfloat16, int64_t, false, kb, vb);
  } else {
    auto kf = static_cast<const float*>(k);
    auto vf = static_cast<const float*>(v);
    if (narrow && p2) MTN_APPEND_LAUNCH(float, uint32_t, true, kf, vf);
    else if (narrow) MTN_APPEND_LAUNCH(float, uint32_t, false, kf, vf);
    else MTN_APPEND_LAUNCH(float, int64_t, false, kf, vf);
  }
#undef MTN_APPEND_LAUNCH
  return mtn::check_launch("kv_append_kernel");
}

int mtn_page_copy(const mtn_kv_layout* pool, const int32_t* src_pages, const int32_t* dst_pages, int64_t n_pages,
                  void* stream) {
  int st = mtn::check_layout(pool, 0, "mtn_page_copy");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_pages >= 0, "mtn_page_copy: n_pages < 0");
  if (n_pages == 0) return MTN_OK;
  MTN_CHECK_ARG(src_pages && dst_pages, "mtn_page_copy: null pointer");
  const int64_t page_vecs = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * pool->head_dim / 8;
  const int64_t work = n_pages * pool->num_layers * 2 * page_vecs;
  const int grid = mtn::grid_for(work, mtn::kThreads * mtn::kUnroll);
  const bool narrow = work + static_cast<int64_t>(grid) * mtn::kThreads * mtn::kUnroll < (int64_t(1) << 31);
  auto* base = static_cast<__nv_bfloat16*>(pool->base);
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t page_bytes = page_vecs * 16;
  if (page_bytes <= mtn::kCopyBulkMaxBytes) {
    // Bulk path: ring slots of whole slabs, about 32 KB of shared memory per CTA.
    const int slots = static_cast<int>(std::min<int64_t>(mtn::kCopyMaxSlots, std::max<int64_t>(4, 32768 / page_bytes)));
    const int smem = 128 + slots * static_cast<int>(page_bytes);
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      MTN_CUDA_TRY(cudaFuncSetAttribute(mtn::page_copy_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        128 + mtn::kCopyMaxSlots * mtn::kCopyBulkMaxBytes),
                   "cudaFuncSetAttribute(page_copy_bulk_kernel)");
      configured[dev] = true;
    }
    // Units spread over the resident CTAs (up to 32 each; more CTAs queue).
    const int64_t units = n_pages * pool->num_layers * 2;
    const int per_sm = std::max(1, std::min(8, (200 * 1024) / smem));
    const int64_t resident = static_cast<int64_t>(mtn::sm_count()) * per_sm;
    const int upc = static_cast<int>(
        std::min<int64_t>(mtn::kCopyUnitsPerCta, std::max<int64_t>(1, (units + resident - 1) / resident)));
    const int64_t grid = (units + upc - 1) / upc;
    MTN_CHECK_ARG(grid < (int64_t(1) << 31), "mtn_page_copy: %lld pages too many", static_cast<long long>(n_pages));
    return mtn::launch_pdl(mtn::page_copy_bulk_kernel, dim3(static_cast<unsigned>(grid)), dim3(32),
                           static_cast<size_t>(smem), s, "page_copy_bulk_kernel", reinterpret_cast<uint8_t*>(base),
                           pool->num_pages, pool->num_layers, page_bytes, src_pages, dst_pages, n_pages, upc, slots,
                           mtn::device_error_ptr());
  }
  if (narrow)
    return mtn::launch_pdl(mtn::page_copy_kernel<uint32_t>, dim3(grid), dim3(mtn::kThreads), 0, s, "page_copy_kernel",
                           base, pool->num_pages, pool->num_layers, page_vecs, src_pages, dst_pages, n_pages,
                           mtn::device_error_ptr());
  return mtn::launch_pdl(mtn::page_copy_kernel<int64_t>, dim3(grid), dim3(mtn::kThreads), 0, s, "page_copy_kernel",
                         base, pool->num_pages, pool->num_layers, page_vecs, src_pages, dst_pages, n_pages,
                         mtn::device_error_ptr());
}

size_t mtn_kv_pages_bytes(const mtn_kv_layout* pool, int64_t n_pages) {
  if (pool == nullptr || n_pages <= 0) return 0;
  return static_cast<size_t>(n_pages) * pool->num_layers * 2 * pool->num_kv_heads * pool->page_size * pool->head_dim * 2;
}

int mtn_kv_pages_pack(const mtn_kv_layout* pool, const int32_t* pages, int64_t n_pages, void* dst, void* stream) {
  return mtn::pages_xfer<false>(pool, pages, n_pages, dst, stream, "mtn_kv_pages_pack");
}

int mtn_kv_pages_unpack(const mtn_kv_layout* pool, const void* src, const int32_t* pages, int64_t n_pages,
                        void* stream) {
  return mtn::pages_xfer<true>(pool, pages, n_pages, const_cast<void*>(src), stream, "mtn_kv_pages_unpack");
}

int mtn_kv_gather(const mtn_kv_layout* pool, int32_t layer, const int32_t* kv_indptr, const int32_t* kv_indices,
                  const int32_t* seq_lens, const int64_t* out_offsets, int32_t n_seqs, void* out_k, void* out_v,
                  int64_t total_tokens, void* stream) {
  int st = mtn::check_layout(pool, layer, "mtn_kv_gather");
  if (st != MTN_OK) return st;
  MTN_CHECK_ARG(n_seqs >= 0 && total_tokens >= 0, "mtn_kv_gather: bad sizes");
  if (total_tokens == 0 || n_seqs == 0) return MTN_OK;
  MTN_CHECK_ARG(kv_indptr && kv_indices && seq_lens && out_offsets && out_k && out_v, "mtn_kv_gather: null pointer");
  const int64_t page_elems = static_cast<int64_t>(pool->num_kv_heads) * pool->page_size * pool->head_dim;
  auto* base = static_cast<const __nv_bfloat16*>(pool->base);
  const __nv_bfloat16* kp = base + (static_cast<int64_t>(layer) * 2 + 0) * pool->num_pages * page_elems;
  const __nv_bfloat16* vp = base + (static_cast<int64_t>(layer) * 2 + 1) * pool->num_pages * page_elems;
  const int64_t work = total_tokens * pool->num_kv_heads * (pool->head_dim / 8);
  const int grid = mtn::grid_for(work, mtn::kThreads);
  mtn::gather_kernel<<<grid, mtn::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      kp, vp, pool->num_pages, pool->num_kv_heads, pool->page_size, pool->head_dim, kv_indptr, kv_indices, seq_lens,
      out_offsets, n_seqs, static_cast<__nv_bfloat16*>(out_k), static_cast<__nv_bfloat16*>(out_v), total_tokens,
      mtn::device_error_ptr());
  return mtn::check_launch("gather_kernel");
}

int mtn_argmax_rows(const float* logits, int64_t n_rows, int64_t vocab, int32_t* out, void* stream) {
  MTN_CHECK_ARG(n_rows >= 0 && vocab > 0 && vocab <= INT32_MAX, "mtn_argmax_rows: bad sizes");
  if (n_rows == 0) return MTN_OK;
  MTN_CHECK_ARG(logits && out, "mtn_argmax_rows: null pointer");
  MTN_CHECK_ARG(n_rows <= INT32_MAX, "mtn_argmax_rows: too many rows");
  mtn::argmax_kernel<<<static_cast<unsigned>(n_rows), 1024, 0, static_cast<cudaStream_t>(stream)>>>(logits, vocab,
                                                                                                    out);
  return mtn::check_launch("argmax_kernel");
}

}  // extern "C"
