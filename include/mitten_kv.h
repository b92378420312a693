/*
 * mitten_kv.h -- C ABI of the B200 (sm_100a) paged-KV library.
 *
 * One shared library (libmitten_kv.so) exports everything below.  Plain C:
 * opaque handles, plain pointers and sizes, int status codes, no callbacks,
 * no exceptions across the boundary.  Every device-pointer argument is
 * caller-owned and must stay alive until the given stream reaches the call.
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *
 * Reference interfaces replaced (paths inside tianhaoz95/mitten):
 *   - page pool / allocator ........ inference-engine/src/kv_pool.rs:4-69
 *   - radix prefix cache ........... inference-engine/src/radix_cache.rs:37-303
 *   - admission / chunked prefill .. inference-engine/src/prefill.rs:6-115
 *   - decode collection ............ inference-engine/src/decode.rs:6-47
 *   - batch assembly / transition .. inference-engine/src/scheduler.rs:8-223
 *   - Batch record ................. inference-backend/src/batch.rs:7-36
 *   - BackendHandle::forward ....... inference-backend/src/backend.rs:16-21,
 *                                    inference-backend/src/burn_backend.rs:31-80
 *   - KVCacheState::Attention ...... inference-model-common/src/lib.rs:5-13
 *   - KV append (Tensor::cat) ...... inference-model-qwen/src/model.rs:390-392
 *   - attention core ............... inference-model-qwen/src/model.rs:394-416
 *   - causal mask .................. inference-model-qwen/src/model.rs:542-555
 *   - phantom zero KV row .......... inference-model-qwen/src/model.rs:207-220
 *
 * Status codes map onto inference-backend/src/error.rs:3-13:
 *   MTN_ENOMEM -> EngineError::OutOfKvPages; every other non-zero code ->
 *   EngineError::Backend(mtn_last_error()).
 */
#ifndef MITTEN_KV_H
#define MITTEN_KV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MTN_API __attribute__((visibility("default")))
#else
#define MTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status and errors                                                        */
/* ------------------------------------------------------------------------ */

enum {
  MTN_OK = 0,
  MTN_EINVAL = 1,    /* invalid argument; nothing was launched            */
  MTN_ENOMEM = 2,    /* out of KV pages (or of device memory)            */
  MTN_ECUDA = 3,     /* CUDA runtime error                                */
  MTN_ETIMEOUT = 4,  /* a bounded device-side wait ran out                */
  MTN_EDEVICE = 5    /* a kernel flagged bad metadata (see device error)  */
};

/* Message for the last non-zero status returned on the calling thread.
 * Replaces the String inside EngineError::Backend (error.rs:5). */
MTN_API const char* mtn_last_error(void);
MTN_API const char* mtn_version(void);

/* Device-side error word written by kernels that meet out-of-range metadata
 * (page id >= num_pages, seq_len beyond its pages, ...).  Kernels never trap:
 * they clamp, finish, and record the first error here.  Reading it
 * synchronises `device`.  Returns MTN_OK and stores the code (0 = none)
 * and the kernel-specific detail word; `clear` resets it.  Codes: 1 page id
 * outside the pool, 2 seq_len negative or beyond its pages, 3 slot outside
 * the pool, 4 a bounded wait ran out, 5 position beyond a sequence's pages,
 * 6 a decode plan made for another grid or not a plan. */
MTN_API int mtn_device_error(int device, int clear, int32_t* code, int32_t* detail);

/* Self-test of the bounded device waits (failure detection without a GPU
 * fault): launches one block on `stream` whose mbarrier wait nothing
 * completes.  After ~1 s the wait gives up, records device error 4
 * (timeout) with detail 99 in the word mtn_device_error reads, and the
 * kernel returns normally: no trap, the context stays usable. */
MTN_API int mtn_selftest_bounded_wait(void* stream);

/* ------------------------------------------------------------------------ */
/* Device KV pool layout                                                    */
/* ------------------------------------------------------------------------ */

/* Pool memory: bf16 [num_layers][2 (K,V)][num_pages][num_kv_heads][page_size][head_dim].
 * One page of one layer is the [num_kv_heads, page_size, head_dim] slice of
 * the reference's per-request KVCacheState::Attention tensor
 * [1, heads, seq, head_dim] (model-common lib.rs:5-13), so each
 * (page, kv head) is one contiguous page_size*head_dim*2-byte slab. */
typedef struct {
  void* base;            /* device pointer, 256-byte aligned               */
  int64_t num_pages;
  int32_t num_layers;
  int32_t page_size;     /* tokens per page                                */
  int32_t num_kv_heads;
  int32_t head_dim;      /* 64, 128 or 256                                 */
} mtn_kv_layout;

/* KvCachePool::required_bytes (kv_pool.rs:58-68):
 * 2 * num_layers * num_pages * page_size * num_kv_heads * head_dim * dtype_bytes. */
MTN_API size_t mtn_kv_required_bytes(int64_t num_pages, int64_t page_size, int64_t num_layers,
                             int64_t num_kv_heads, int64_t head_dim, int64_t dtype_bytes);

/* Allocate (cudaMalloc on `device`) and zero a pool; fills `out`.  The
 * caller may instead point `base` at its own allocation of
 * mtn_kv_required_bytes(..., 2) bytes. */
MTN_API int mtn_kv_pool_alloc(int device, mtn_kv_layout* out);
MTN_API int mtn_kv_pool_free(mtn_kv_layout* pool);

/* Element offset helpers (host-side, no device access). */
MTN_API int64_t mtn_kv_page_offset(const mtn_kv_layout* pool, int32_t layer, int32_t kv, int64_t page);

/* ------------------------------------------------------------------------ */
/* Kernels                                                                  */
/* ------------------------------------------------------------------------ */

enum {
  MTN_DTYPE_BF16 = 0,
  MTN_DTYPE_F32 = 1
};

/* Attention flags. */
enum {
  /* Add the reference's all-zero first K/V row (qwen model.rs:207-220) to
   * every softmax: one key with score 0 and a zero value. */
  MTN_ATTN_PHANTOM_ZERO_SLOT = 1u << 0,
  /* mtn_paged_prefill only: run the one-query-tile kernel even where the
   * two-tile kernel applies (head_dim <= 128 and at least two query tiles
   * per SM); same results, for comparison. */
  MTN_ATTN_PREFILL_ONE_TILE = 1u << 1,
  /* Split the tensor-core operands Q and P into bf16 hi + lo pairs
   * (hi = bf16(x), lo = bf16(x - hi)) and accumulate both products in f32,
   * so f32 queries and the softmax weights keep about 16 significant bits
   * (the reference computes q.k and P.v in f32, model.rs:413-416).  K and
   * V are the pool's bf16 values either way.  Decode: no extra tensor-core
   * work (the lo rows fill the padding of the 16-wide query-head operand).
   * Prefill: twice the tensor-core work; head_dim <= 128; always the
   * one-query-tile kernel. */
  MTN_ATTN_SPLIT_BF16 = 1u << 2
};

/* Per-token pool slot for a batch (Batch -> slot map; batch.rs:7-36):
 *   token t of sequence r (qo_indptr[r] <= t < qo_indptr[r+1]) at absolute
 *   position positions[t] goes to
 *   slot = kv_indices[kv_indptr[r] + pos / page_size] * page_size + pos % page_size.
 * Positions past a sequence's pages give slot -1 and a device error. */
MTN_API int mtn_build_slot_mapping(const int32_t* qo_indptr, const int32_t* positions,
                           const int32_t* kv_indptr, const int32_t* kv_indices,
                           int32_t n_seqs, int64_t n_tokens, int32_t page_size,
                           int64_t* slots, void* stream);

/* KV append: the paged replacement for the per-layer Tensor::cat of
 * qwen model.rs:390-392.  k/v: [n_tokens][num_kv_heads][head_dim], element
 * type `src_dtype` (bf16 copied bit-exact, f32 rounded to nearest even),
 * token rows `src_stride` elements apart (>= num_kv_heads*head_dim; lets a
 * caller pass a slice of a fused QKV projection).  slot < 0 skips a token. */
MTN_API int mtn_kv_append(const mtn_kv_layout* pool, int32_t layer,
                  const void* k, const void* v, int32_t src_dtype, int64_t src_stride,
                  const int64_t* slots, int64_t n_tokens, void* stream);

/* Page copy for copy-on-write and prefix forks: for i < n_pages copy page
 * src[i] onto page dst[i] in every layer, K and V, every head.  Pairs with
 * src[i] == dst[i] are skipped; a page id outside the pool is recorded as
 * device error 1 (detail = i) and its pair skipped.  Pages of up to 16 KB
 * per (layer, K|V) move as whole slabs with 1-D bulk copies. */
MTN_API int mtn_page_copy(const mtn_kv_layout* pool, const int32_t* src_pages,
                  const int32_t* dst_pages, int64_t n_pages, void* stream);

/* KV offload and prefill -> decode handoff (the reference designs these
 * without code: KvOffloadManager's host KV buffers, design/phase1-
 * deliverable.md:253-337, and the disaggregation KvHandoff of request id,
 * pages and cached length, design/phase2b-deliverable.md:272-354): the
 * listed pages (device array of page ids) of every layer, K and V, to or
 * from a flat buffer laid out [n_pages][num_layers][2][num_kv_heads]
 * [page_size][head_dim] bf16, mtn_kv_pages_bytes(pool, n_pages) bytes,
 * 16-byte aligned: device memory, pinned host memory the device can reach
 * (offload), or another GPU's memory under peer access (handoff between
 * replicas).  Page ids outside the pool are skipped and flagged (device
 * error 1). */
MTN_API size_t mtn_kv_pages_bytes(const mtn_kv_layout* pool, int64_t n_pages);
MTN_API int mtn_kv_pages_pack(const mtn_kv_layout* pool, const int32_t* pages, int64_t n_pages, void* dst,
                              void* stream);
MTN_API int mtn_kv_pages_unpack(const mtn_kv_layout* pool, const void* src, const int32_t* pages,
                                int64_t n_pages, void* stream);

/* Fused attention prologue (the per-head work of qwen model.rs:372-392
 * between the projection GEMMs and attention), one launch for every token
 * row of a batch: q = RoPE(RMSNorm_(1+w)(q head)) written to q_out
 * [n_tokens][num_q_heads][head_dim] f32; k = RoPE(RMSNorm_(1+w)(k head)) and
 * v stored as bf16 (round to nearest even) into the pool at slots[t]
 * (page * page_size + offset; < 0 skips the token's K/V).  q / k / v:
 * src_dtype rows q_stride / k_stride / v_stride elements apart (a slice of a
 * fused projection is fine); q rows are [num_q_heads][1 + q_gated][head_dim]
 * (q then its gate per head, model.rs:372-375; the gate is left for the
 * caller).  q_norm_w1 / k_norm_w1: (1 + w) per element, or NULL for no
 * norm (Gemma).  RoPE: rotate-half over the first rotary_dim elements
 * (a multiple of 64), angle = positions[t] * inv_freq[i] in f32.  With
 * the step's rows stored here, mtn_paged_decode runs without k_new / v_new. */
MTN_API int mtn_qkv_prologue(const mtn_kv_layout* pool, int32_t layer, const void* q, const void* k, const void* v,
                             int32_t src_dtype, int64_t q_stride, int64_t k_stride, int64_t v_stride,
                             int32_t q_gated, int32_t num_q_heads, const float* q_norm_w1, const float* k_norm_w1,
                             float eps, const float* inv_freq, int32_t rotary_dim, const int32_t* positions,
                             const int64_t* slots, int64_t n_tokens, float* q_out, void* stream);

/* Gather sequences back into the reference's contiguous cache layout
 * KVCacheState::Attention [num_kv_heads][seq_len][head_dim] (bf16):
 * sequence r lands at out + out_offsets[r]*num_kv_heads*head_dim, where
 * out_offsets is the exclusive prefix sum of seq_lens. */
MTN_API int mtn_kv_gather(const mtn_kv_layout* pool, int32_t layer,
                  const int32_t* kv_indptr, const int32_t* kv_indices,
                  const int32_t* seq_lens, const int64_t* out_offsets, int32_t n_seqs,
                  void* out_k, void* out_v, int64_t total_tokens, void* stream);

/* Paged decode attention (one query token per sequence) with the step's KV
 * append fused in (tcgen05 tensor cores, persistent split-KV).
 *   q: [n_seqs][num_q_heads][head_dim] (q_dtype), o: same shape (o_dtype).
 *   Sequence r reads pages kv_indices[kv_indptr[r] .. kv_indptr[r+1]) and its
 *   first seq_lens[r] tokens.
 *   k_new / v_new (both or neither; new_dtype): [n_seqs][num_kv_heads][head_dim]
 *   rows of the token each sequence appends this step.  When given, the
 *   kernel first stores them at position seq_lens[r]-1 (the paged form of
 *   the Tensor::cat at qwen model.rs:390-392), then attends over them; when
 *   NULL the cache must already hold seq_lens[r] tokens.
 *   q head h uses kv head h / (num_q_heads / num_kv_heads) (model.rs:398-408),
 *   at most 8 query heads per kv head.  scale multiplies q.k (model.rs:298, 413).
 *   workspace: mtn_paged_decode_workspace_bytes(...) bytes, zeroed once before
 *   first use (calls leave it reusable; after a call that reports a device
 *   timeout, mtn_device_error code 4, zero it again); concurrent calls must
 *   not share one.
 *   Programmatic dependent launch: a decode launch lets the next kernel of
 *   its stream start early, and itself may start while the previous kernel
 *   of the stream finishes; before waiting for that kernel it reads only
 *   kv_indptr and seq_lens, which therefore must not be written by a kernel
 *   that itself allows early launch (no kernel of this library writes them).
 *   The pool memory must have been zero-initialised (mtn_kv_pool_alloc does). */
MTN_API size_t mtn_paged_decode_workspace_bytes(int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                                        int32_t head_dim);
MTN_API int mtn_paged_decode(const mtn_kv_layout* pool, int32_t layer,
                     const void* q, int32_t q_dtype, void* o, int32_t o_dtype,
                     const void* k_new, const void* v_new, int32_t new_dtype,
                     int32_t n_seqs, int32_t num_q_heads,
                     const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens,
                     float scale, uint32_t flags,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Work plan for mtn_paged_decode_with_plan (no counterpart in the reference,
 * whose decode runs per request on the CPU).  Made on the host from the
 * batch's host-side CSR metadata (the scheduler builds it there every step;
 * every layer of a step shares one plan): the launch's (sequence, kv head)
 * segments are cut into 128-token tiles laid end to end, and each CTA of the
 * persistent grid gets a contiguous range of equal cost -- a tile costs 8, a
 * segment start 16 more -- plus its start sequence, so the kernel's first
 * loads need one read of the plan instead of a scan of seq_lens.  plan:
 * host memory of mtn_paged_decode_plan_bytes(head_dim) bytes; copy it to the
 * device (16-byte aligned) before the launch that uses it.  The plan holds
 * the device's SM count: a plan made on another GPU model is rejected by the
 * kernel (device error 6, nothing computed). */
MTN_API size_t mtn_paged_decode_plan_bytes(int32_t head_dim);
MTN_API int mtn_paged_decode_plan(const int32_t* kv_indptr, const int32_t* seq_lens, int32_t n_seqs,
                                  int32_t page_size, int32_t num_kv_heads, int32_t head_dim, void* plan,
                                  size_t plan_bytes);
/* mtn_paged_decode with a device copy of a plan made for these kv_indptr /
 * seq_lens (NULL: the kernel splits the tiles evenly itself). */
MTN_API int mtn_paged_decode_with_plan(const mtn_kv_layout* pool, int32_t layer,
                     const void* q, int32_t q_dtype, void* o, int32_t o_dtype,
                     const void* k_new, const void* v_new, int32_t new_dtype,
                     int32_t n_seqs, int32_t num_q_heads,
                     const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens,
                     float scale, uint32_t flags, const void* plan,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of mtn_paged_decode (no counterpart in the
 * reference).  For callers that cannot call cudaMalloc: a host engine whose
 * device memory is all handed out up front by its own arena (the KV pool
 * typically takes nearly all of HBM), or a serving loop that must not
 * allocate mid-step because cudaMalloc can synchronise the device and stall
 * the streams in flight.  Same arguments and results as mtn_paged_decode,
 * without the workspace: the scratch is a static 8 MiB device array inside
 * this library, present on every GPU that loads it until the process exits.
 * Batches needing more scratch than that (mtn_paged_decode_workspace_bytes
 * > 8 MiB) are rejected with MTN_EINVAL: the fixed part is
 * ctas x 32 x (head_dim + 2) x 4 bytes (ctas = SMs x 2 at head_dim 64, SMs
 * otherwise) and each sequence x kv-head pair adds 4 bytes, so a 148-SM B200
 * takes up to about 1.47 million pairs at head_dim 64 or 128 and 0.87
 * million at head_dim 256.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress with that device current), so make that
 * first call before any stream capture.  Every call on a device shares the
 * one array and it keeps the previous call's contents; the part that must
 * start at zero is cleared on the call's stream.  Calls that can overlap on
 * the GPU (different streams without ordering between them) race on the
 * array: serialise them. */
MTN_API int mtn_paged_decode_noalloc(const mtn_kv_layout* pool, int32_t layer,
                     const void* q, int32_t q_dtype, void* o, int32_t o_dtype,
                     const void* k_new, const void* v_new, int32_t new_dtype,
                     int32_t n_seqs, int32_t num_q_heads,
                     const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens,
                     float scale, uint32_t flags, void* stream);

/* Decode over a prefix that every sequence of the batch shares (the
 * refcounted prefix pages of the radix cache, radix_cache.rs:64-117; config
 * 3's shared prompt head).  No counterpart call in the reference, which
 * attends over each request's own cache (qwen model.rs:394-416): the result
 * equals mtn_paged_decode over the block tables prefix_pages ++ own pages,
 * up to f32 rounding.  Sequence r's keys are the n_prefix_pages full pages
 * prefix_pages[] (n_prefix_pages * page_size tokens, read-only) followed by
 * its own pages kv_indices[kv_indptr[r] ..] holding seq_lens[r] tokens
 * (k_new/v_new, if given, are stored at own position seq_lens[r]-1).  The
 * prefix part runs once for all sequences (prefill kernel, non-causal), the
 * own part through the decode kernel, then the two are combined by their
 * log-sum-exps; MTN_ATTN_PHANTOM_ZERO_SLOT counts the zero row once
 * (MTN_ATTN_SPLIT_BF16 is rejected).
 * workspace: mtn_paged_decode_shared_prefix_workspace_bytes(...) bytes,
 * 256-byte aligned, zeroed once before first use, one stream at a time
 * (zero it again after a call that reports a device timeout). */
MTN_API size_t mtn_paged_decode_shared_prefix_workspace_bytes(int32_t n_seqs, int32_t num_q_heads,
                                                      int32_t num_kv_heads, int32_t head_dim);
MTN_API int mtn_paged_decode_shared_prefix(const mtn_kv_layout* pool, int32_t layer,
                     const void* q, int32_t q_dtype, void* o, int32_t o_dtype,
                     const void* k_new, const void* v_new, int32_t new_dtype,
                     int32_t n_seqs, int32_t num_q_heads,
                     const int32_t* prefix_pages, int32_t n_prefix_pages,
                     const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens,
                     float scale, uint32_t flags, void* workspace, size_t workspace_bytes, void* stream);

/* Chunked-prefill attention over paged KV (tcgen05 / TMEM tensor cores).
 *   q: [total_q][num_q_heads][head_dim] (q_dtype: bf16, or f32 rounded to
 *   bf16 -- or split into bf16 hi + lo with MTN_ATTN_SPLIT_BF16 -- on
 *   load); o: same shape (o_dtype).
 *   Sequence r owns query rows qo_indptr[r] .. qo_indptr[r+1]; those are its
 *   LAST q_len = qo_indptr[r+1]-qo_indptr[r] tokens out of seq_lens[r]
 *   (their K/V already appended), so query i sits at position
 *   seq_lens[r] - q_len + i and sees keys at positions <= its own
 *   (generate_causal_mask, model.rs:542-555).
 *   workspace: launches with few (query tile, head) units (at most 3/4 of
 *   the SM count, counted as (total_q / 128 + n_seqs) x num_q_heads) cut
 *   long units into up to 4 pieces of kv tiles on separate CTAs and merge
 *   them; that takes mtn_paged_prefill_workspace_bytes(...) bytes (0 above
 *   296 units), 256-byte aligned, zeroed once before first use and left
 *   zeroed by every call, one stream at a time (after a call that reports
 *   a device timeout, zero it again).  With no or a smaller workspace the
 *   launch runs unsplit. */
MTN_API size_t mtn_paged_prefill_workspace_bytes(int32_t n_seqs, int64_t total_q, int32_t num_q_heads,
                                         int32_t num_kv_heads, int32_t head_dim);
MTN_API int mtn_paged_prefill(const mtn_kv_layout* pool, int32_t layer,
                      const void* q, int32_t q_dtype, void* o, int32_t o_dtype,
                      int32_t n_seqs, int64_t total_q, int32_t num_q_heads,
                      const int32_t* qo_indptr, const int32_t* kv_indptr,
                      const int32_t* kv_indices, const int32_t* seq_lens,
                      int32_t max_q_len, float scale, uint32_t flags,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Greedy sampling on the device (scheduler.rs:186-199 temperature <= 0):
 * out[r] = index of the first strict maximum of logits row r. */
MTN_API int mtn_argmax_rows(const float* logits, int64_t n_rows, int64_t vocab, int32_t* out, void* stream);

/* sample_token (scheduler.rs:186-223) for every row on the device, with
 * row r's temperature temperatures[r] (device array): greedy first strict
 * maximum when <= 0; otherwise the reference's pick -- hash of the first
 * 100 logits' bit patterns -> rand in [0, 1), exp(logit / t) in f32, their
 * sum and running sum in index order, first index reaching rand -- with the
 * same f32 operations in the same order.  workspace: device memory of
 * mtn_sample_rows_workspace_bytes(n_rows, vocab) bytes (any contents). */
MTN_API size_t mtn_sample_rows_workspace_bytes(int64_t n_rows, int64_t vocab);
MTN_API int mtn_sample_rows(const float* logits, const float* temperatures, int64_t n_rows, int64_t vocab,
                            int32_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Host mirror: page allocator (kv_pool.rs:4-69) + refcount extension       */
/* ------------------------------------------------------------------------ */

typedef struct mtn_page_pool mtn_page_pool;

/* KvCachePool::new (kv_pool.rs:18-27): free stack 0..n reversed, so the
 * first allocations are 0, 1, 2, ... */
MTN_API int mtn_page_pool_create(int64_t num_pages, int32_t page_size, mtn_page_pool** out);
MTN_API void mtn_page_pool_destroy(mtn_page_pool* pool);
/* KvCachePool::allocate (kv_pool.rs:30-37); MTN_ENOMEM when exhausted.
 * owner is the 128-bit RequestId as two halves.  The page starts with
 * reference count 1. */
MTN_API int mtn_page_pool_allocate(mtn_page_pool* pool, uint64_t owner_hi, uint64_t owner_lo, uint32_t* page);
/* KvCachePool::free (kv_pool.rs:40-47): MTN_EINVAL for a page that is not
 * in use (the reference's debug_assert), leaving the pool unchanged. */
MTN_API int mtn_page_pool_free(mtn_page_pool* pool, uint32_t page);
MTN_API int64_t mtn_page_pool_free_pages(const mtn_page_pool* pool);
MTN_API int64_t mtn_page_pool_total_pages(const mtn_page_pool* pool);
MTN_API int32_t mtn_page_pool_page_size(const mtn_page_pool* pool);
/* 0 = Free, 1 = InUse (owner halves stored when non-NULL). */
MTN_API int mtn_page_pool_state(const mtn_page_pool* pool, uint32_t page, int32_t* in_use,
                        uint64_t* owner_hi, uint64_t* owner_lo);
/* Extension (no counterpart in the reference): shared pages.  retain adds a
 * reference; release drops one and returns the page to the free stack when
 * the count reaches zero (*freed = 1). */
MTN_API int mtn_page_pool_retain(mtn_page_pool* pool, uint32_t page);
MTN_API int mtn_page_pool_release(mtn_page_pool* pool, uint32_t page, int32_t* freed);
MTN_API int32_t mtn_page_pool_refcount(const mtn_page_pool* pool, uint32_t page);

/* ------------------------------------------------------------------------ */
/* Host mirror: radix prefix cache (radix_cache.rs:37-303)                  */
/* ------------------------------------------------------------------------ */

typedef struct mtn_radix mtn_radix;

MTN_API int mtn_radix_create(int32_t page_size, int64_t max_pages, mtn_radix** out);
MTN_API void mtn_radix_destroy(mtn_radix* r);
/* match_prefix (radix_cache.rs:64-117).  Writes up to *n_pages page ids and
 * *n_nodes node ids (capacities in, counts out; MTN_EINVAL if too small). */
MTN_API int mtn_radix_match_prefix(mtn_radix* r, const uint32_t* tokens, int64_t n_tokens,
                           int64_t* matched_len, uint32_t* pages, int64_t* n_pages,
                           uint64_t* nodes, int64_t* n_nodes);
/* insert_prefix (radix_cache.rs:123-187).  Pages evicted to make room are
 * reported in evicted (capacity/count in *n_evicted; may be NULL to drop
 * them, as the reference does at radix_cache.rs:133). */
MTN_API int mtn_radix_insert_prefix(mtn_radix* r, const uint32_t* tokens, int64_t n_tokens,
                            const uint32_t* pages, int64_t n_pages,
                            uint32_t* evicted, int64_t* n_evicted);
MTN_API int mtn_radix_unlock_nodes(mtn_radix* r, const uint64_t* nodes, int64_t n_nodes);
/* evict_pages (radix_cache.rs:243-282): frees LRU unlocked leaves until
 * target pages are collected or nothing is evictable. */
MTN_API int mtn_radix_evict_pages(mtn_radix* r, int64_t target, uint32_t* freed, int64_t* n_freed);
/* promote_request (radix_cache.rs:287-294). */
MTN_API int mtn_radix_promote(mtn_radix* r, const uint32_t* input_ids, int64_t n_input,
                      int64_t device_len, const uint32_t* kv_pages, int64_t n_kv_pages);
MTN_API int64_t mtn_radix_total_cached_pages(const mtn_radix* r);
MTN_API int64_t mtn_radix_num_nodes(const mtn_radix* r);

/* ------------------------------------------------------------------------ */
/* Host mirror: scheduler (prefill.rs, decode.rs, scheduler.rs)             */
/* ------------------------------------------------------------------------ */

typedef struct mtn_sched mtn_sched;

enum {
  /* Exactly the reference's page lifecycle: a finished request frees every
   * page it lists, radix-shared ones included (scheduler.rs:164-172). */
  MTN_SCHED_REFERENCE = 0,
  /* Refcounted pages: radix-shared pages stay alive while the tree holds
   * them; decode grows a request by one page when its last page fills;
   * a partially filled shared page is copied before the first append. */
  MTN_SCHED_REFCOUNT = 1
};

typedef struct {
  int64_t num_pages;
  int32_t page_size;
  int32_t max_prefill_tokens_per_iter;  /* EngineConfig, config.rs:3-16 */
  int32_t max_decode_batch_size;
  int64_t radix_max_pages;
  int32_t mode;                         /* MTN_SCHED_REFERENCE / _REFCOUNT */
  int32_t n_eos;
  const uint32_t* eos_token_ids;        /* ModelConfig::eos_token_ids     */
} mtn_sched_config;

enum {
  MTN_REQ_WAITING = 0,
  MTN_REQ_PREFILLING = 1,
  MTN_REQ_DECODING = 2,
  MTN_REQ_DONE = 3,
  MTN_REQ_ABORTED = 4
};

enum { MTN_PHASE_PREFILL_ONLY = 0, MTN_PHASE_DECODE_ONLY = 1, MTN_PHASE_MIXED = 2 };

/* A scheduled batch (Batch, batch.rs:7-36) in CSR form.  Arrays are owned
 * by the scheduler and valid until its next schedule call. */
typedef struct {
  int32_t phase;
  int32_t n_reqs;              /* prefill rows first, then decode rows     */
  int32_t n_prefill;
  int64_t n_tokens;
  const uint64_t* req_ids;     /* [n_reqs]                                 */
  const uint32_t* input_ids;   /* [n_tokens]                               */
  const int32_t* position_ids; /* [n_tokens]                               */
  const int32_t* qo_indptr;    /* [n_reqs+1] token ranges                  */
  const int32_t* kv_indptr;    /* [n_reqs+1] page ranges (page_table CSR)  */
  const int32_t* kv_indices;   /* [kv_indptr[n_reqs]]                      */
  const int32_t* seq_lens;     /* [n_reqs] KV tokens after this step       */
  int64_t n_cow;               /* copy-on-write page pairs to run first   */
  const int32_t* cow_src;
  const int32_t* cow_dst;
  const float* temperatures;   /* [n_reqs] SamplingParams::temperature     */
} mtn_batch_view;

MTN_API int mtn_sched_create(const mtn_sched_config* cfg, mtn_sched** out);
MTN_API void mtn_sched_destroy(mtn_sched* s);
/* Queue a request (Request::new, request.rs:85-101; engine_loop.rs:36-39).
 * temperature <= 0 selects greedy sampling (scheduler.rs:186-199). */
MTN_API int mtn_sched_add_request(mtn_sched* s, uint64_t req_id, const uint32_t* input_ids, int64_t n_input,
                          float temperature, int32_t max_new_tokens);
/* schedule_batch (scheduler.rs:8-27).  *has_batch = 0 when nothing runs. */
MTN_API int mtn_sched_schedule(mtn_sched* s, mtn_batch_view* out, int32_t* has_batch);
/* process_and_transition (scheduler.rs:79-184) with host logits, one row
 * per batch request: [n_rows][vocab] f32. */
MTN_API int mtn_sched_process_logits(mtn_sched* s, const float* logits, int64_t n_rows, int64_t vocab);
/* Same transition with tokens already sampled on the device. */
MTN_API int mtn_sched_process_tokens(mtn_sched* s, const uint32_t* tokens, int64_t n_rows);
/* Abort every request of the last batch (engine_loop.rs:47-57). */
MTN_API int mtn_sched_abort_batch(mtn_sched* s);
MTN_API int mtn_sched_request_info(const mtn_sched* s, uint64_t req_id, int32_t* state,
                           int64_t* device_len, int64_t* cached_len, int64_t* n_pages,
                           int64_t* n_output);
MTN_API int mtn_sched_request_pages(const mtn_sched* s, uint64_t req_id, uint32_t* pages, int64_t* n_pages);
MTN_API int mtn_sched_request_output(const mtn_sched* s, uint64_t req_id, uint32_t* out, int64_t* n_out);
/* Prefix fork (refcount mode; no counterpart in the reference, whose pages
 * carry no reference counts): queue child_id with the prompt
 * parent prompt + suffix (n_suffix >= 1), sharing the parent's pages of its
 * whole prompt -- the partially filled last page too -- with cached_len set
 * to the parent's prompt length.  The first write into a shared partial
 * page is preceded by a copy-on-write pair in the batch (cow_src/cow_dst).
 * The parent must have finished its prompt and still hold its pages. */
MTN_API int mtn_sched_fork(mtn_sched* s, uint64_t parent_id, uint64_t child_id, const uint32_t* suffix,
                           int64_t n_suffix, float temperature, int32_t max_new_tokens);
/* Prefill -> decode handoff on the host side (KvHandoff, phase2b-deliverable
 * .md:272-354).  Export: a Decoding request (its prompt done) leaves this
 * scheduler -- its pages (capacity/count in *n_pages), device_len (tokens of
 * KV they hold) and generated tokens (capacity/count in *n_output) are
 * reported, its page references returned and it ends Done here.  Pack the
 * pages (mtn_kv_pages_pack, on the stream this scheduler's kernels use)
 * before this scheduler's next launch, which may reuse them.
 * Import: admit a handed-over request straight into Decoding on this
 * scheduler -- prompt, generated tokens (at least one), device_len with
 * n_input <= device_len < n_input + n_output -- on ceil(device_len /
 * page_size) freshly allocated pages returned in pages (evicting radix
 * pages when needed; MTN_ENOMEM when the pool cannot hold them).  Unpack
 * the KV there (mtn_kv_pages_unpack) before its next decode batch.  The id
 * may be one this scheduler exported (or saw finish) earlier: swapping a
 * request out to host memory and back in. */
MTN_API int mtn_sched_export(mtn_sched* s, uint64_t req_id, uint32_t* pages, int64_t* n_pages, int64_t* device_len,
                             uint32_t* output_ids, int64_t* n_output);
MTN_API int mtn_sched_import(mtn_sched* s, uint64_t req_id, const uint32_t* input_ids, int64_t n_input,
                             const uint32_t* output_ids, int64_t n_output, int64_t device_len, float temperature,
                             int32_t max_new_tokens, uint32_t* pages, int64_t* n_pages);
/* Inspection for tests: a page's reference count (0 = free, -1 = out of
 * range) and every page the radix cache lists (capacity/count in *n_pages). */
MTN_API int32_t mtn_sched_page_refcount(const mtn_sched* s, uint32_t page);
MTN_API int mtn_sched_tree_pages(const mtn_sched* s, uint32_t* pages, int64_t* n_pages);
MTN_API int64_t mtn_sched_free_pages(const mtn_sched* s);
MTN_API int64_t mtn_sched_cached_pages(const mtn_sched* s);
MTN_API int32_t mtn_sched_num_active(const mtn_sched* s);

#ifdef __cplusplus
}
#endif

#endif /* MITTEN_KV_H */
