// Chunked-prefill attention over paged KV (tcgen05 / TMEM) -- in progress.
#include "common.cuh"

using mtn::set_error;

extern "C" {

size_t mtn_paged_prefill_workspace_bytes(int32_t n_seqs, int64_t total_q, int32_t num_q_heads, int32_t num_kv_heads,
                                         int32_t head_dim) {
  (void)n_seqs; (void)total_q; (void)num_q_heads; (void)num_kv_heads; (void)head_dim;
  return 0;
}

int mtn_paged_prefill(const mtn_kv_layout* pool, int32_t layer, const void* q, void* o, int32_t o_dtype,
                      int32_t n_seqs, int64_t total_q, int32_t num_q_heads, const int32_t* qo_indptr,
                      const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* seq_lens, int32_t max_q_len,
                      float scale, uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  return set_error(MTN_EINVAL, "mtn_paged_prefill: not built yet");
}

}
