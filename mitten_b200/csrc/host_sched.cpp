// Host mirror of the reference scheduler:
//   PrefillAdder::run / schedule_prefill_chunk  (inference-engine/src/prefill.rs:21-114)
//   collect_decode_requests                      (inference-engine/src/decode.rs:6-47)
//   schedule_batch / assemble_batch              (inference-engine/src/scheduler.rs:8-77)
//   process_and_transition / sample_token        (inference-engine/src/scheduler.rs:79-223)
// producing the Batch (inference-backend/src/batch.rs:7-36) in CSR form.
//
// MTN_SCHED_REFERENCE keeps the reference's page lifecycle verbatim.
// MTN_SCHED_REFCOUNT is the device engine's mode: pages carry reference
// counts (the radix tree holds one per cached page, each request one per
// page it lists), a decoding request gains a page when its last one is full,
// a fully cached prompt still recomputes its last token, and a request that
// would write into a shared page first gets a private copy (copy-on-write
// pairs are returned with the batch).
#include <algorithm>
#include <cmath>
#include <cstring>

#include "host.hpp"

namespace mtn {

namespace {

struct Req {
  uint64_t id = 0;
  std::vector<uint32_t> input_ids;
  int32_t state = MTN_REQ_WAITING;
  int64_t cached_len = 0;
  int64_t device_len = 0;
  int64_t extend_len = 0;
  std::vector<uint32_t> kv_pages;
  std::vector<uint32_t> output_ids;
  float temperature = 1.0f;
  int32_t max_new_tokens = 512;
  std::vector<uint64_t> locked_nodes;
  bool forked = false;  // holds its parent's prompt pages from mtn_sched_fork
};

}  // namespace

struct Sched {
  mtn_sched_config cfg;
  std::vector<uint32_t> eos;
  PagePool pool;
  RadixTree radix;
  std::deque<Req*> waiting;
  std::vector<Req*> prefilling;
  std::vector<Req*> decoding;
  std::unordered_map<uint64_t, std::unique_ptr<Req>> reqs;

  // Last scheduled batch and its CSR view.
  std::vector<Req*> batch;
  std::vector<uint64_t> v_ids;
  std::vector<uint32_t> v_input;
  std::vector<int32_t> v_pos, v_qo, v_kvp, v_kvi, v_len, v_cow_src, v_cow_dst;
  std::vector<float> v_temp;

  Sched(const mtn_sched_config& c)
      : cfg(c), pool(c.num_pages, c.page_size), radix(c.page_size, c.radix_max_pages) {
    if (c.eos_token_ids && c.n_eos > 0) eos.assign(c.eos_token_ids, c.eos_token_ids + c.n_eos);
    cfg.eos_token_ids = nullptr;
  }

  // First failed page return since the last schedule/process call.  The
  // reference's KvCachePool::free debug_asserts that the page is in use
  // (kv_pool.rs:40-45), which panics in the debug builds its tests run in;
  // here the call that hit it reports MTN_EINVAL with that message.
  int fault = MTN_OK;

  bool refcount() const { return cfg.mode == MTN_SCHED_REFCOUNT; }

  int take_fault() {
    const int f = fault;
    fault = MTN_OK;
    return f;
  }

  // --------------------------------------------------------------- pages

  // Return a page the request (or the tree) no longer lists.
  int drop_page(uint32_t page) {
    const int st = refcount() ? pool.release(page, nullptr) : pool.free(page);  // kv_pool.rs:40-47
    if (st != MTN_OK && fault == MTN_OK) fault = st;
    return st;
  }

  int drop_pages(std::vector<uint32_t>& pages) {
    int st = MTN_OK;
    for (uint32_t p : pages) {
      const int e = drop_page(p);
      if (e != MTN_OK && st == MTN_OK) st = e;
    }
    pages.clear();
    return st;
  }

  // Pages evicted from the tree go back to the pool (prefill.rs:46-49).
  void return_evicted(std::vector<uint32_t>& freed) {
    for (uint32_t p : freed) drop_page(p);
    freed.clear();
  }

  // One page for `r`, evicting from the tree if the pool is empty.
  bool alloc_page(Req* r, uint32_t* page) {
    if (pool.allocate(r->id >> 32, r->id, page)) return true;
    std::vector<uint32_t> freed;
    while (pool.free_pages() == 0) {
      radix.evict_pages(1, &freed);
      if (freed.empty()) return false;
      return_evicted(freed);
    }
    return pool.allocate(r->id >> 32, r->id, page);
  }

  void promote(Req* r) {
    // scheduler.rs:116-117 -> radix_cache.rs:287-294.
    std::vector<uint32_t> evicted, adopted;
    radix.promote(r->input_ids.data(), static_cast<int64_t>(r->input_ids.size()), r->device_len,
                  r->kv_pages.data(), static_cast<int64_t>(r->kv_pages.size()), &evicted, &adopted);
    if (refcount()) {
      for (uint32_t p : adopted) pool.retain(p);  // the tree's own reference
      return_evicted(evicted);
    }
    // Reference mode: insert_prefix drops evicted pages (radix_cache.rs:133).
  }

  void release_request(Req* r) {
    // scheduler.rs:164-172 / decode.rs:20-28.
    radix.unlock_nodes(r->locked_nodes.data(), static_cast<int64_t>(r->locked_nodes.size()));
    r->locked_nodes.clear();
    drop_pages(r->kv_pages);
  }

  static void erase_from(std::vector<Req*>& v, Req* r) {
    auto it = std::find(v.begin(), v.end(), r);
    if (it != v.end()) v.erase(it);
  }

  void abort_request(Req* r) {
    r->state = MTN_REQ_ABORTED;
    release_request(r);
    erase_from(prefilling, r);
    erase_from(decoding, r);
    auto it = std::find(waiting.begin(), waiting.end(), r);
    if (it != waiting.end()) waiting.erase(it);
  }

  // ------------------------------------------------------------ scheduling

  std::vector<Req*> collect_decode() {
    // decode.rs:6-47.
    std::vector<Req*> out;
    size_t i = 0;
    while (i < decoding.size()) {
      Req* r = decoding[i];
      if (r->state == MTN_REQ_DECODING) {
        out.push_back(r);
        ++i;
      } else if (r->state == MTN_REQ_DONE || r->state == MTN_REQ_ABORTED) {
        release_request(r);
        decoding.erase(decoding.begin() + static_cast<std::ptrdiff_t>(i));
      } else {
        ++i;
      }
    }
    if (static_cast<int64_t>(out.size()) > cfg.max_decode_batch_size) out.resize(cfg.max_decode_batch_size);
    return out;
  }

  // prefill.rs:99-114.  Returns -1 for None.
  int64_t prefill_chunk(Req* r, int64_t budget, int64_t* used) {
    const int64_t remaining = static_cast<int64_t>(r->input_ids.size()) - r->device_len;
    if (remaining == 0) return 0;
    const int64_t chunk = std::min(remaining, budget - *used);
    if (chunk > 0) {
      r->extend_len = chunk;
      *used += chunk;
      return chunk;
    }
    return -1;
  }

  std::vector<Req*> run_prefill(int64_t budget) {
    // prefill.rs:21-97.
    std::vector<Req*> added;
    int64_t used = 0;
    const std::vector<Req*> in_progress = prefilling;
    for (Req* r : in_progress) {
      if (used >= budget) break;
      if (prefill_chunk(r, budget, &used) > 0) added.push_back(r);
    }
    const int64_t ps = cfg.page_size;
    while (used < budget && !waiting.empty()) {
      Req* r = waiting.front();
      const int64_t input_len = static_cast<int64_t>(r->input_ids.size());
      // A fork already holds its parent's prompt pages: it needs the rest of
      // its prompt's pages plus one for the copy of a shared partial page.
      const int64_t pages_needed =
          r->forked ? (input_len + ps - 1) / ps - static_cast<int64_t>(r->kv_pages.size()) +
                          ((r->cached_len % ps) != 0 ? 1 : 0)
                    : (input_len + ps - 1) / ps;
      if (pool.free_pages() < pages_needed) {
        std::vector<uint32_t> freed;
        if (refcount()) {
          // Shared pages free nothing until their last holder lets go: keep evicting.
          while (pool.free_pages() < pages_needed) {
            radix.evict_pages(pages_needed - pool.free_pages(), &freed);
            if (freed.empty()) break;
            return_evicted(freed);
          }
        } else {
          radix.evict_pages(pages_needed - pool.free_pages(), &freed);
          return_evicted(freed);
        }
        if (pool.free_pages() < pages_needed) break;  // cannot admit yet
      }
      waiting.pop_front();
      if (!r->forked) {
        int64_t cached = 0;
        std::vector<uint32_t> pages;
        std::vector<uint64_t> nodes;
        // A fully cached prompt would leave nothing to compute and no logits
        // to sample from; the refcount engine always recomputes the last token.
        const int64_t match_n = refcount() ? std::max<int64_t>(0, input_len - 1) : input_len;
        radix.match_prefix(r->input_ids.data(), match_n, &cached, &pages, &nodes);
        r->cached_len = cached;
        r->device_len = cached;
        r->locked_nodes = nodes;
        r->kv_pages = pages;
        if (refcount())
          for (uint32_t p : r->kv_pages) pool.retain(p);
      }
      const int64_t prompt_pages = (input_len + ps - 1) / ps;
      while (static_cast<int64_t>(r->kv_pages.size()) < prompt_pages) {
        uint32_t p = 0;
        if (!pool.allocate(r->id >> 32, r->id, &p)) break;  // unreachable after the check above
        r->kv_pages.push_back(p);
      }
      r->state = MTN_REQ_PREFILLING;
      prefilling.push_back(r);
      if (prefill_chunk(r, budget, &used) > 0) added.push_back(r);
    }
    return added;
  }

  // Decode-time page growth and copy-on-write (refcount mode only).
  bool prepare_write(Req* r, int64_t first_pos, int64_t end_pos) {
    const int64_t ps = cfg.page_size;
    const int64_t need = (end_pos + ps - 1) / ps;
    while (static_cast<int64_t>(r->kv_pages.size()) < need) {
      uint32_t p = 0;
      if (!alloc_page(r, &p)) return false;
      r->kv_pages.push_back(p);
    }
    const int64_t idx = first_pos / ps;
    if (idx < static_cast<int64_t>(r->kv_pages.size()) && pool.refcnt[r->kv_pages[idx]] > 1) {
      uint32_t fresh = 0;
      if (!alloc_page(r, &fresh)) return false;
      const uint32_t old = r->kv_pages[idx];
      v_cow_src.push_back(static_cast<int32_t>(old));
      v_cow_dst.push_back(static_cast<int32_t>(fresh));
      r->kv_pages[idx] = fresh;
      pool.release(old, nullptr);
    }
    return true;
  }

  // A new request whose prompt is the parent's whole prompt plus `suffix`,
  // holding (one more reference each) the parent's pages of that prompt,
  // its partially filled last page included; its first write into that
  // page makes it a private copy (prepare_write).  Refcount mode only.
  int fork(uint64_t parent_id, uint64_t child_id, const uint32_t* suffix, int64_t n_suffix, float temperature,
           int32_t max_new_tokens) {
    MTN_CHECK_ARG(refcount(), "mtn_sched_fork: needs MTN_SCHED_REFCOUNT (the reference frees shared pages)");
    auto it = reqs.find(parent_id);
    MTN_CHECK_ARG(it != reqs.end(), "mtn_sched_fork: unknown parent %llu", (unsigned long long)parent_id);
    MTN_CHECK_ARG(reqs.find(child_id) == reqs.end(), "mtn_sched_fork: duplicate request id %llu",
                  (unsigned long long)child_id);
    Req* par = it->second.get();
    const int64_t n_prompt = static_cast<int64_t>(par->input_ids.size());
    const int64_t ps = cfg.page_size;
    MTN_CHECK_ARG((par->state == MTN_REQ_DECODING || par->state == MTN_REQ_PREFILLING) && par->device_len >= n_prompt &&
                      static_cast<int64_t>(par->kv_pages.size()) >= (n_prompt + ps - 1) / ps,
                  "mtn_sched_fork: parent %llu has not finished its prompt or no longer holds its pages",
                  (unsigned long long)parent_id);
    MTN_CHECK_ARG(suffix != nullptr && n_suffix > 0 && n_prompt + n_suffix < (int64_t(1) << 31),
                  "mtn_sched_fork: the suffix must hold at least one token");
    auto r = std::make_unique<Req>();
    r->id = child_id;
    r->input_ids = par->input_ids;
    r->input_ids.insert(r->input_ids.end(), suffix, suffix + n_suffix);
    r->temperature = temperature;
    r->max_new_tokens = max_new_tokens;
    r->cached_len = n_prompt;
    r->device_len = n_prompt;
    r->forked = true;
    r->kv_pages.assign(par->kv_pages.begin(), par->kv_pages.begin() + (n_prompt + ps - 1) / ps);
    for (uint32_t p : r->kv_pages) pool.retain(p);
    waiting.push_back(r.get());
    reqs.emplace(child_id, std::move(r));
    return MTN_OK;
  }

  // Prefill -> decode handoff (the reference's KvHandoff: request id, its
  // pages, the tokens they hold).  Export: a Decoding request leaves this
  // scheduler; the caller gets its pages (pack them before this scheduler's
  // next launch) and its state, and the request's page references are
  // returned (it ends Done here).
  int export_request(uint64_t id, std::vector<uint32_t>* pages, int64_t* device_len,
                     std::vector<uint32_t>* outputs) {
    auto it = reqs.find(id);
    MTN_CHECK_ARG(it != reqs.end(), "mtn_sched_export: unknown request %llu", (unsigned long long)id);
    Req* r = it->second.get();
    MTN_CHECK_ARG(r->state == MTN_REQ_DECODING, "mtn_sched_export: request %llu is not decoding",
                  (unsigned long long)id);
    *pages = r->kv_pages;
    *device_len = r->device_len;
    *outputs = r->output_ids;
    r->state = MTN_REQ_DONE;
    release_request(r);
    erase_from(decoding, r);
    return take_fault();
  }

  // Import: admit a handed-over request straight into Decoding with
  // device_len tokens of KV on pages allocated here (returned: unpack the KV
  // into them before its next decode batch).
  int import_request(uint64_t id, const uint32_t* input_ids, int64_t n_input, const uint32_t* outputs,
                     int64_t n_output, int64_t device_len, float temperature, int32_t max_new_tokens,
                     std::vector<uint32_t>* pages) {
    // A finished request (Done or Aborted, no pages) may come back under its
    // id: a request swapped out to host memory by export and swapped in again.
    auto prev = reqs.find(id);
    MTN_CHECK_ARG(prev == reqs.end() || ((prev->second->state == MTN_REQ_DONE || prev->second->state == MTN_REQ_ABORTED) &&
                                         prev->second->kv_pages.empty()),
                  "mtn_sched_import: request id %llu is still live here", (unsigned long long)id);
    MTN_CHECK_ARG(input_ids && n_input > 0 && n_output >= 1 && outputs && device_len >= n_input &&
                      device_len < n_input + n_output,
                  "mtn_sched_import: inconsistent request (prompt %lld, outputs %lld, device_len %lld)",
                  (long long)n_input, (long long)n_output, (long long)device_len);
    const int64_t ps = cfg.page_size;
    const int64_t need = (device_len + ps - 1) / ps;
    auto r = std::make_unique<Req>();
    r->id = id;
    r->input_ids.assign(input_ids, input_ids + n_input);
    r->output_ids.assign(outputs, outputs + n_output);
    r->temperature = temperature;
    r->max_new_tokens = max_new_tokens;
    r->device_len = device_len;
    while (static_cast<int64_t>(r->kv_pages.size()) < need) {
      uint32_t p = 0;
      if (!alloc_page(r.get(), &p)) {
        drop_pages(r->kv_pages);
        return set_error(MTN_ENOMEM, "mtn_sched_import: %lld pages needed, the pool is exhausted", (long long)need);
      }
      r->kv_pages.push_back(p);
    }
    r->state = MTN_REQ_DECODING;
    *pages = r->kv_pages;
    decoding.push_back(r.get());
    if (prev != reqs.end()) {
      std::replace(batch.begin(), batch.end(), prev->second.get(), r.get());
      prev->second = std::move(r);
    } else {
      reqs.emplace(id, std::move(r));
    }
    return MTN_OK;
  }

  int schedule(mtn_batch_view* out, int32_t* has_batch) {
    // scheduler.rs:8-27.
    *has_batch = 0;
    std::memset(out, 0, sizeof(*out));
    v_cow_src.clear();
    v_cow_dst.clear();
    std::vector<Req*> dec = collect_decode();
    if (refcount()) {
      std::vector<Req*> kept;
      for (Req* r : dec) {
        if (prepare_write(r, r->device_len, r->device_len + 1)) {
          kept.push_back(r);
        } else {
          abort_request(r);  // EngineError::OutOfKvPages for this request
        }
      }
      dec.swap(kept);
    }
    const int64_t budget = std::max<int64_t>(0, cfg.max_prefill_tokens_per_iter - static_cast<int64_t>(dec.size()));
    std::vector<Req*> pre = run_prefill(budget);
    if (refcount()) {
      std::vector<Req*> kept;
      for (Req* r : pre) {
        if (prepare_write(r, r->device_len, r->device_len + r->extend_len)) {
          kept.push_back(r);
        } else {
          abort_request(r);
        }
      }
      pre.swap(kept);
    }
    batch.clear();
    if (fault != MTN_OK) return take_fault();
    if (dec.empty() && pre.empty()) return MTN_OK;
    assemble(pre, dec);
    out->phase = pre.empty() ? MTN_PHASE_DECODE_ONLY : (dec.empty() ? MTN_PHASE_PREFILL_ONLY : MTN_PHASE_MIXED);
    out->n_reqs = static_cast<int32_t>(batch.size());
    out->n_prefill = static_cast<int32_t>(pre.size());
    out->n_tokens = static_cast<int64_t>(v_input.size());
    out->req_ids = v_ids.data();
    out->input_ids = v_input.data();
    out->position_ids = v_pos.data();
    out->qo_indptr = v_qo.data();
    out->kv_indptr = v_kvp.data();
    out->kv_indices = v_kvi.data();
    out->seq_lens = v_len.data();
    out->n_cow = static_cast<int64_t>(v_cow_src.size());
    out->cow_src = v_cow_src.data();
    out->cow_dst = v_cow_dst.data();
    out->temperatures = v_temp.data();
    *has_batch = 1;
    return MTN_OK;
  }

  void assemble(const std::vector<Req*>& pre, const std::vector<Req*>& dec) {
    // scheduler.rs:29-77 (prefill rows first), page_table as CSR.
    v_ids.clear();
    v_input.clear();
    v_pos.clear();
    v_qo.assign(1, 0);
    v_kvp.assign(1, 0);
    v_kvi.clear();
    v_len.clear();
    v_temp.clear();
    for (Req* r : pre) {
      const int64_t start = r->device_len, end = r->device_len + r->extend_len;
      for (int64_t i = start; i < end; ++i) {
        v_input.push_back(r->input_ids[i]);
        v_pos.push_back(static_cast<int32_t>(i));
      }
      add_row(r, end);
    }
    for (Req* r : dec) {
      const uint32_t last = r->output_ids.empty() ? r->input_ids.back() : r->output_ids.back();
      v_input.push_back(last);
      v_pos.push_back(static_cast<int32_t>(r->device_len));
      add_row(r, r->device_len + 1);
    }
  }

  void add_row(Req* r, int64_t kv_len) {
    batch.push_back(r);
    v_ids.push_back(r->id);
    v_qo.push_back(static_cast<int32_t>(v_input.size()));
    for (uint32_t p : r->kv_pages) v_kvi.push_back(static_cast<int32_t>(p));
    v_kvp.push_back(static_cast<int32_t>(v_kvi.size()));
    v_len.push_back(static_cast<int32_t>(kv_len));
    v_temp.push_back(r->temperature);
  }

  // ------------------------------------------------------------ transition

  static uint32_t sample(const float* row, int64_t vocab, float temperature) {
    // scheduler.rs:186-223.
    if (temperature <= 0.0f) {
      float best = -INFINITY;
      int64_t idx = 0;
      for (int64_t i = 0; i < vocab; ++i) {
        if (row[i] > best) {
          best = row[i];
          idx = i;
        }
      }
      return static_cast<uint32_t>(idx);
    }
    uint64_t hash = 0;
    for (int64_t i = 0; i < std::min<int64_t>(vocab, 100); ++i) {
      uint32_t bits;
      std::memcpy(&bits, &row[i], 4);
      hash = hash * 31u + static_cast<uint64_t>(bits);
    }
    const float rand_val = static_cast<float>(hash % 1000) / 1000.0f;
    std::vector<float> e(static_cast<size_t>(vocab));
    float sum = 0.0f;
    for (int64_t i = 0; i < vocab; ++i) {
      e[i] = std::exp(row[i] / temperature);
      sum += e[i];
    }
    float cum = 0.0f;
    for (int64_t i = 0; i < vocab; ++i) {
      cum += e[i] / sum;
      if (rand_val <= cum) return static_cast<uint32_t>(i);
    }
    return static_cast<uint32_t>(vocab - 1);
  }

  template <typename TokenOf>
  int transition(int64_t n_rows, TokenOf token_of) {
    // scheduler.rs:79-184.
    int64_t row = 0;
    for (Req* r : batch) {
      if (r->state == MTN_REQ_PREFILLING) {
        r->device_len += r->extend_len;
        r->extend_len = 0;
        if (r->device_len == static_cast<int64_t>(r->input_ids.size())) {
          if (row >= n_rows) return set_error(MTN_EINVAL, "process: %lld rows for a larger batch", (long long)n_rows);
          const uint32_t tok = token_of(row, r);
          r->output_ids.push_back(tok);
          r->state = MTN_REQ_DECODING;
          erase_from(prefilling, r);
          decoding.push_back(r);
          promote(r);
        }
        ++row;
      } else if (r->state == MTN_REQ_DECODING) {
        if (row >= n_rows) return set_error(MTN_EINVAL, "process: %lld rows for a larger batch", (long long)n_rows);
        const uint32_t tok = token_of(row, r);
        r->output_ids.push_back(tok);
        r->device_len += 1;
        bool done = false;
        if (std::find(eos.begin(), eos.end(), tok) != eos.end()) {
          done = true;
        } else if (static_cast<int64_t>(r->output_ids.size()) >= r->max_new_tokens) {
          done = true;
        }
        if (done) {
          r->state = MTN_REQ_DONE;
          release_request(r);
          erase_from(decoding, r);
        }
        ++row;
      }
    }
    batch.clear();
    return take_fault();
  }
};

}  // namespace mtn

struct mtn_sched {
  mtn::Sched impl;
  explicit mtn_sched(const mtn_sched_config& c) : impl(c) {}
};

using mtn::set_error;

extern "C" {

int mtn_sched_create(const mtn_sched_config* cfg, mtn_sched** out) {
  MTN_CHECK_ARG(cfg && out, "mtn_sched_create: null argument");
  MTN_CHECK_ARG(cfg->num_pages >= 0 && cfg->num_pages <= (int64_t(1) << 31), "mtn_sched_create: bad num_pages");
  MTN_CHECK_ARG(cfg->page_size > 0, "mtn_sched_create: page_size must be positive");
  MTN_CHECK_ARG(cfg->max_decode_batch_size >= 0 && cfg->max_prefill_tokens_per_iter >= 0,
                "mtn_sched_create: negative budget");
  MTN_CHECK_ARG(cfg->mode == MTN_SCHED_REFERENCE || cfg->mode == MTN_SCHED_REFCOUNT, "mtn_sched_create: bad mode");
  MTN_CHECK_ARG(cfg->n_eos >= 0 && (cfg->n_eos == 0 || cfg->eos_token_ids), "mtn_sched_create: bad eos list");
  *out = new mtn_sched(*cfg);
  return MTN_OK;
}

void mtn_sched_destroy(mtn_sched* s) { delete s; }

int mtn_sched_add_request(mtn_sched* s, uint64_t req_id, const uint32_t* input_ids, int64_t n_input,
                          float temperature, int32_t max_new_tokens) {
  MTN_CHECK_ARG(s && input_ids && n_input > 0, "mtn_sched_add_request: empty prompt");
  MTN_CHECK_ARG(n_input < (int64_t(1) << 31), "mtn_sched_add_request: prompt too long");
  auto& m = s->impl.reqs;
  MTN_CHECK_ARG(m.find(req_id) == m.end(), "mtn_sched_add_request: duplicate request id %llu",
                (unsigned long long)req_id);
  auto r = std::make_unique<mtn::Req>();
  r->id = req_id;
  r->input_ids.assign(input_ids, input_ids + n_input);
  r->temperature = temperature;
  r->max_new_tokens = max_new_tokens;
  s->impl.waiting.push_back(r.get());
  m.emplace(req_id, std::move(r));
  return MTN_OK;
}

int mtn_sched_schedule(mtn_sched* s, mtn_batch_view* out, int32_t* has_batch) {
  MTN_CHECK_ARG(s && out && has_batch, "mtn_sched_schedule: null argument");
  return s->impl.schedule(out, has_batch);
}

int mtn_sched_process_logits(mtn_sched* s, const float* logits, int64_t n_rows, int64_t vocab) {
  MTN_CHECK_ARG(s && (logits || n_rows == 0) && vocab > 0, "mtn_sched_process_logits: bad argument");
  return s->impl.transition(n_rows, [&](int64_t row, mtn::Req* r) {
    return mtn::Sched::sample(logits + row * vocab, vocab, r->temperature);
  });
}

int mtn_sched_process_tokens(mtn_sched* s, const uint32_t* tokens, int64_t n_rows) {
  MTN_CHECK_ARG(s && (tokens || n_rows == 0), "mtn_sched_process_tokens: bad argument");
  return s->impl.transition(n_rows, [&](int64_t row, mtn::Req*) { return tokens[row]; });
}

int mtn_sched_abort_batch(mtn_sched* s) {
  // engine_loop.rs:47-57: every request of the failed batch is aborted.
  MTN_CHECK_ARG(s, "mtn_sched_abort_batch: null scheduler");
  std::vector<mtn::Req*> b = s->impl.batch;
  for (mtn::Req* r : b) s->impl.abort_request(r);
  s->impl.batch.clear();
  return MTN_OK;
}

int mtn_sched_request_info(const mtn_sched* s, uint64_t req_id, int32_t* state, int64_t* device_len,
                           int64_t* cached_len, int64_t* n_pages, int64_t* n_output) {
  MTN_CHECK_ARG(s, "mtn_sched_request_info: null scheduler");
  auto it = s->impl.reqs.find(req_id);
  MTN_CHECK_ARG(it != s->impl.reqs.end(), "mtn_sched_request_info: unknown request %llu",
                (unsigned long long)req_id);
  const mtn::Req& r = *it->second;
  if (state) *state = r.state;
  if (device_len) *device_len = r.device_len;
  if (cached_len) *cached_len = r.cached_len;
  if (n_pages) *n_pages = static_cast<int64_t>(r.kv_pages.size());
  if (n_output) *n_output = static_cast<int64_t>(r.output_ids.size());
  return MTN_OK;
}

int mtn_sched_request_pages(const mtn_sched* s, uint64_t req_id, uint32_t* pages, int64_t* n_pages) {
  MTN_CHECK_ARG(s && n_pages, "mtn_sched_request_pages: null argument");
  auto it = s->impl.reqs.find(req_id);
  MTN_CHECK_ARG(it != s->impl.reqs.end(), "mtn_sched_request_pages: unknown request");
  const auto& v = it->second->kv_pages;
  MTN_CHECK_ARG(static_cast<int64_t>(v.size()) <= *n_pages && (pages || v.empty()),
                "mtn_sched_request_pages: buffer too small (%zu pages)", v.size());
  std::copy(v.begin(), v.end(), pages);
  *n_pages = static_cast<int64_t>(v.size());
  return MTN_OK;
}

int mtn_sched_request_output(const mtn_sched* s, uint64_t req_id, uint32_t* out, int64_t* n_out) {
  MTN_CHECK_ARG(s && n_out, "mtn_sched_request_output: null argument");
  auto it = s->impl.reqs.find(req_id);
  MTN_CHECK_ARG(it != s->impl.reqs.end(), "mtn_sched_request_output: unknown request");
  const auto& v = it->second->output_ids;
  MTN_CHECK_ARG(static_cast<int64_t>(v.size()) <= *n_out && (out || v.empty()),
                "mtn_sched_request_output: buffer too small (%zu tokens)", v.size());
  std::copy(v.begin(), v.end(), out);
  *n_out = static_cast<int64_t>(v.size());
  return MTN_OK;
}

int mtn_sched_export(mtn_sched* s, uint64_t req_id, uint32_t* pages, int64_t* n_pages, int64_t* device_len,
                     uint32_t* output_ids, int64_t* n_output) {
  MTN_CHECK_ARG(s && n_pages && device_len && n_output, "mtn_sched_export: null argument");
  auto it = s->impl.reqs.find(req_id);
  MTN_CHECK_ARG(it != s->impl.reqs.end(), "mtn_sched_export: unknown request %llu", (unsigned long long)req_id);
  const mtn::Req& r = *it->second;
  MTN_CHECK_ARG(static_cast<int64_t>(r.kv_pages.size()) <= *n_pages && (pages || r.kv_pages.empty()) &&
                    static_cast<int64_t>(r.output_ids.size()) <= *n_output && (output_ids || r.output_ids.empty()),
                "mtn_sched_export: buffers too small (%zu pages, %zu tokens)", r.kv_pages.size(), r.output_ids.size());
  std::vector<uint32_t> pg, out;
  int64_t dl = 0;
  const int st = s->impl.export_request(req_id, &pg, &dl, &out);
  if (st != MTN_OK) return st;
  std::copy(pg.begin(), pg.end(), pages);
  std::copy(out.begin(), out.end(), output_ids);
  *n_pages = static_cast<int64_t>(pg.size());
  *n_output = static_cast<int64_t>(out.size());
  *device_len = dl;
  return MTN_OK;
}

int mtn_sched_import(mtn_sched* s, uint64_t req_id, const uint32_t* input_ids, int64_t n_input,
                     const uint32_t* output_ids, int64_t n_output, int64_t device_len, float temperature,
                     int32_t max_new_tokens, uint32_t* pages, int64_t* n_pages) {
  MTN_CHECK_ARG(s && n_pages, "mtn_sched_import: null argument");
  const int64_t need = (device_len + s->impl.cfg.page_size - 1) / s->impl.cfg.page_size;
  MTN_CHECK_ARG(device_len >= 0 && need <= *n_pages && (pages || need == 0),
                "mtn_sched_import: page buffer too small (%lld pages)", (long long)need);
  std::vector<uint32_t> pg;
  const int st = s->impl.import_request(req_id, input_ids, n_input, output_ids, n_output, device_len, temperature,
                                        max_new_tokens, &pg);
  if (st != MTN_OK) return st;
  std::copy(pg.begin(), pg.end(), pages);
  *n_pages = static_cast<int64_t>(pg.size());
  return MTN_OK;
}

int mtn_sched_fork(mtn_sched* s, uint64_t parent_id, uint64_t child_id, const uint32_t* suffix, int64_t n_suffix,
                   float temperature, int32_t max_new_tokens) {
  MTN_CHECK_ARG(s, "mtn_sched_fork: null scheduler");
  return s->impl.fork(parent_id, child_id, suffix, n_suffix, temperature, max_new_tokens);
}

int32_t mtn_sched_page_refcount(const mtn_sched* s, uint32_t page) {
  if (!s || page >= static_cast<uint64_t>(s->impl.pool.num_pages)) return -1;
  return s->impl.pool.in_use[page] ? s->impl.pool.refcnt[page] : 0;
}

int mtn_sched_tree_pages(const mtn_sched* s, uint32_t* pages, int64_t* n_pages) {
  MTN_CHECK_ARG(s && n_pages, "mtn_sched_tree_pages: null argument");
  const mtn::RadixTree& t = s->impl.radix;
  std::vector<uint32_t> all;
  for (size_t i = 0; i < t.entries.size(); ++i)
    if (t.occupied[i]) all.insert(all.end(), t.entries[i].kv_pages.begin(), t.entries[i].kv_pages.end());
  MTN_CHECK_ARG(static_cast<int64_t>(all.size()) <= *n_pages && (pages || all.empty()),
                "mtn_sched_tree_pages: buffer too small (%zu pages)", all.size());
  std::copy(all.begin(), all.end(), pages);
  *n_pages = static_cast<int64_t>(all.size());
  return MTN_OK;
}

int64_t mtn_sched_free_pages(const mtn_sched* s) { return s ? s->impl.pool.free_pages() : -1; }

int64_t mtn_sched_cached_pages(const mtn_sched* s) { return s ? s->impl.radix.total_pages : -1; }

int32_t mtn_sched_num_active(const mtn_sched* s) {
  if (!s) return -1;
  return static_cast<int32_t>(s->impl.waiting.size() + s->impl.prefilling.size() + s->impl.decoding.size());
}

}  // extern "C"
