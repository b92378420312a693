// Host mirror of the engine's page bookkeeping:
//   - PagePool  : KvCachePool, inference-engine/src/kv_pool.rs:4-69, plus
//                 per-page reference counts (extension for shared pages).
//   - RadixTree : RadixCache, inference-engine/src/radix_cache.rs:37-303.
// Both keep the reference's observable order exactly: the LIFO free stack
// (kv_pool.rs:19-20, 31, 46), slab node-id reuse (most recently removed id
// first, as the `slab` crate does), and the eviction heap ordered by
// (Reverse(last_used), node id) (radix_cache.rs:41).  `Instant::now()` is
// replaced by a logical clock that ticks on every call site the reference
// reads the clock, so ties never depend on timer resolution.
#include "host.hpp"

#include <algorithm>

namespace mtn {

// ------------------------------------------------------------------ PagePool

PagePool::PagePool(int64_t n, int32_t ps) : num_pages(n), page_size(ps) {
  free_stack.reserve(static_cast<size_t>(n));
  for (int64_t i = n - 1; i >= 0; --i) free_stack.push_back(static_cast<uint32_t>(i));  // kv_pool.rs:19-20
  in_use.assign(static_cast<size_t>(n), 0);
  owner_hi.assign(static_cast<size_t>(n), 0);
  owner_lo.assign(static_cast<size_t>(n), 0);
  refcnt.assign(static_cast<size_t>(n), 0);
}

bool PagePool::allocate(uint64_t hi, uint64_t lo, uint32_t* page) {
  if (free_stack.empty()) return false;  // kv_pool.rs:30-37: None
  const uint32_t p = free_stack.back();
  free_stack.pop_back();
  in_use[p] = 1;
  owner_hi[p] = hi;
  owner_lo[p] = lo;
  refcnt[p] = 1;
  *page = p;
  return true;
}

int PagePool::free(uint32_t page) {
  if (page >= static_cast<uint64_t>(num_pages)) return set_error(MTN_EINVAL, "free: page %u outside pool", page);
  if (!in_use[page]) return set_error(MTN_EINVAL, "Attempted to free a page that is not in use (page %u)", page);
  in_use[page] = 0;  // kv_pool.rs:45-46
  refcnt[page] = 0;
  free_stack.push_back(page);
  return MTN_OK;
}

int PagePool::retain(uint32_t page) {
  if (page >= static_cast<uint64_t>(num_pages) || !in_use[page])
    return set_error(MTN_EINVAL, "retain: page %u is not in use", page);
  ++refcnt[page];
  return MTN_OK;
}

int PagePool::release(uint32_t page, bool* freed) {
  if (freed) *freed = false;
  if (page >= static_cast<uint64_t>(num_pages) || !in_use[page])
    return set_error(MTN_EINVAL, "release: page %u is not in use", page);
  if (--refcnt[page] == 0) {
    if (freed) *freed = true;
    return free(page);
  }
  return MTN_OK;
}

// ----------------------------------------------------------------- RadixTree

RadixTree::RadixTree(int32_t ps, int64_t max_pages) : page_size(ps), max_pages(max_pages) {
  RadixNode r;
  r.last_used = tick();
  root = slab_insert(std::move(r));
}

uint64_t RadixTree::slab_insert(RadixNode&& n) {
  if (next_vacant == entries.size()) {
    entries.push_back(std::move(n));
    occupied.push_back(1);
    vacant_next.push_back(0);
    ++len;
    next_vacant = entries.size();
    return entries.size() - 1;
  }
  const uint64_t key = next_vacant;
  next_vacant = vacant_next[key];
  entries[key] = std::move(n);
  occupied[key] = 1;
  ++len;
  return key;
}

void RadixTree::slab_remove(uint64_t key) {
  entries[key] = RadixNode();
  occupied[key] = 0;
  vacant_next[key] = next_vacant;
  next_vacant = key;
  --len;
}

void RadixTree::push_evictable(uint64_t t, uint64_t id) { heap.push(HeapEntry{t, id}); }

int RadixTree::match_prefix(const uint32_t* tokens, int64_t n, int64_t* matched, std::vector<uint32_t>* pages,
                            std::vector<uint64_t>* nodes) {
  // radix_cache.rs:64-117.
  pages->clear();
  nodes->clear();
  int64_t offset = 0;
  uint64_t cur = root;
  while (offset < n) {
    const uint32_t first = tokens[offset];
    auto it = entries[cur].children.find(first);
    if (it == entries[cur].children.end()) break;
    const uint64_t child = it->second;
    const std::vector<uint32_t>& edge = entries[child].edge_tokens;
    int64_t match_len = 0;
    const int64_t lim = std::min<int64_t>(static_cast<int64_t>(edge.size()), n - offset);
    while (match_len < lim && edge[match_len] == tokens[offset + match_len]) ++match_len;
    if (match_len == 0) break;
    const int64_t full_pages = match_len / page_size;  // only count full pages
    if (full_pages == 0) break;
    if (full_pages > static_cast<int64_t>(entries[child].kv_pages.size()))
      return set_error(MTN_EINVAL, "radix invariant: node %llu holds %zu pages, match needs %lld",
                       (unsigned long long)child, entries[child].kv_pages.size(), (long long)full_pages);
    pages->insert(pages->end(), entries[child].kv_pages.begin(), entries[child].kv_pages.begin() + full_pages);
    offset += full_pages * page_size;
    const bool partial = match_len < static_cast<int64_t>(edge.size());
    nodes->push_back(child);
    entries[child].lock_ref += 1;
    entries[child].last_used = tick();
    if (partial) break;
    cur = child;
  }
  *matched = offset;
  return MTN_OK;
}

int RadixTree::insert_prefix(const uint32_t* tokens, int64_t n_tokens, const uint32_t* pages, int64_t n_pages,
                             std::vector<uint32_t>* evicted, std::vector<uint32_t>* adopted) {
  // radix_cache.rs:123-187.
  if (adopted) adopted->clear();
  const int64_t full_pages = n_pages;
  const int64_t full_tokens = full_pages * page_size;
  if (full_pages == 0) return MTN_OK;
  if (full_tokens > n_tokens)
    return set_error(MTN_EINVAL, "insert_prefix: %lld pages need %lld tokens, got %lld", (long long)n_pages,
                     (long long)full_tokens, (long long)n_tokens);
  if (total_pages + full_pages > max_pages) {
    std::vector<uint32_t> freed;
    evict_pages(total_pages + full_pages - max_pages, &freed);
    if (evicted) evicted->insert(evicted->end(), freed.begin(), freed.end());
  }
  int64_t offset = 0;
  uint64_t cur = root;
  while (offset < full_tokens) {
    const uint32_t first = tokens[offset];
    auto it = entries[cur].children.find(first);
    if (it == entries[cur].children.end()) {
      RadixNode leaf;
      leaf.edge_tokens.assign(tokens + offset, tokens + full_tokens);
      leaf.kv_pages.assign(pages + offset / page_size, pages + full_pages);
      leaf.parent = static_cast<int64_t>(cur);
      leaf.last_used = tick();
      const int64_t added = full_pages - offset / page_size;
      if (adopted) adopted->insert(adopted->end(), leaf.kv_pages.begin(), leaf.kv_pages.end());
      const uint64_t id = slab_insert(std::move(leaf));
      entries[cur].children[first] = id;
      total_pages += added;
      push_evictable(tick(), id);  // new leaf is immediately evictable
      break;
    }
    const uint64_t child = it->second;
    const int64_t edge_len = static_cast<int64_t>(entries[child].edge_tokens.size());
    int64_t match_len = 0;
    const int64_t lim = std::min<int64_t>(edge_len, full_tokens - offset);
    while (match_len < lim && entries[child].edge_tokens[match_len] == tokens[offset + match_len]) ++match_len;
    if (match_len == edge_len) {
      entries[child].last_used = tick();
      offset += edge_len;
      cur = child;
    } else {
      const uint64_t mid = split_edge(cur, child, match_len);
      offset += match_len;
      cur = mid;
    }
  }
  return MTN_OK;
}

uint64_t RadixTree::split_edge(uint64_t parent, uint64_t child, int64_t split_at) {
  // radix_cache.rs:191-223.
  const int64_t page_split = split_at / page_size;
  RadixNode& c = entries[child];
  std::vector<uint32_t> prefix_tokens(c.edge_tokens.begin(), c.edge_tokens.begin() + split_at);
  std::vector<uint32_t> suffix_tokens(c.edge_tokens.begin() + split_at, c.edge_tokens.end());
  const int64_t np = static_cast<int64_t>(c.kv_pages.size());
  const int64_t cut = std::min(page_split, np);
  std::vector<uint32_t> prefix_pages(c.kv_pages.begin(), c.kv_pages.begin() + cut);
  std::vector<uint32_t> suffix_pages(c.kv_pages.begin() + cut, c.kv_pages.end());
  const uint32_t first_suffix = suffix_tokens[0];
  const uint32_t first_prefix = prefix_tokens[0];
  c.edge_tokens = std::move(suffix_tokens);
  c.kv_pages = std::move(suffix_pages);
  RadixNode mid;
  mid.edge_tokens = std::move(prefix_tokens);
  mid.kv_pages = std::move(prefix_pages);
  mid.children[first_suffix] = child;
  mid.parent = static_cast<int64_t>(parent);
  mid.last_used = tick();
  const uint64_t mid_id = slab_insert(std::move(mid));
  entries[child].parent = static_cast<int64_t>(mid_id);
  entries[parent].children[first_prefix] = mid_id;
  return mid_id;
}

void RadixTree::unlock_nodes(const uint64_t* ids, int64_t n) {
  // radix_cache.rs:227-238.
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t id = ids[i];
    if (id >= entries.size() || !occupied[id]) continue;
    RadixNode& node = entries[id];
    node.lock_ref = std::max(node.lock_ref - 1, 0);
    node.last_used = tick();
    if (node.evictable()) push_evictable(node.last_used, id);
  }
}

void RadixTree::evict_pages(int64_t target, std::vector<uint32_t>* freed) {
  // radix_cache.rs:243-282.
  freed->clear();
  while (static_cast<int64_t>(freed->size()) < target) {
    uint64_t cand = 0;
    bool found = false;
    while (!heap.empty()) {
      const HeapEntry e = heap.top();
      heap.pop();
      if (e.id < entries.size() && occupied[e.id] && entries[e.id].evictable()) {
        cand = e.id;
        found = true;
        break;
      }
    }
    if (!found) return;
    std::vector<uint32_t> pages = std::move(entries[cand].kv_pages);
    entries[cand].kv_pages.clear();
    total_pages -= static_cast<int64_t>(pages.size());
    freed->insert(freed->end(), pages.begin(), pages.end());
    if (entries[cand].parent >= 0) {
      const uint64_t par = static_cast<uint64_t>(entries[cand].parent);
      if (!entries[cand].edge_tokens.empty()) {
        entries[par].children.erase(entries[cand].edge_tokens.front());
        if (entries[par].evictable()) push_evictable(entries[par].last_used, par);
      }
    }
    slab_remove(cand);
  }
}

int RadixTree::promote(const uint32_t* input_ids, int64_t n_input, int64_t device_len, const uint32_t* kv_pages,
                       int64_t n_kv_pages, std::vector<uint32_t>* evicted, std::vector<uint32_t>* adopted) {
  // radix_cache.rs:287-294.
  if (adopted) adopted->clear();
  const int64_t full_pages = device_len / page_size;
  const int64_t cache_tokens = full_pages * page_size;
  if (full_pages == 0) return MTN_OK;
  if (cache_tokens > n_input || full_pages > n_kv_pages)
    return set_error(MTN_EINVAL, "promote: device_len %lld exceeds %lld tokens / %lld pages", (long long)device_len,
                     (long long)n_input, (long long)n_kv_pages);
  return insert_prefix(input_ids, cache_tokens, kv_pages, full_pages, evicted, adopted);
}

}  // namespace mtn

// ===================================================================== C ABI

using mtn::set_error;

struct mtn_page_pool {
  mtn::PagePool impl;
  mtn_page_pool(int64_t n, int32_t ps) : impl(n, ps) {}
};

struct mtn_radix {
  mtn::RadixTree impl;
  mtn_radix(int32_t ps, int64_t mp) : impl(ps, mp) {}
};

extern "C" {

int mtn_page_pool_create(int64_t num_pages, int32_t page_size, mtn_page_pool** out) {
  MTN_CHECK_ARG(out != nullptr, "mtn_page_pool_create: null out");
  MTN_CHECK_ARG(num_pages >= 0 && num_pages <= (int64_t(1) << 32), "mtn_page_pool_create: bad num_pages");
  MTN_CHECK_ARG(page_size > 0, "mtn_page_pool_create: page_size must be positive");
  *out = new mtn_page_pool(num_pages, page_size);
  return MTN_OK;
}

void mtn_page_pool_destroy(mtn_page_pool* pool) { delete pool; }

int mtn_page_pool_allocate(mtn_page_pool* pool, uint64_t owner_hi, uint64_t owner_lo, uint32_t* page) {
  MTN_CHECK_ARG(pool && page, "mtn_page_pool_allocate: null argument");
  if (!pool->impl.allocate(owner_hi, owner_lo, page)) return set_error(MTN_ENOMEM, "out of KV pages");
  return MTN_OK;
}

int mtn_page_pool_free(mtn_page_pool* pool, uint32_t page) {
  MTN_CHECK_ARG(pool, "mtn_page_pool_free: null pool");
  return pool->impl.free(page);
}

int64_t mtn_page_pool_free_pages(const mtn_page_pool* pool) {
  return pool ? static_cast<int64_t>(pool->impl.free_stack.size()) : -1;
}

int64_t mtn_page_pool_total_pages(const mtn_page_pool* pool) { return pool ? pool->impl.num_pages : -1; }

int32_t mtn_page_pool_page_size(const mtn_page_pool* pool) { return pool ? pool->impl.page_size : -1; }

int mtn_page_pool_state(const mtn_page_pool* pool, uint32_t page, int32_t* in_use, uint64_t* owner_hi,
                        uint64_t* owner_lo) {
  MTN_CHECK_ARG(pool && in_use, "mtn_page_pool_state: null argument");
  MTN_CHECK_ARG(page < static_cast<uint64_t>(pool->impl.num_pages), "mtn_page_pool_state: page %u outside pool",
                page);
  *in_use = pool->impl.in_use[page];
  if (owner_hi) *owner_hi = pool->impl.owner_hi[page];
  if (owner_lo) *owner_lo = pool->impl.owner_lo[page];
  return MTN_OK;
}

int mtn_page_pool_retain(mtn_page_pool* pool, uint32_t page) {
  MTN_CHECK_ARG(pool, "mtn_page_pool_retain: null pool");
  return pool->impl.retain(page);
}

int mtn_page_pool_release(mtn_page_pool* pool, uint32_t page, int32_t* freed) {
  MTN_CHECK_ARG(pool, "mtn_page_pool_release: null pool");
  bool f = false;
  const int st = pool->impl.release(page, &f);
  if (freed) *freed = f ? 1 : 0;
  return st;
}

int32_t mtn_page_pool_refcount(const mtn_page_pool* pool, uint32_t page) {
  if (!pool || page >= static_cast<uint64_t>(pool->impl.num_pages)) return -1;
  return pool->impl.refcnt[page];
}

int mtn_radix_create(int32_t page_size, int64_t max_pages, mtn_radix** out) {
  MTN_CHECK_ARG(out != nullptr, "mtn_radix_create: null out");
  MTN_CHECK_ARG(page_size > 0 && max_pages >= 0, "mtn_radix_create: bad sizes");
  *out = new mtn_radix(page_size, max_pages);
  return MTN_OK;
}

void mtn_radix_destroy(mtn_radix* r) { delete r; }

int mtn_radix_match_prefix(mtn_radix* r, const uint32_t* tokens, int64_t n_tokens, int64_t* matched_len,
                           uint32_t* pages, int64_t* n_pages, uint64_t* nodes, int64_t* n_nodes) {
  MTN_CHECK_ARG(r && matched_len && n_pages && n_nodes, "mtn_radix_match_prefix: null argument");
  MTN_CHECK_ARG(n_tokens >= 0 && (tokens || n_tokens == 0), "mtn_radix_match_prefix: bad tokens");
  std::vector<uint32_t> pv;
  std::vector<uint64_t> nv;
  int64_t m = 0;
  const int st = r->impl.match_prefix(tokens, n_tokens, &m, &pv, &nv);
  if (st != MTN_OK) return st;
  if (static_cast<int64_t>(pv.size()) > *n_pages || static_cast<int64_t>(nv.size()) > *n_nodes) {
    r->impl.unlock_nodes(nv.data(), static_cast<int64_t>(nv.size()));
    return set_error(MTN_EINVAL, "mtn_radix_match_prefix: output buffers too small (%zu pages, %zu nodes)",
                     pv.size(), nv.size());
  }
  *matched_len = m;
  std::copy(pv.begin(), pv.end(), pages);
  std::copy(nv.begin(), nv.end(), nodes);
  *n_pages = static_cast<int64_t>(pv.size());
  *n_nodes = static_cast<int64_t>(nv.size());
  return MTN_OK;
}

int mtn_radix_insert_prefix(mtn_radix* r, const uint32_t* tokens, int64_t n_tokens, const uint32_t* pages,
                            int64_t n_pages, uint32_t* evicted, int64_t* n_evicted) {
  MTN_CHECK_ARG(r, "mtn_radix_insert_prefix: null radix");
  MTN_CHECK_ARG(n_tokens >= 0 && n_pages >= 0, "mtn_radix_insert_prefix: negative size");
  std::vector<uint32_t> ev;
  const int st = r->impl.insert_prefix(tokens, n_tokens, pages, n_pages, &ev, nullptr);
  if (evicted && n_evicted) {
    const int64_t cap = *n_evicted;
    const int64_t k = std::min<int64_t>(cap, static_cast<int64_t>(ev.size()));
    std::copy(ev.begin(), ev.begin() + k, evicted);
    *n_evicted = static_cast<int64_t>(ev.size());
  } else if (n_evicted) {
    *n_evicted = static_cast<int64_t>(ev.size());
  }
  return st;
}

int mtn_radix_unlock_nodes(mtn_radix* r, const uint64_t* nodes, int64_t n_nodes) {
  MTN_CHECK_ARG(r && (nodes || n_nodes == 0), "mtn_radix_unlock_nodes: null argument");
  r->impl.unlock_nodes(nodes, n_nodes);
  return MTN_OK;
}

int mtn_radix_evict_pages(mtn_radix* r, int64_t target, uint32_t* freed, int64_t* n_freed) {
  MTN_CHECK_ARG(r && n_freed, "mtn_radix_evict_pages: null argument");
  std::vector<uint32_t> f;
  r->impl.evict_pages(target, &f);
  const int64_t cap = *n_freed;
  if (static_cast<int64_t>(f.size()) > cap || (freed == nullptr && !f.empty())) {
    *n_freed = static_cast<int64_t>(f.size());
    return set_error(MTN_EINVAL, "mtn_radix_evict_pages: %zu pages freed but buffer holds %lld (pages are gone)",
                     f.size(), (long long)cap);
  }
  std::copy(f.begin(), f.end(), freed);
  *n_freed = static_cast<int64_t>(f.size());
  return MTN_OK;
}

int mtn_radix_promote(mtn_radix* r, const uint32_t* input_ids, int64_t n_input, int64_t device_len,
                      const uint32_t* kv_pages, int64_t n_kv_pages) {
  MTN_CHECK_ARG(r, "mtn_radix_promote: null radix");
  return r->impl.promote(input_ids, n_input, device_len, kv_pages, n_kv_pages, nullptr, nullptr);
}

int64_t mtn_radix_total_cached_pages(const mtn_radix* r) { return r ? r->impl.total_pages : -1; }

int64_t mtn_radix_num_nodes(const mtn_radix* r) { return r ? static_cast<int64_t>(r->impl.len) : -1; }

}  // extern "C"
