// Host-side mirror of the reference engine's page bookkeeping and scheduler
// (inference-engine/src/{kv_pool,radix_cache,prefill,decode,scheduler}.rs).
// Plain C++17; no CUDA.  Exposed through the C ABI in include/mitten_kv.h.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <deque>
#include <memory>
#include <queue>
#include <unordered_map>
#include <vector>

#include "../../include/mitten_kv.h"

namespace mtn {

int set_error(int code, const char* fmt, ...);

#ifndef MTN_CHECK_ARG
#define MTN_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::mtn::set_error(MTN_EINVAL, __VA_ARGS__); \
  } while (0)
#endif

// KvCachePool (kv_pool.rs:4-69) with per-page reference counts.
struct PagePool {
  int64_t num_pages;
  int32_t page_size;
  std::vector<uint32_t> free_stack;  // back() is the top of the stack
  std::vector<uint8_t> in_use;       // PageState::InUse
  std::vector<uint64_t> owner_hi, owner_lo;
  std::vector<int32_t> refcnt;

  PagePool(int64_t n, int32_t ps);
  bool allocate(uint64_t hi, uint64_t lo, uint32_t* page);
  int free(uint32_t page);
  int retain(uint32_t page);
  int release(uint32_t page, bool* freed);
  int64_t free_pages() const { return static_cast<int64_t>(free_stack.size()); }
};

struct RadixNode {
  std::vector<uint32_t> edge_tokens;
  std::vector<uint32_t> kv_pages;
  std::unordered_map<uint32_t, uint64_t> children;
  int64_t parent = -1;
  int32_t lock_ref = 0;
  uint64_t last_used = 0;
  bool leaf() const { return children.empty(); }
  bool evictable() const { return leaf() && lock_ref == 0 && !kv_pages.empty(); }  // radix_cache.rs:32-34
};

// RadixCache (radix_cache.rs:37-303).
struct RadixTree {
  struct HeapEntry {
    uint64_t t;
    uint64_t id;
  };
  // BinaryHeap<(Reverse<Instant>, NodeId)> is a max-heap: the top has the
  // oldest time, ties broken by the larger node id.
  struct HeapLess {
    bool operator()(const HeapEntry& a, const HeapEntry& b) const {
      if (a.t != b.t) return a.t > b.t;
      return a.id < b.id;
    }
  };

  int32_t page_size;
  int64_t max_pages;
  int64_t total_pages = 0;
  uint64_t clock = 0;
  // slab::Slab: dense entries, vacant ids reused most-recently-freed first.
  std::vector<RadixNode> entries;
  std::vector<uint8_t> occupied;
  std::vector<uint64_t> vacant_next;
  uint64_t next_vacant = 0;
  uint64_t len = 0;
  uint64_t root = 0;
  std::priority_queue<HeapEntry, std::vector<HeapEntry>, HeapLess> heap;

  RadixTree(int32_t ps, int64_t max_pages);
  uint64_t tick() { return ++clock; }
  uint64_t slab_insert(RadixNode&& n);
  void slab_remove(uint64_t key);
  void push_evictable(uint64_t t, uint64_t id);

  int match_prefix(const uint32_t* tokens, int64_t n, int64_t* matched, std::vector<uint32_t>* pages,
                   std::vector<uint64_t>* nodes);
  // `adopted` (may be null) receives the pages the tree took into a new leaf.
  int insert_prefix(const uint32_t* tokens, int64_t n_tokens, const uint32_t* pages, int64_t n_pages,
                    std::vector<uint32_t>* evicted, std::vector<uint32_t>* adopted);
  uint64_t split_edge(uint64_t parent, uint64_t child, int64_t split_at);
  void unlock_nodes(const uint64_t* ids, int64_t n);
  void evict_pages(int64_t target, std::vector<uint32_t>* freed);
  int promote(const uint32_t* input_ids, int64_t n_input, int64_t device_len, const uint32_t* kv_pages,
              int64_t n_kv_pages, std::vector<uint32_t>* evicted, std::vector<uint32_t>* adopted);
};

}  // namespace mtn
