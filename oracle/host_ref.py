"""TEST INFRASTRUCTURE -- pure-Python restatement of the reference engine's
page bookkeeping, used only by the test suite as the checker for the C++
host mirror in mitten_b200/csrc (never imported by the product path).

Follows tianhaoz95/mitten line by line:
  KvCachePool ............. inference-engine/src/kv_pool.rs:4-69
  RadixCache .............. inference-engine/src/radix_cache.rs:37-303
  PrefillAdder ............ inference-engine/src/prefill.rs:6-115
  collect_decode_requests . inference-engine/src/decode.rs:6-47
  schedule_batch etc. ..... inference-engine/src/scheduler.rs:8-223
Pinned by the reference's own unit tests (kv_pool.rs:104-161,
radix_cache.rs:305-424), ported in tests/test_reference_kats.py.

Two details the Rust leaves to its dependencies are made explicit:
  * `slab::Slab` hands out the most recently vacated key first;
  * `Instant::now()` becomes a logical clock that ticks at every call site,
    so eviction ties never depend on timer resolution.
"""
from __future__ import annotations

import heapq
import math
import struct
from collections import deque
from dataclasses import dataclass, field


class RefError(Exception):
    """Where the Rust would panic (debug_assert!, slice out of range)."""


# ------------------------------------------------------------------ kv_pool.rs
class KvCachePool:
    def __init__(self, num_pages: int, page_size: int):  # kv_pool.rs:18-27
        self.num_pages = num_pages
        self.page_size = page_size
        self.free_list = list(range(num_pages))[::-1]  # used as a stack
        self.states: list = [None] * num_pages          # None = Free, else owner

    def allocate(self, owner):  # kv_pool.rs:30-37
        if not self.free_list:
            return None
        page = self.free_list.pop()
        self.states[page] = owner
        return page

    def free(self, page: int):  # kv_pool.rs:40-47 (debug build semantics)
        if self.states[page] is None:
            raise RefError("Attempted to free a page that is not in use")
        self.states[page] = None
        self.free_list.append(page)

    def free_pages(self) -> int:
        return len(self.free_list)

    def total_pages(self) -> int:
        return self.num_pages

    @staticmethod
    def required_bytes(num_pages, page_size, num_layers, num_kv_heads, head_dim, dtype_bytes):  # :58-68
        return 2 * num_layers * num_pages * page_size * num_kv_heads * head_dim * dtype_bytes


# -------------------------------------------------------------- radix_cache.rs
@dataclass
class RadixNode:
    edge_tokens: list
    kv_pages: list
    children: dict = field(default_factory=dict)
    parent: int | None = None
    lock_ref: int = 0
    last_used: int = 0

    def is_leaf(self):
        return not self.children

    def is_evictable(self):  # radix_cache.rs:32-34
        return self.is_leaf() and self.lock_ref == 0 and len(self.kv_pages) > 0


class _Slab:
    """slab::Slab: insert reuses the most recently removed key."""

    def __init__(self):
        self.entries: list = []
        self.vacant_next: list = []
        self.next = 0
        self.len = 0

    def insert(self, v) -> int:
        if self.next == len(self.entries):
            self.entries.append(v)
            self.vacant_next.append(None)
            self.next = len(self.entries)
            key = len(self.entries) - 1
        else:
            key = self.next
            self.next = self.vacant_next[key]
            self.entries[key] = v
        self.len += 1
        return key

    def remove(self, key):
        self.entries[key] = None
        self.vacant_next[key] = self.next
        self.next = key
        self.len -= 1

    def contains(self, key):
        return 0 <= key < len(self.entries) and self.entries[key] is not None

    def __getitem__(self, key) -> RadixNode:
        v = self.entries[key]
        if v is None:
            raise RefError(f"invalid slab key {key}")
        return v


class RadixCache:
    def __init__(self, page_size: int, max_pages: int):  # radix_cache.rs:48-59
        self.clock = 0
        self.nodes = _Slab()
        self.root = self.nodes.insert(RadixNode([], [], last_used=self._now()))
        # BinaryHeap<(Reverse<Instant>, NodeId)>: max-heap => pop oldest time,
        # ties -> larger node id.  heapq is a min-heap on (t, -id).
        self.evictable: list = []
        self.page_size = page_size
        self.total_pages = 0
        self.max_pages = max_pages

    def _now(self) -> int:
        self.clock += 1
        return self.clock

    def _push(self, t, nid):
        heapq.heappush(self.evictable, (t, -nid))

    def match_prefix(self, tokens):  # radix_cache.rs:64-117
        matched_pages, matched_nodes = [], []
        offset, cur = 0, self.root
        while True:
            if offset >= len(tokens):
                break
            first = tokens[offset]
            child_id = self.nodes[cur].children.get(first)
            if child_id is None:
                break
            edge = self.nodes[child_id].edge_tokens
            remaining = tokens[offset:]
            match_len = 0
            for a, b in zip(edge, remaining):
                if a != b:
                    break
                match_len += 1
            if match_len == 0:
                break
            full_pages = match_len // self.page_size
            if full_pages == 0:
                break
            pages = self.nodes[child_id].kv_pages
            if full_pages > len(pages):
                raise RefError("slice index out of range in match_prefix")
            matched_pages.extend(pages[:full_pages])
            offset += full_pages * self.page_size
            is_partial = match_len < len(edge)
            matched_nodes.append(child_id)
            self.nodes[child_id].lock_ref += 1
            self.nodes[child_id].last_used = self._now()
            if is_partial:
                break
            cur = child_id
        return offset, matched_pages, matched_nodes

    def insert_prefix(self, tokens, pages):  # radix_cache.rs:123-187
        """Returns the pages evict_pages freed (the Rust discards them)."""
        full_pages = len(pages)
        full_tokens = full_pages * self.page_size
        evicted = []
        if full_pages == 0:
            return evicted
        if full_tokens > len(tokens):
            raise RefError("range end index out of range in insert_prefix")
        tokens = tokens[:full_tokens]
        if self.total_pages + full_pages > self.max_pages:
            evicted = self.evict_pages(self.total_pages + full_pages - self.max_pages)
        offset, cur = 0, self.root
        while True:
            if offset >= len(tokens):
                break
            first = tokens[offset]
            child_id = self.nodes[cur].children.get(first)
            if child_id is None:
                new_id = self.nodes.insert(RadixNode(
                    edge_tokens=list(tokens[offset:]),
                    kv_pages=list(pages[offset // self.page_size:]),
                    parent=cur, lock_ref=0, last_used=self._now()))
                self.nodes[cur].children[first] = new_id
                self.total_pages += len(pages[offset // self.page_size:])
                self._push(self._now(), new_id)
                break
            edge_len = len(self.nodes[child_id].edge_tokens)
            match_len = 0
            for a, b in zip(self.nodes[child_id].edge_tokens, tokens[offset:]):
                if a != b:
                    break
                match_len += 1
            if match_len == edge_len:
                self.nodes[child_id].last_used = self._now()
                offset += edge_len
                cur = child_id
            else:
                mid = self._split_edge(cur, child_id, match_len)
                offset += match_len
                cur = mid
        return evicted

    def _split_edge(self, parent, child, split_at):  # radix_cache.rs:191-223
        page_split = split_at // self.page_size
        c = self.nodes[child]
        prefix_tokens, suffix_tokens = c.edge_tokens[:split_at], c.edge_tokens[split_at:]
        prefix_pages, suffix_pages = c.kv_pages[:page_split], c.kv_pages[page_split:]
        first_suffix, first_prefix = suffix_tokens[0], prefix_tokens[0]
        c.edge_tokens, c.kv_pages = suffix_tokens, suffix_pages
        mid_id = self.nodes.insert(RadixNode(edge_tokens=prefix_tokens, kv_pages=prefix_pages,
                                             children={first_suffix: child}, parent=parent,
                                             lock_ref=0, last_used=self._now()))
        self.nodes[child].parent = mid_id
        self.nodes[parent].children[first_prefix] = mid_id
        return mid_id

    def unlock_nodes(self, node_ids):  # radix_cache.rs:227-238
        for nid in node_ids:
            if not self.nodes.contains(nid):
                continue
            node = self.nodes[nid]
            node.lock_ref = max(node.lock_ref - 1, 0)
            node.last_used = self._now()
            if node.is_evictable():
                self._push(node.last_used, nid)

    def evict_pages(self, target_pages):  # radix_cache.rs:243-282
        freed = []
        while len(freed) < target_pages:
            cand = None
            while self.evictable:
                _, neg = heapq.heappop(self.evictable)
                nid = -neg
                if self.nodes.contains(nid) and self.nodes[nid].is_evictable():
                    cand = nid
                    break
            if cand is None:
                return freed
            pages = self.nodes[cand].kv_pages
            self.nodes[cand].kv_pages = []
            self.total_pages -= len(pages)
            freed.extend(pages)
            parent = self.nodes[cand].parent
            if parent is not None and self.nodes[cand].edge_tokens:
                t = self.nodes[cand].edge_tokens[0]
                self.nodes[parent].children.pop(t, None)
                if self.nodes[parent].is_evictable():
                    self._push(self.nodes[parent].last_used, parent)
            self.nodes.remove(cand)
        return freed

    def promote_request(self, input_ids, device_len, kv_pages):  # radix_cache.rs:287-294
        full_pages = device_len // self.page_size
        cache_tokens = full_pages * self.page_size
        if full_pages == 0:
            return []
        if full_pages > len(kv_pages) or cache_tokens > len(input_ids):
            raise RefError("slice index out of range in promote_request")
        return self.insert_prefix(input_ids[:cache_tokens], kv_pages[:full_pages])

    def total_cached_pages(self):
        return self.total_pages

    def num_nodes(self):
        return self.nodes.len


# ----------------------------------------------- prefill.rs / decode.rs / scheduler.rs
WAITING, PREFILLING, DECODING, DONE, ABORTED = range(5)


@dataclass
class Request:  # inference-backend/src/request.rs:41-101
    id: int
    input_ids: list
    temperature: float = 1.0
    max_new_tokens: int = 512
    state: int = WAITING
    cached_len: int = 0
    device_len: int = 0
    extend_len: int = 0
    kv_pages: list = field(default_factory=list)
    output_ids: list = field(default_factory=list)
    locked_nodes: list = field(default_factory=list)


@dataclass
class Batch:  # inference-backend/src/batch.rs:7-36
    phase: int
    requests: list
    input_ids: list
    position_ids: list
    page_table: list


def sample_token(logits, temperature: float) -> int:  # scheduler.rs:186-223
    if temperature <= 0.0:
        import numpy as np

        row = np.asarray(logits, dtype=np.float32)
        if not np.isnan(row).any():
            # Without NaNs the first strict maximum is numpy's first argmax.
            return int(np.argmax(row)) if row.size else 0
        max_val, max_idx = -math.inf, 0
        for i, v in enumerate(logits):
            if v > max_val:
                max_val, max_idx = v, i
        return max_idx
    import numpy as np

    row = np.asarray(logits, dtype=np.float32)
    h = 0
    for v in row[:100]:
        bits = struct.unpack("<I", struct.pack("<f", float(v)))[0]
        h = (h * 31 + bits) & 0xFFFFFFFFFFFFFFFF
    rand_val = np.float32(h % 1000) / np.float32(1000.0)
    e = np.exp(row / np.float32(temperature), dtype=np.float32)
    s = np.float32(0.0)
    for x in e:
        s = np.float32(s + x)
    cum = np.float32(0.0)
    for i, x in enumerate(e):
        cum = np.float32(cum + np.float32(x / s))
        if rand_val <= cum:
            return i
    return len(logits) - 1


class EngineContext:
    """EngineContext (engine_loop.rs:11-21) with the scheduler functions."""

    def __init__(self, num_pages, page_size, max_prefill_tokens_per_iter, max_decode_batch_size,
                 radix_max_pages=None, eos_token_ids=(99,)):
        self.kv_pool = KvCachePool(num_pages, page_size)
        self.radix_cache = RadixCache(page_size, num_pages if radix_max_pages is None else radix_max_pages)
        self.waiting: deque = deque()
        self.prefilling: list = []
        self.decoding: list = []
        self.max_prefill = max_prefill_tokens_per_iter
        self.max_decode = max_decode_batch_size
        self.eos = list(eos_token_ids)

    # decode.rs:6-47
    def collect_decode_requests(self):
        out, i = [], 0
        while i < len(self.decoding):
            r = self.decoding[i]
            if r.state == DECODING:
                out.append(r)
                i += 1
            elif r.state in (DONE, ABORTED):
                self.radix_cache.unlock_nodes(r.locked_nodes)
                r.locked_nodes = []
                for p in r.kv_pages:
                    self.kv_pool.free(p)
                r.kv_pages = []
                self.decoding.pop(i)
            else:
                i += 1
        return out[: self.max_decode]

    # prefill.rs:99-114
    @staticmethod
    def _chunk(r, budget, used):
        remaining = len(r.input_ids) - r.device_len
        if remaining == 0:
            return 0, used
        chunk = min(remaining, budget - used)
        if chunk > 0:
            r.extend_len = chunk
            return chunk, used + chunk
        return None, used

    # prefill.rs:21-97
    def prefill_run(self, budget):
        added, used = [], 0
        for r in list(self.prefilling):
            if used >= budget:
                break
            c, used = self._chunk(r, budget, used)
            if c:
                added.append(r)
        ps = self.kv_pool.page_size
        while used < budget and self.waiting:
            r = self.waiting[0]
            pages_needed = (len(r.input_ids) + ps - 1) // ps
            if self.kv_pool.free_pages() < pages_needed:
                deficit = pages_needed - self.kv_pool.free_pages()
                for p in self.radix_cache.evict_pages(deficit):
                    self.kv_pool.free(p)
                if self.kv_pool.free_pages() < pages_needed:
                    break
            self.waiting.popleft()
            cached, pages, nodes = self.radix_cache.match_prefix(r.input_ids)
            r.cached_len, r.device_len, r.locked_nodes, r.kv_pages = cached, cached, nodes, list(pages)
            while len(r.kv_pages) < pages_needed:
                p = self.kv_pool.allocate(r.id)
                if p is None:
                    raise RefError("KV pool exhausted despite check")
                r.kv_pages.append(p)
            r.state = PREFILLING
            self.prefilling.append(r)
            c, used = self._chunk(r, budget, used)
            if c:
                added.append(r)
        return added

    # scheduler.rs:8-27
    def schedule_batch(self):
        dec = self.collect_decode_requests()
        budget = max(0, self.max_prefill - len(dec))
        pre = self.prefill_run(budget)
        if not dec and not pre:
            return None
        return self.assemble_batch(pre, dec)

    # scheduler.rs:29-77
    @staticmethod
    def assemble_batch(pre, dec):
        input_ids, position_ids, page_table, reqs = [], [], [], []
        for r in pre:
            s, e = r.device_len, r.device_len + r.extend_len
            input_ids.extend(r.input_ids[s:e])
            position_ids.extend(range(s, e))
            page_table.append(list(r.kv_pages))
            reqs.append(r)
        for r in dec:
            last = r.output_ids[-1] if r.output_ids else r.input_ids[-1]
            input_ids.append(last)
            position_ids.append(r.device_len)
            page_table.append(list(r.kv_pages))
            reqs.append(r)
        phase = 0 if (pre and not dec) else (1 if (dec and not pre) else 2)
        return Batch(phase, reqs, input_ids, position_ids, page_table)

    # engine_loop.rs:47-57: a failed forward marks every request of the batch
    # Aborted; pages and radix locks are released later by
    # collect_decode_requests (decode.rs:20-33) for requests in `decoding`.
    @staticmethod
    def abort_batch(batch: Batch):
        for r in batch.requests:
            r.state = ABORTED

    # scheduler.rs:79-184
    def process_and_transition(self, batch: Batch, logits_rows):
        row = 0
        for r in batch.requests:
            if r.state == PREFILLING:
                r.device_len += r.extend_len
                r.extend_len = 0
                if r.device_len == len(r.input_ids):
                    tok = sample_token(logits_rows[row], r.temperature)
                    r.output_ids.append(tok)
                    r.state = DECODING
                    if r in self.prefilling:
                        self.prefilling.remove(r)
                    self.decoding.append(r)
                    self.radix_cache.promote_request(r.input_ids, r.device_len, r.kv_pages)
                row += 1
            elif r.state == DECODING:
                tok = sample_token(logits_rows[row], r.temperature)
                r.output_ids.append(tok)
                r.device_len += 1
                done = tok in self.eos or len(r.output_ids) >= r.max_new_tokens
                if done:
                    r.state = DONE
                    self.radix_cache.unlock_nodes(r.locked_nodes)
                    r.locked_nodes = []
                    for p in r.kv_pages:
                        self.kv_pool.free(p)
                    r.kv_pages = []
                    if r in self.decoding:
                        self.decoding.remove(r)
                row += 1


# ---------------------------------------------------------------- stub.rs
def stub_logits(requests, vocab_size: int, eos_token_ids, forced_tokens=(), rng_seed: int = 42):
    """StubBackend::forward (inference-backend/src/stub.rs:32-67): one row per
    request, all zeros except 10.0 at the token it forces -- forced_tokens
    indexed by the request's output length (EOS past their end), or, with no
    forced tokens, (rng_seed ^ low 64 bits of the id ^ step) % vocab_size."""
    import numpy as np

    data = np.zeros((len(requests), vocab_size), dtype=np.float32)
    for i, r in enumerate(requests):
        idx = len(r.output_ids)
        if forced_tokens:
            tok = forced_tokens[idx] if idx < len(forced_tokens) else eos_token_ids[0]
        else:
            tok = (rng_seed ^ (int(r.id) & 0xFFFFFFFFFFFFFFFF) ^ idx) % vocab_size
        data[i, int(tok) % vocab_size] = 10.0
    return data
