"""Refcount mode (MTN_SCHED_REFCOUNT), the page lifecycle the device engine
runs, checked on the CPU.  Every place it deliberately differs from the
reference scheduler is named by a test below, next to what the reference
(oracle.host_ref / reference mode of the mirror) does on the same stream:

  * a prompt whose every page is cached still recomputes its last token
    (match on input_len - 1 tokens; the reference's admission at
    prefill.rs:60-70 matches all of it and the request never runs);
  * decode grows a request by one page when its last page is full (the
    reference never allocates after admission, scheduler.rs:133);
  * pages carry reference counts, so a finished request or an eviction
    returns only its own reference (the reference frees radix-shared pages
    on Done, scheduler.rs:164-172, and hands evicted pages of live requests
    to new ones, radix_cache.rs:243-294);
  * prefix forks share a parent's partially filled last page, and the first
    writer gets a private copy (copy-on-write pairs in the batch).

At every iteration: each page's count equals the live requests listing it
plus the radix cache's references, free pages = total - pages in use, every
batch row's seq_len fits its page table, and copy-on-write pairs read a
page the writer shared and write a page nobody else holds.  Streams end
with no leaked page.
"""
from __future__ import annotations

from collections import Counter

import numpy as np
import pytest

import oracle.host_ref as ref
from mitten_b200 import _lib, host

LIVE = (_lib.MTN_REQ_WAITING, _lib.MTN_REQ_PREFILLING, _lib.MTN_REQ_DECODING)


class Engine:
    """The refcount scheduler driven with host-chosen tokens (no EOS)."""

    def __init__(self, num_pages, page_size, budget=256, max_decode=16, radix_max_pages=None, mode=None):
        self.s = host.Scheduler(num_pages, page_size, budget, max_decode, radix_max_pages,
                                mode=_lib.MTN_SCHED_REFCOUNT if mode is None else mode, eos_token_ids=(10 ** 6,))
        self.num_pages, self.ps = num_pages, page_size
        self.ids: list[int] = []
        self.cow_pairs: list[tuple[int, int, int]] = []  # (request, src, dst)
        self.batches = 0

    def add(self, rid, toks, max_new=4):
        self.s.add_request(rid, toks, 0.0, max_new)
        self.ids.append(rid)

    def fork(self, parent, rid, suffix, max_new=4):
        self.s.fork(parent, rid, suffix, 0.0, max_new)
        self.ids.append(rid)

    def invariants(self):
        holders = Counter()
        for rid in self.ids:
            if self.s.request_info(rid)["state"] in LIVE:
                holders.update(self.s.request_pages(rid))
        holders.update(self.s.tree_pages())
        used = 0
        for p in range(self.num_pages):
            rc = self.s.page_refcount(p)
            assert rc == holders.get(p, 0), (p, rc, holders.get(p, 0))
            used += rc > 0
        assert self.s.free_pages() == self.num_pages - used

    def step(self):
        b = self.s.schedule()
        self.invariants()
        if b is None:
            return None
        self.batches += 1
        for i in range(b.n_reqs):
            npg = b.kv_indptr[i + 1] - b.kv_indptr[i]
            assert b.seq_lens[i] <= npg * self.ps, "a row's keys must fit its page table"
        owner = {}
        for i in range(b.n_reqs):
            for p in b.page_table()[i]:
                owner.setdefault(p, []).append(int(b.req_ids[i]))
        for src, dst in zip(b.cow_src.tolist(), b.cow_dst.tolist()):
            (writer,) = owner[dst]  # the copy belongs to exactly one row
            assert src not in self.s.request_pages(writer)
            self.cow_pairs.append((writer, src, dst))
        # every row writes positions [seq_len - q_len, seq_len): those pages
        # must be held by that row alone
        for i in range(b.n_reqs):
            q = b.qo_indptr[i + 1] - b.qo_indptr[i]
            pages = b.page_table()[i]
            for pos in range(b.seq_lens[i] - q, b.seq_lens[i]):
                assert self.s.page_refcount(pages[pos // self.ps]) == 1, "a row writes into a shared page"
        self.s.process_tokens(np.full(b.n_reqs, 7, np.uint32))
        self.invariants()
        return b

    def drain(self, max_iters=500):
        for _ in range(max_iters):
            if self.step() is None and self.s.num_active() == 0:
                return
        raise AssertionError("did not drain")


def test_fully_cached_prompt_recomputes_last_token():
    """Refcount: match on input_len - 1 tokens, so a prompt whose pages are all
    cached still computes its last token and samples.  Reference: cached_len =
    input_len, the prefill chunk is empty (prefill.rs:99-104) and the request
    stays Prefilling forever."""
    toks = list(range(8))  # two full pages of 4
    # reference, oracle and mirror agree that request 2 never runs
    ctx = ref.EngineContext(32, 4, 64, 8)
    mir = host.Scheduler(32, 4, 64, 8, mode=_lib.MTN_SCHED_REFERENCE)
    r1, r2 = ref.Request(1, toks, temperature=0.0, max_new_tokens=20), ref.Request(2, toks, 0.0, 20)
    ctx.waiting.append(r1)
    mir.add_request(1, toks, 0.0, 20)
    for it in range(12):
        if it == 2:
            ctx.waiting.append(r2)
            mir.add_request(2, toks, 0.0, 20)
        b = ctx.schedule_batch()
        mb = mir.schedule()
        rows = np.zeros((len(b.requests), 16), np.float32)
        rows[:, 3] = 1.0
        ctx.process_and_transition(b, rows)
        mir.process_logits(rows)
    assert r2.cached_len == 8 and r2.state == ref.PREFILLING and r2.output_ids == []
    assert mir.request_info(2)["state"] == _lib.MTN_REQ_PREFILLING and mir.request_output(2) == []
    # refcount: request 2 reuses one page, recomputes tokens 4..7 and finishes
    e = Engine(32, 4)
    e.add(1, toks, max_new=20)
    e.step()
    e.step()
    e.add(2, toks, max_new=3)
    e.drain()
    assert e.s.request_info(2)["cached_len"] == 4
    assert e.s.request_info(2)["state"] == _lib.MTN_REQ_DONE and len(e.s.request_output(2)) == 3


def test_decode_time_page_growth():
    """Refcount: a decoding request gets a new page when its last one is full
    (row A9); every decode row's seq_len fits its table.  Reference: the table
    keeps its admission size while device_len grows past it."""
    e = Engine(32, 4)
    e.add(1, [5, 6, 7, 8, 9], max_new=12)
    seen = []
    while True:
        b = e.step()
        if b is None:
            break
        seen.append((int(b.seq_lens[0]), int(b.kv_indptr[1])))
    assert all(n == (L + 3) // 4 for L, n in seen)
    assert seen[-1] == (16, 4)
    mir = host.Scheduler(32, 4, 64, 8, mode=_lib.MTN_SCHED_REFERENCE)
    mir.add_request(1, [5, 6, 7, 8, 9], 0.0, 12)
    last = None
    while (b := mir.schedule()) is not None:
        last = (int(b.seq_lens[0]), int(b.kv_indptr[1]))
        mir.process_tokens([7])
    assert last == (16, 2)  # 16 keys against two pages of 4


def test_shared_prefix_has_no_double_free():
    """The lockstep stream on which the reference double-frees shared prefix
    pages (tests/test_sched_lockstep.py::test_shared_prefix_lockstep) runs to
    completion here; afterwards only the radix cache holds pages."""
    prefix = list(range(100, 112))
    e = Engine(64, 4)
    e.add(1, prefix + [7, 8, 9, 10, 11], max_new=12)
    e.step()
    e.step()
    e.add(2, prefix + [20, 21], max_new=4)
    e.add(3, prefix[:8] + [30, 31, 32, 33, 34], max_new=5)
    e.step()
    e.add(4, prefix + [40], max_new=3)
    e.drain()
    assert [e.s.request_info(i)["cached_len"] for i in (2, 3, 4)] == [12, 8, 12]
    tree = e.s.tree_pages()
    assert len(tree) == len(set(tree)) == e.s.cached_pages()
    assert all(e.s.page_refcount(p) == 1 for p in tree)
    assert e.s.free_pages() + len(tree) == 64


def test_eviction_returns_only_the_tree_reference():
    """The reference's eviction stream (test_eviction_pressure_lockstep): the
    tree gives up its reference to request 1's pages, but they stay with
    request 1, so request 2 waits until request 1 finishes instead of
    receiving pages in use."""
    e = Engine(12, 4)
    e.add(1, list(range(8)), max_new=6)
    e.step()
    e.step()
    e.add(2, list(range(50, 94)), max_new=3)  # 11 pages
    while e.s.request_info(1)["state"] != _lib.MTN_REQ_DONE:
        e.step()
        if e.s.request_info(2)["state"] != _lib.MTN_REQ_WAITING:
            assert not set(e.s.request_pages(2)) & set(e.s.request_pages(1))
    e.drain()
    assert e.s.request_info(2)["state"] == _lib.MTN_REQ_DONE


def test_fork_shares_partial_page_and_copies_on_write():
    """A parent with a 10-token prompt (pages of 4: two full, one holding 2
    tokens) forks three children.  The first schedule after the forks puts
    the parent's decode write and the children's suffixes into the shared
    partial page: every writer but the last holder gets a copy-on-write pair,
    each writer at most once, and afterwards no one writes a shared page."""
    e = Engine(64, 4)
    parent_prompt = list(range(200, 210))
    e.add(1, parent_prompt, max_new=10)
    e.step()  # prefill the parent
    par_pages = e.s.request_pages(1)
    assert len(par_pages) == 3
    for k, suffix in enumerate(([1, 2, 3], [4], [5, 6, 7, 8, 9, 10, 11])):
        e.fork(1, 10 + k, suffix, max_new=3)
        info = e.s.request_info(10 + k)
        assert info["cached_len"] == 10 and info["device_len"] == 10
        assert e.s.request_pages(10 + k) == par_pages
    assert e.s.page_refcount(par_pages[2]) == 4 and e.s.page_refcount(par_pages[0]) == 5  # + the tree
    b = e.step()
    assert b.n_reqs == 4 and len(b.cow_src) == 3
    assert all(src == par_pages[2] for src in b.cow_src.tolist())
    writers = [w for w, _, _ in e.cow_pairs]
    assert len(writers) == len(set(writers)) == 3
    # one of the four sharers keeps the original page, now its only writer
    # (the radix cache may hold it too once that sharer's prompt is promoted)
    holders = [r for r in (1, 10, 11, 12) if par_pages[2] in e.s.request_pages(r)]
    in_tree = par_pages[2] in e.s.tree_pages()
    assert len(holders) == 1 and e.s.page_refcount(par_pages[2]) == 1 + in_tree
    e.drain()
    assert all(e.s.request_info(r)["state"] == _lib.MTN_REQ_DONE for r in (1, 10, 11, 12))
    assert e.s.free_pages() + len(e.s.tree_pages()) == 64


def test_fork_rejections():
    e = Engine(16, 4)
    e.add(1, [1, 2, 3], max_new=2)
    with pytest.raises(_lib.MittenError, match="not finished its prompt"):
        e.fork(1, 2, [4])
    e.step()
    with pytest.raises(_lib.MittenError, match="at least one token"):
        e.s.fork(1, 3, [], 0.0, 2)
    with pytest.raises(_lib.MittenError, match="duplicate"):
        e.fork(1, 1, [4])
    ref_mode = host.Scheduler(16, 4, mode=_lib.MTN_SCHED_REFERENCE)
    ref_mode.add_request(1, [1, 2, 3], 0.0, 2)
    ref_mode.schedule()
    ref_mode.process_tokens([5])
    with pytest.raises(_lib.MittenError, match="REFCOUNT"):
        ref_mode.fork(1, 2, [4])


@pytest.mark.parametrize("seed", range(12))
def test_random_streams_no_leak(seed):
    """Random streams with shared prefixes, forks, small pools (evictions,
    admission waits) and small budgets (chunking): invariants hold at every
    iteration and all pages come back at the end."""
    rng = np.random.default_rng(500 + seed)
    ps = int(rng.choice([2, 4, 8, 16]))
    num_pages = int(rng.integers(32, 128))
    e = Engine(num_pages, ps, budget=int(rng.integers(8, 64)), max_decode=int(rng.integers(2, 10)),
               radix_max_pages=int(rng.integers(4, num_pages)))
    bases = [rng.integers(0, 50, int(rng.integers(ps, 5 * ps))).tolist() for _ in range(3)]
    rid = 1
    for it in range(60):
        if it < 40 and rng.random() < 0.4:
            base = bases[int(rng.integers(0, 3))]
            toks = base[: int(rng.integers(1, len(base) + 1))] + rng.integers(0, 50, int(rng.integers(0, 8))).tolist()
            if (len(toks) + 16) // ps + 2 < num_pages // 3:
                e.add(rid, toks, max_new=int(rng.integers(1, 12)))
                rid += 1
        if it < 40 and rng.random() < 0.2:
            parents = [r for r in e.ids if e.s.request_info(r)["state"] == _lib.MTN_REQ_DECODING]
            if parents:
                p = parents[int(rng.integers(0, len(parents)))]
                n_prompt = e.s.request_info(p)["device_len"]
                if (n_prompt + 24) // ps + 2 < num_pages // 3:
                    e.fork(p, rid, rng.integers(0, 50, int(rng.integers(1, 6))).tolist(), max_new=int(rng.integers(1, 8)))
                    rid += 1
        e.step()
    e.drain()
    assert all(e.s.request_info(r)["state"] in (_lib.MTN_REQ_DONE, _lib.MTN_REQ_ABORTED) for r in e.ids)
    tree = e.s.tree_pages()
    assert e.s.free_pages() + len(set(tree)) == num_pages


def test_export_import_handoff():
    """Prefill -> decode handoff (KvHandoff): a decoding request exported from
    one scheduler leaves it with its references returned, and an import into
    another admits it straight into Decoding on fresh pages, which then grow
    as it decodes; both schedulers keep their page invariants."""
    a, b = Engine(64, 4), Engine(64, 4)
    a.add(1, list(range(30, 41)), max_new=6)  # 11 prompt tokens: 3 pages
    a.step()  # prefill: first token out, Decoding
    info = a.s.request_info(1)
    assert info["state"] == _lib.MTN_REQ_DECODING and info["device_len"] == 11
    h = a.s.export_request(1)
    assert h["device_len"] == 11 and len(h["pages"]) == 3 and h["outputs"] == [7]
    assert a.s.request_info(1)["state"] == _lib.MTN_REQ_DONE and a.s.request_pages(1) == []
    a.invariants()
    assert a.s.free_pages() + len(a.s.tree_pages()) == 64
    pages = b.s.import_request(1, list(range(30, 41)), h["outputs"], h["device_len"], 0.0, 6)
    b.ids.append(1)
    assert len(pages) == 3 and b.s.request_info(1)["state"] == _lib.MTN_REQ_DECODING
    b.invariants()
    seen = []
    while (bt := b.step()) is not None:
        seen.append((int(bt.seq_lens[0]), int(bt.input_ids[0]), int(bt.position_ids[0])))
    assert seen[0] == (12, 7, 11)  # the handed-over token is decoded at position 11
    assert b.s.request_output(1) == [7] * 6 and b.s.free_pages() + len(b.s.tree_pages()) == 64


def test_export_import_rejections():
    a = Engine(8, 4)
    a.add(1, [1, 2, 3], max_new=3)
    with pytest.raises(_lib.MittenError, match="not decoding"):
        a.s.export_request(1)
    with pytest.raises(_lib.MittenError, match="inconsistent"):
        a.s.import_request(2, [1, 2, 3], [5], 9, 0.0, 3)  # device_len past prompt + outputs
    with pytest.raises(_lib.OutOfKvPages):
        a.s.import_request(3, list(range(40)), [5], 40, 0.0, 3)  # 10 pages in an 8-page pool
    a.invariants()
    assert a.s.free_pages() == 8
