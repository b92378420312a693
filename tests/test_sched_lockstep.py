"""The C++ scheduler mirror (mitten_b200.host.Scheduler, reference mode) run in
lockstep with the oracle restatement of the reference engine
(oracle.host_ref.EngineContext) on the same request streams, with logits
from the reference's StubBackend (inference-backend/src/stub.rs:32-67).

Every iteration compares the scheduled Batch (scheduler.rs:29-77: request
order, input_ids, position_ids, page tables as CSR, phase) and, after
process_and_transition (scheduler.rs:79-184), every request's state,
device_len, cached_len, kv_pages and output_ids, the pool's free-page count
and the radix cache's page count.  Streams cover config 1's prompts, a
shared prefix, a small prefill budget that forces chunking, pool pressure
that forces eviction, EOS / max-token finishes and aborts, plus seeded
random streams.  Where the reference would hit its own debug_assert
(KvCachePool::free of a page that is not in use, kv_pool.rs:40-45) both
sides must fail at the same iteration.

Also ported: the reference's engine scenarios (inference-engine/tests/
engine_tests.rs:60-186) driven through both implementations.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle.host_ref as ref
from mitten_b200 import _lib, host


class _Both:
    """One request stream fed to the mirror and the oracle side by side."""

    def __init__(self, num_pages, page_size, budget, max_decode, vocab, radix_max_pages=None, eos=(99,),
                 forced=(), rng_seed=42):
        self.mir = host.Scheduler(num_pages, page_size, budget, max_decode, radix_max_pages,
                                  mode=_lib.MTN_SCHED_REFERENCE, eos_token_ids=eos)
        self.ctx = ref.EngineContext(num_pages, page_size, budget, max_decode, radix_max_pages, eos_token_ids=eos)
        self.vocab, self.eos, self.forced, self.seed = vocab, list(eos), tuple(forced), rng_seed
        self.reqs: dict[int, ref.Request] = {}
        self.iters = 0

    def add(self, rid, tokens, temperature=0.0, max_new_tokens=8):
        self.mir.add_request(rid, tokens, temperature, max_new_tokens)
        r = ref.Request(rid, [int(t) for t in tokens], temperature=temperature, max_new_tokens=max_new_tokens)
        self.ctx.waiting.append(r)
        self.reqs[rid] = r

    def _check_requests(self, skip_pages=()):
        for rid, r in self.reqs.items():
            info = self.mir.request_info(rid)
            assert info["state"] == r.state, (self.iters, rid)
            assert info["device_len"] == r.device_len, (self.iters, rid)
            assert info["cached_len"] == r.cached_len, (self.iters, rid)
            assert self.mir.request_output(rid) == r.output_ids, (self.iters, rid)
            if rid not in skip_pages:
                assert self.mir.request_pages(rid) == list(r.kv_pages), (self.iters, rid)

    def _check_pool(self):
        assert self.mir.free_pages() == self.ctx.kv_pool.free_pages(), self.iters
        assert self.mir.cached_pages() == self.ctx.radix_cache.total_cached_pages(), self.iters

    def step(self, abort=False):
        """One engine iteration (engine_loop.rs:35-80, serialised): schedule,
        forward (stub), process -- or abort the batch.  Returns the oracle
        batch (None when nothing was schedulable)."""
        self.iters += 1
        err_ref = err_mir = None
        try:
            b_ref = self.ctx.schedule_batch()
        except ref.RefError as e:
            err_ref = e
        try:
            b_mir = self.mir.schedule()
        except _lib.MittenError as e:
            err_mir = e
        assert (err_ref is None) == (err_mir is None), (self.iters, err_ref, err_mir)
        if err_ref is not None:
            raise ref.RefError(f"both failed at schedule: {err_ref}")
        assert (b_ref is None) == (b_mir is None), self.iters
        if b_ref is None:
            self._check_requests()
            self._check_pool()
            return None
        self._check_batch(b_ref, b_mir)
        logits = ref.stub_logits(b_ref.requests, self.vocab, self.eos, self.forced, self.seed)
        if abort:
            self.mir.abort_batch()
            ref.EngineContext.abort_batch(b_ref)
            # The mirror releases an aborted request at once; the reference does
            # it in the next collect_decode_requests (decode.rs:20-33), before
            # anything else touches the pool: pages are compared after that.
            self._check_requests(skip_pages={r.id for r in b_ref.requests})
            return b_ref
        try:
            self.ctx.process_and_transition(b_ref, logits)
        except ref.RefError as e:
            err_ref = e
        try:
            self.mir.process_logits(logits)
        except _lib.MittenError as e:
            err_mir = e
        assert (err_ref is None) == (err_mir is None), (self.iters, err_ref, err_mir)
        if err_ref is not None:
            raise ref.RefError(f"both failed at process: {err_ref}")
        self._check_requests()
        self._check_pool()
        return b_ref

    def _check_batch(self, b_ref, b_mir):
        it = self.iters
        assert b_mir.phase == b_ref.phase, it
        assert b_mir.req_ids.tolist() == [r.id for r in b_ref.requests], it
        assert b_mir.input_ids.tolist() == [int(t) for t in b_ref.input_ids], it
        assert b_mir.position_ids.tolist() == list(b_ref.position_ids), it
        assert b_mir.page_table() == [list(p) for p in b_ref.page_table], it
        # CSR rows: prefill rows carry extend_len query tokens and see
        # device_len + extend_len keys; decode rows one token, device_len + 1 keys.
        qo, lens, n_pre = [0], [], 0
        for r in b_ref.requests:
            if r.state == ref.PREFILLING:
                qo.append(qo[-1] + r.extend_len)
                lens.append(r.device_len + r.extend_len)
                n_pre += 1
            else:
                qo.append(qo[-1] + 1)
                lens.append(r.device_len + 1)
        assert b_mir.qo_indptr.tolist() == qo, it
        assert b_mir.seq_lens.tolist() == lens, it
        assert b_mir.n_prefill == n_pre, it
        assert len(b_mir.cow_src) == 0, it

    def active(self):
        return self.mir.num_active()


def _run(both: _Both, arrivals: dict, aborts=(), max_iters=400):
    """Feed arrivals (iteration -> [(id, tokens, temperature, max_new)]) and
    step until idle; returns the number of iterations that ran a batch."""
    ran = 0
    last = max(arrivals) if arrivals else 0
    for it in range(max_iters):
        for rid, toks, temp, mx in arrivals.get(it, []):
            both.add(rid, toks, temp, mx)
        b = both.step(abort=it in aborts)
        ran += b is not None
        if b is None and it >= last and both.active() == 0:
            return ran
    raise AssertionError("stream did not drain")


# ------------------------------------------------------------------ streams
def test_config1_prompts_lockstep():
    """Config 1: 4 x 128 random prompt tokens (seed 1, vocab 151 936), page 16,
    prefilled together, then 32 greedy steps each."""
    vocab = 151936
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, vocab, size=(4, 128))
    both = _Both(num_pages=512, page_size=16, budget=8192, max_decode=32, vocab=vocab, eos=(vocab + 7,))
    arrivals = {0: [(i + 1, prompts[i].tolist(), 0.0, 33) for i in range(4)]}
    ran = _run(both, arrivals)
    assert ran == 33
    for i in range(4):
        assert both.reqs[i + 1].state == ref.DONE
        assert len(both.reqs[i + 1].output_ids) == 33
    assert both.mir.free_pages() == 512


def test_shared_prefix_lockstep():
    """Later requests match the first one's promoted full pages
    (radix_cache.rs:64-117) while it is still decoding.  In the reference a
    request frees every page it lists when it finishes, shared prefix pages
    included (scheduler.rs:164-172), so the second sharer to finish frees
    pages that are already free: the reference's own debug_assert
    (kv_pool.rs:40-45) fires, and the mirror reports it at the same
    iteration.  (The refcount mode fixes this: tests/test_sched_refcount.py.)"""
    prefix = list(range(100, 112))  # three pages of 4
    both = _Both(num_pages=64, page_size=4, budget=64, max_decode=8, vocab=256)
    arrivals = {
        0: [(1, prefix + [7, 8, 9, 10, 11], 0.0, 12)],
        2: [(2, prefix + [20, 21], 0.0, 4), (3, prefix[:8] + [30, 31, 32, 33, 34], 1.0, 5)],
        3: [(4, prefix + [40], 0.0, 3)],
    }
    with pytest.raises(ref.RefError, match="both failed at process: Attempted to free a page that is not in use"):
        _run(both, arrivals)
    assert both.reqs[2].cached_len == 12 and both.reqs[3].cached_len == 8 and both.reqs[4].cached_len == 12
    # request 1 still lists the prefix pages 0-2 that a finished sharer already returned
    assert both.reqs[1].kv_pages[:3] == [0, 1, 2] and both.reqs[2].kv_pages == []


def test_chunked_prefill_lockstep():
    """A 10-token budget (less the decode rows, scheduler.rs:13-17) cuts the
    prompts into chunks across iterations (prefill.rs:99-114); mixed batches."""
    rng = np.random.default_rng(11)
    both = _Both(num_pages=64, page_size=4, budget=10, max_decode=8, vocab=64)
    arrivals = {0: [(1, rng.integers(0, 64, 23).tolist(), 0.0, 6), (2, rng.integers(0, 64, 17).tolist(), 1.0, 4)],
                3: [(3, rng.integers(0, 64, 9).tolist(), 0.5, 5)]}
    _run(both, arrivals)
    assert all(r.state == ref.DONE for r in both.reqs.values())


def test_eos_and_abort_lockstep():
    """Forced tokens end two requests at EOS; a decode-only batch is aborted
    (engine_loop.rs:47-57) and its requests are released at the next schedule."""
    both = _Both(num_pages=32, page_size=4, budget=64, max_decode=8, vocab=100, forced=(5, 6, 7, 8, 9, 10))
    arrivals = {0: [(1, [1, 2, 3, 4, 5], 0.0, 4), (2, [9, 8, 7], 0.0, 50)],
                4: [(3, [5, 5, 5, 5, 6, 6], 0.0, 50), (4, [3, 3, 3], 0.0, 2)]}
    # iteration 2 is decode-only (both prefilled at 0); after it the survivors hit EOS
    _run(both, arrivals, aborts={2})
    assert both.reqs[1].state == ref.ABORTED and both.reqs[2].state == ref.ABORTED
    assert both.reqs[3].state == ref.DONE and both.reqs[3].output_ids[-1] == 99  # forced EOS
    assert both.reqs[4].state == ref.DONE and len(both.reqs[4].output_ids) == 2
    assert both.mir.free_pages() == both.ctx.kv_pool.free_pages()


def test_eviction_pressure_lockstep():
    """A full pool makes admission evict the radix cache's LRU leaves
    (prefill.rs:44-55, radix_cache.rs:243-282).  In the reference the
    evicted pages may still belong to a live request (promote_request does
    not transfer ownership, radix_cache.rs:287-294), so the pages are handed
    out twice and a later free hits KvCachePool::free's debug_assert; the
    mirror must fail at exactly the same iteration."""
    both = _Both(num_pages=12, page_size=4, budget=64, max_decode=8, vocab=128)
    both.add(1, list(range(8)), 0.0, 6)
    both.step()
    both.step()
    assert both.mir.cached_pages() == 2  # request 1's two full pages, promoted
    both.add(2, list(range(50, 94)), 0.0, 3)  # 11 pages: one more than the pool has free
    both.step()
    # request 2 was admitted by evicting request 1's promoted pages 0 and 1,
    # which it received first (LIFO) while request 1 still lists them; the tree
    # now holds request 2's 11 promoted pages only
    assert both.mir.cached_pages() == 11
    assert both.reqs[2].kv_pages[:2] == [1, 0] and both.reqs[1].kv_pages == [0, 1]
    with pytest.raises(ref.RefError, match="both failed at process: Attempted to free a page that is not in use"):
        _run(both, {})


@pytest.mark.parametrize("seed", range(24))
def test_random_streams_lockstep(seed):
    """Seeded random streams, mixed temperatures and budgets, occasional aborts
    of decode-only batches.  Even seeds: prompts built from a few shared
    prefixes in small pools (prefix hits and evictions, which in the
    reference end in its double free); odd seeds: prompts that share nothing
    in pools large enough that nothing is evicted (long clean runs).  Either
    both sides agree at every iteration until idle, or both fail at the same
    iteration."""
    rng = np.random.default_rng(1000 + seed)
    ps = int(rng.choice([2, 4, 8]))
    shared = seed % 2 == 0
    vocab = 97 if shared else 4099
    bases = [rng.integers(0, vocab, int(rng.integers(ps, 6 * ps))).tolist() for _ in range(3)]
    both = _Both(num_pages=int(rng.integers(24, 96)) if shared else 2048, page_size=ps,
                 budget=int(rng.integers(4, 48)), max_decode=int(rng.integers(2, 8)), vocab=vocab,
                 eos=(int(rng.integers(0, vocab)),),
                 forced=() if seed % 4 < 2 else tuple(rng.integers(0, vocab, 12).tolist()), rng_seed=seed)
    arrivals, rid = {}, 1
    for it in range(0, 40, 2):
        for _ in range(int(rng.integers(0, 3))):
            if shared:
                base = bases[int(rng.integers(0, 3))]
                toks = base[: int(rng.integers(1, len(base) + 1))]
                toks = toks + rng.integers(0, vocab, int(rng.integers(0, 10))).tolist()
            else:  # a distinct first token: no radix edge is ever shared
                toks = [rid] + rng.integers(0, vocab, int(rng.integers(0, 40))).tolist()
            if len(toks) * 1.0 / ps >= both.ctx.kv_pool.num_pages:
                continue
            arrivals.setdefault(it, []).append((rid, toks, float(rng.choice([0.0, 1.0])), int(rng.integers(1, 24))))
            rid += 1
    aborts = set()
    failed = False
    try:
        # abort only decode-only batches (the mirror and the reference differ
        # on aborted prefill rows: the reference keeps scheduling them)
        last = max(arrivals) if arrivals else 0
        for it in range(600):
            for a in arrivals.get(it, []):
                both.add(*a)
            want_abort = rng.random() < 0.05 and both.ctx.prefilling == [] and not both.ctx.waiting \
                and any(r.state == ref.DECODING for r in both.ctx.decoding)
            b = both.step(abort=want_abort)
            if want_abort and b is not None:
                aborts.add(it)
            if b is None and it >= last and both.active() == 0:
                break
        else:
            raise AssertionError("stream did not drain")
    except ref.RefError as e:
        assert "both failed" in str(e)
        failed = True
    if not shared:
        assert not failed and all(r.state in (ref.DONE, ref.ABORTED) for r in both.reqs.values())
        assert both.mir.free_pages() == both.ctx.kv_pool.free_pages()


# ------------------------------------------------- engine_tests.rs scenarios
ENGINE_CFG = dict(num_pages=16, page_size=4, budget=1024, max_decode=32, vocab=100, eos=(99,), forced=(42, 42, 42))


def _engine_request(both, rid, max_new):
    # SamplingParams::default() has temperature 1.0 (request.rs:29-38)
    both.add(rid, [1, 2, 3, 4], 1.0, max_new)


def test_engine_request_completes():  # engine_tests.rs:60-85
    both = _Both(**ENGINE_CFG)
    _engine_request(both, 1, 2)
    _run(both, {})
    assert len(both.reqs[1].output_ids) == 2
    assert both.mir.request_output(1) == both.reqs[1].output_ids


def test_engine_state_transitions():  # engine_tests.rs:87-109
    both = _Both(**ENGINE_CFG)
    _engine_request(both, 1, 1)
    _run(both, {})
    assert both.reqs[1].state == ref.DONE
    assert both.mir.request_info(1)["state"] == _lib.MTN_REQ_DONE


def test_engine_concurrent_8_requests():  # engine_tests.rs:111-138
    both = _Both(**dict(ENGINE_CFG, num_pages=64))
    for i in range(8):
        _engine_request(both, i + 1, 2)
    _run(both, {})
    for i in range(8):
        assert both.mir.request_info(i + 1)["state"] == _lib.MTN_REQ_DONE
        assert len(both.reqs[i + 1].output_ids) == 2


def test_engine_kv_pages_freed_on_done():  # engine_tests.rs:140-165
    both = _Both(**ENGINE_CFG)
    _engine_request(both, 1, 1)
    _run(both, {})
    assert both.reqs[1].kv_pages == [] and both.mir.request_pages(1) == []
    assert both.mir.free_pages() == 16


def test_engine_idle_schedules_nothing():  # engine_tests.rs:167-186
    both = _Both(**ENGINE_CFG)
    for _ in range(5):
        assert both.step() is None
