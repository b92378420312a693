"""The host-made decode work plan (mtn_paged_decode_plan), on the CPU.

Definition checked by brute force: tiles (128 tokens of one (sequence, kv
head) segment) are laid end to end, sequence by sequence, kv head by kv
head; tile x's start cost is 8 per earlier tile plus w per segment start up
to and including its own segment (w = 16 when there are at least 25/8
tiles per CTA, else 0); CTA c's range starts at the first tile whose start
cost reaches floor(c * total / ctas).  Also: the header, each CTA's start
entry (sequence, tiles before it, clamped length, first page index), and
the balance the split buys on config 2 (a CTA whose range spans two
segments gets fewer tiles)."""
from __future__ import annotations

import numpy as np
import pytest

from mitten_b200 import _lib, paged

GRID64 = 2 * 148  # decode CTAs at head_dim 64 on a 148-SM B200 (the planner's count without a GPU)


def _plan(lens, hkv, ps=16, d=64, indptr=None):
    lens = np.asarray(lens, np.int32)
    if indptr is None:
        indptr = np.concatenate([[0], np.cumsum((lens + ps - 1) // ps)]).astype(np.int32)
    p = paged.DecodePlan.__new__(paged.DecodePlan)
    p.head_dim = d
    p.nbytes = int(_lib.lib().mtn_paged_decode_plan_bytes(d))
    buf = np.zeros(p.nbytes // 4, np.int32)
    i32 = _lib.C.POINTER(_lib.C.c_int32)
    _lib.check(_lib.lib().mtn_paged_decode_plan(indptr.ctypes.data_as(i32), lens.ctypes.data_as(i32), lens.size, ps,
                                                hkv, d, buf.ctypes.data, p.nbytes))
    return buf, indptr


def _brute(lens, hkv, grid, ps=16, indptr=None):
    lens = np.asarray(lens, np.int64)
    if indptr is not None:
        lens = np.minimum(lens, (np.diff(indptr).astype(np.int64)) * ps)
    T = (lens + 127) // 128
    U = int(T.sum()) * hkv
    ctas = min(grid, U)
    if U == 0:
        return U, ctas, None
    if U <= grid:
        return U, ctas, np.arange(ctas + 1)
    w = 16 if 8 * U >= 25 * ctas else 0
    starts, cost = [], 0
    for t in T:
        for _ in range(hkv):
            for j in range(t):
                cost += w if j == 0 else 0
                starts.append(cost)
                cost += 8
    starts = np.asarray(starts, np.int64)
    start0 = starts - np.where(np.concatenate([[True], np.diff(starts) != 8]), w, 0)  # cost before the segment's w
    total = cost
    bnd = [int(np.searchsorted(start0, c * total // ctas, side="left")) for c in range(ctas)] + [U]
    return U, ctas, np.asarray(bnd)


def _check(lens, hkv, indptr=None):
    w, ip = _plan(lens, hkv, indptr=indptr)
    U, ctas, bnd = _brute(lens, hkv, GRID64, indptr=indptr)
    assert w[0] == 0x504E544D and w[2] == GRID64 and w[1] == ctas and w[3] == U
    if ctas == 0:
        return w
    table = w[4 + 8 * GRID64: 4 + 8 * GRID64 + GRID64 + 1]
    np.testing.assert_array_equal(table[:ctas + 1], bnd)
    assert np.all(np.diff(table[:ctas + 1]) > 0) and np.all(table[ctas:] == U)
    lens_c = np.minimum(np.maximum(np.asarray(lens, np.int64), 0), np.diff(ip).astype(np.int64) * 16)
    T = (lens_c + 127) // 128
    pre_tiles = np.concatenate([[0], np.cumsum(T)])
    for c in range(ctas):
        e = w[4 + 8 * c: 4 + 8 * c + 8]
        t0, n, s0, pre0, len0, pbeg0 = (int(x) for x in e[:6])
        assert t0 == bnd[c] and n == bnd[c + 1] - bnd[c] and n > 0
        assert pre0 == pre_tiles[s0] and pre0 * hkv <= t0 < (pre0 + T[s0]) * hkv
        assert len0 == lens_c[s0] and pbeg0 == ip[s0]
    return w


def test_config2_plan_and_balance():
    rng = np.random.default_rng(2)
    lens = rng.integers(256, 4097, size=64)
    w = _check(lens, 2)
    table = w[4 + 8 * GRID64: 4 + 8 * GRID64 + GRID64 + 1]
    T = (lens + 127) // 128
    seg_starts = set(np.cumsum(np.repeat(T, 2))[:-1].tolist()) | {0}
    tiles = np.diff(table)
    segs = np.array([1 + sum(1 for x in seg_starts if table[c] < x < table[c + 1]) for c in range(GRID64)])
    # CTAs spanning more segments take fewer tiles; a range's cost (8 per tile,
    # 16 per segment start in it) misses the ideal by less than one segment's
    # first tile (24) at either end
    assert tiles[segs >= 2].mean() < tiles[segs == 1].mean()
    starts = np.array([sum(1 for x in seg_starts if table[c] <= x < table[c + 1]) for c in range(GRID64)])
    cost = 8 * tiles + 16 * starts
    assert cost.max() - cost.min() <= 48


@pytest.mark.parametrize("seed", range(40))
def test_random_batches(seed):
    rng = np.random.default_rng(100 + seed)
    n = int(rng.integers(1, 300))
    top = int(rng.choice([3, 200, 3000, 40000]))
    lens = rng.integers(0, top, size=n)
    if seed % 3 == 0:
        lens[rng.integers(0, n, size=max(1, n // 4))] = 0
    _check(lens, int(rng.choice([1, 2, 4, 8])))


def test_lengths_clamped_to_block_tables():
    # a seq_len beyond its pages is clamped exactly as the kernel clamps it
    lens = np.array([5000, 300, 129], np.int32)
    indptr = np.array([0, 10, 40, 49], np.int32)  # 160 tokens of room for the first sequence
    _check(lens, 2, indptr=indptr)


def test_empty_and_tiny_batches():
    w, _ = _plan([0, 0, 0], 2)
    assert w[1] == 0 and w[3] == 0
    _check([1], 1)            # one tile, one CTA
    _check([129, 1, 0, 7], 4)  # fewer tiles than CTAs: one tile each


def test_rejects_small_buffers_and_bad_head_dim():
    lens = np.array([10], np.int32)
    ip = np.array([0, 1], np.int32)
    i32 = _lib.C.POINTER(_lib.C.c_int32)
    buf = np.zeros(16, np.int32)
    assert _lib.lib().mtn_paged_decode_plan(ip.ctypes.data_as(i32), lens.ctypes.data_as(i32), 1, 16, 2, 64,
                                            buf.ctypes.data, 64) == _lib.MTN_EINVAL
    assert _lib.lib().mtn_paged_decode_plan_bytes(96) == 0
