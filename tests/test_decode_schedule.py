"""CPU replay of the persistent decode kernel's work split (integer logic
only, mirrored from mitten_b200/csrc/decode.cu): every tile of every
(sequence, kv head) segment is owned by exactly one CTA, each CTA's range is
contiguous and non-empty, partial segments use distinct workspace slots, and
the pieces the merge kernel reads (CTAs ca..cb with slot wa for ca) are
exactly the pieces the CTAs wrote."""
from __future__ import annotations

import numpy as np
import pytest

TILE = 128


def tile_begin(c, U, C):
    return c * U // C


def cta_of(x, U, C):
    return min(C - 1, ((x + 1) * C - 1) // U)


def simulate(lens, hkv, grid):
    T = [(n + TILE - 1) // TILE for n in lens]
    U = sum(T) * hkv
    C = min(grid, U)
    seg_tiles = []          # (s, g, T, start)
    pre = 0
    for s, t in enumerate(T):
        for g in range(hkv):
            if t:
                seg_tiles.append((s, g, t, pre * hkv + g * t))
        pre += t
    owner = {}
    writes = {}             # seg -> list of (cta, which)
    for c in range(C):
        t0, t1 = tile_begin(c, U, C), tile_begin(c + 1, U, C)
        assert t1 > t0, "participating CTAs own at least one tile"
        first_seg = None
        for (s, g, t, start) in seg_tiles:
            lo, hi = max(start, t0), min(start + t, t1)
            if lo >= hi:
                continue
            for x in range(lo, hi):
                assert x not in owner
                owner[x] = c
            if first_seg is None:
                first_seg = (s, g)
            ca, cb = cta_of(start, U, C), cta_of(start + t - 1, U, C)
            if ca != cb:
                which = 1 if (c == ca and t0 != start) else 0
                writes.setdefault((s, g), []).append((c, which))
    assert sorted(owner) == list(range(U))
    slots = set()
    for (s, g, t, start) in seg_tiles:
        ca, cb = cta_of(start, U, C), cta_of(start + t - 1, U, C)
        assert owner[start] == ca and owner[start + t - 1] == cb
        if ca == cb:
            assert (s, g) not in writes
            continue
        w = writes[(s, g)]
        assert len(w) == cb - ca + 1, "every CTA in ca..cb wrote a piece"
        wa = 1 if tile_begin(ca, U, C) != start else 0
        assert [x for x in w] == [(cc, wa if cc == ca else 0) for cc in range(ca, cb + 1)]
        for slot in w:
            assert slot not in slots
            slots.add(slot)


@pytest.mark.parametrize("grid", [1, 2, 5, 148, 296])
def test_split_invariants_random(grid):
    rng = np.random.default_rng(grid)
    for trial in range(30):
        n = int(rng.integers(1, 70))
        lens = rng.integers(0, 5000, size=n).tolist()
        if rng.random() < 0.2:
            lens = [0] * n
            lens[int(rng.integers(0, n))] = int(rng.integers(1, 300))
        hkv = int(rng.choice([1, 2, 4]))
        if sum(lens) == 0:
            continue
        simulate(lens, hkv, grid)


def test_split_config2_shape():
    rng = np.random.default_rng(2)
    lens = rng.integers(256, 4097, size=64).tolist()
    simulate(lens, 2, 296)


def test_split_fewer_tiles_than_ctas():
    simulate([1, 16, 17, 129, 300, 1000], 2, 296)
    simulate([10000], 2, 296)
