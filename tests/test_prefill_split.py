"""CPU replay of the chunked-prefill kernel's unit split (integer logic only,
mirrored from mitten_b200/csrc/prefill.cu): the host turns the split on for
launches whose unit bound (total_q / 128 + n_seqs) x heads is at most 3/4
of the SM count; the kernel then cuts each unit into k <= 4 pieces of
consecutive kv tiles.  The pieces partition the unit's tiles, every piece is
non-empty, all pieces fit in one wave, unit indices are distinct and inside
the workspace, and the workspace size the C-ABI reports covers every slot
the kernel touches."""
from __future__ import annotations

import numpy as np
import pytest

BM = 128
MAX_PIECES = 4
MIN_PIECE = 8
SPLIT_MAX_UNITS = 296


def units_bound(n_seqs, total_q, hq):
    return (total_q // BM + n_seqs) * hq


def host_splits(n_seqs, total_q, hq, sms=148):
    u = units_bound(n_seqs, total_q, hq)
    return u <= SPLIT_MAX_UNITS and 4 * u <= 3 * sms


def piece_len(q_lens, kv_lens, hq, bn, sms):
    t = u = 0
    for ql, kl in zip(q_lens, kv_lens):
        if ql <= 0:
            continue
        kl = max(kl, ql)
        qt = 0
        while qt * BM < ql:
            t += (kl - ql + min(ql, (qt + 1) * BM) - 1) // bn + 1
            u += 1
            qt += 1
    t, u = t * hq, u * hq
    if u >= sms:
        return 0
    return max(MIN_PIECE, -(-t // (sms - u)))


def replay(q_lens, kv_lens, hq, d, sms=148):
    bn = 128 if d <= 128 else 64
    n = len(q_lens)
    total_q = sum(q_lens)
    units = units_bound(n, total_q, hq)
    assert units <= SPLIT_MAX_UNITS
    plen = piece_len(q_lens, kv_lens, hq, bn, sms)
    q0 = np.concatenate([[0], np.cumsum(q_lens)])
    seen = set()
    ctas = 0
    for s in range(n):
        ql, kl = q_lens[s], max(kv_lens[s], q_lens[s])
        for tile in range(-(-ql // BM)):
            nrows = min(BM, ql - tile * BM)
            last_pos = kl - ql + tile * BM + nrows - 1
            n_tiles = last_pos // bn + 1
            for h in range(hq):
                uid = (q0[s] // BM + s + tile) * hq + h
                assert 0 <= uid < units and uid not in seen
                seen.add(uid)
                k = min(MAX_PIECES, -(-n_tiles // plen)) if plen else 1
                covered = []
                for piece in range(MAX_PIECES):
                    if piece >= k:
                        continue
                    ja, jb = piece * n_tiles // k, (piece + 1) * n_tiles // k
                    assert jb > ja
                    covered.extend(range(ja, jb))
                    ctas += 1
                assert covered == list(range(n_tiles))
    assert ctas <= max(sms, len(seen)), "the pieces fit in one wave"
    return plen, ctas


@pytest.mark.parametrize("seed", range(6))
def test_split_pieces_partition_units(seed):
    rng = np.random.default_rng(seed)
    for _ in range(40):
        d = int(rng.choice([64, 128, 256]))
        hq = int(rng.choice([1, 4, 8, 14, 28]))
        n = int(rng.integers(1, 6))
        q_lens = rng.integers(1, 700, size=n).tolist()
        if units_bound(n, sum(q_lens), hq) > SPLIT_MAX_UNITS:
            continue
        kv_lens = [ql + int(rng.integers(0, 20000)) for ql in q_lens]
        replay(q_lens, kv_lens, hq, d)


def test_split_config4_shape():
    # four 512-token chunks after 5632, 2560, 1536 and 7680 cached tokens, Hq 8,
    # D 256: 128 units on 148 SMs, one piece per unit but the longest
    pri = [5632, 2560, 1536, 7680]
    plen, ctas = replay([512] * 4, [p + 512 for p in pri], 8, 256)
    assert plen == 468 and ctas == 128
    assert not host_splits(4, 2048, 8)  # bound 160 units: the host runs it unsplit
    assert host_splits(4, 2048, 4)


def test_split_single_long_chunk_fills_the_gpu():
    plen, ctas = replay([512], [8192], 8, 256)
    assert plen == 35 and ctas == 128  # every unit cut in 4: 32 units -> 128 CTAs
    plen, ctas = replay([512], [8192], 14, 64)
    assert ctas == 112  # 56 units cut in 2
    plen, ctas = replay([512], [8192], 28, 128)
    assert plen == 195 and ctas == 112  # 112 units: too few idle SMs to cut any
    assert host_splits(1, 512, 8) and host_splits(1, 512, 14) and not host_splits(1, 512, 28)


def test_workspace_bytes_cover_slots():
    from mitten_b200 import _lib as L
    lib = L.lib()
    for n, tq, hq, d in [(4, 2048, 8, 256), (1, 512, 8, 256), (5, 580, 28, 128), (2, 100, 14, 64)]:
        units = units_bound(n, tq, hq)
        nb = lib.mtn_paged_prefill_workspace_bytes(n, tq, hq, 1, d)
        need = units * MAX_PIECES * (2 * BM * 4 + BM * d * 4) + units * 4
        assert nb >= need and nb < need + 1024
    assert lib.mtn_paged_prefill_workspace_bytes(16, 8192, 28, 4, 128) == 0  # many units: unsplit
