"""Paged decode and prefill kernels against the committed golden fixtures.

Each case's K/V are written into a pool through the append kernel under a
seeded random block table; the kernels' outputs must match the stored f32
oracle outputs within the spec's 2e-2 max-abs (the oracle fed unrounded
inputs, the kernels reading bf16 K/V).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mitten_b200 import paged
from tests.golden import make_golden as G

pytestmark = pytest.mark.gpu

TOL = 2e-2
PS = 16


def _pool_with(case, ks, vs):
    lens = case["lens"]
    need = [(n + PS - 1) // PS for n in lens]
    num_pages = sum(need) + 8
    pool = paged.PagedKVPool(1, num_pages, PS, case["hkv"], case["d"])
    perm = np.random.default_rng(case["seed"] + 1000).permutation(num_pages)[:sum(need)].astype(np.int32)
    tables, indptr, off = [], [0], 0
    for n in need:
        tables.append(perm[off:off + n])
        off += n
        indptr.append(off)
    slots = np.concatenate([tables[r][np.arange(n) // PS] * PS + np.arange(n) % PS for r, n in enumerate(lens)])
    pool.append(0, torch.from_numpy(np.concatenate(ks)).cuda(), torch.from_numpy(np.concatenate(vs)).cuda(),
                torch.from_numpy(slots.astype(np.int64)).cuda())
    return (pool, torch.tensor(indptr, dtype=torch.int32, device="cuda"), torch.from_numpy(perm).cuda(),
            torch.tensor(lens, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("case", G.CASES, ids=[c["name"] for c in G.CASES])
def test_kernels_match_golden(cuda_device, case):
    golden = np.load(G.OUT)
    q, ks, vs = G.inputs(case)
    assert bytes(golden[case["name"] + "/digest"]).hex() == G.digest(q, ks, vs)
    pool, indptr, indices, seq_lens = _pool_with(case, ks, vs)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    if case["kind"] == "decode":
        out = paged.paged_decode(pool, 0, qt, indptr, indices, seq_lens, phantom=case["phantom"],
                                 out_dtype=torch.float32)
    else:
        qo = torch.tensor(np.concatenate([[0], np.cumsum(case["q_lens"])]), dtype=torch.int32, device="cuda")
        out = paged.paged_prefill(pool, 0, qt, qo, indptr, indices, seq_lens, max(case["q_lens"]),
                                  phantom=case["phantom"], out_dtype=torch.float32)
    got = out.cpu().numpy()
    got = got[G.kept_rows(got.shape[0], case.get("stride", 7))]
    assert float(np.abs(got - golden[case["name"] + "/out"]).max()) <= TOL
    assert paged.device_error(0) == (0, 0)
