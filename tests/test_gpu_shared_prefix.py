"""Decode over a prefix shared by every sequence (mtn_paged_decode_shared_prefix)
against the f32 oracle on the concatenated keys, and against the plain paged
decode over the concatenated block tables.

Tolerances as in test_gpu_decode.py: 2e-2 max-abs against the oracle fed the
unrounded f32 Q/K/V, 1e-2 against the oracle fed the bf16 values the kernels
read.  The two GPU paths (shared prefix vs one block table per sequence)
differ only in f32 rounding and the bf16 rounding of P, so they agree to
1e-2 as well.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import _lib, paged

pytestmark = pytest.mark.gpu

TOL_SPEC, TOL_KERNEL = 2e-2, 1e-2


def _case(hkv, d, n_prefix_pages, own_lens, ps=16, seed=0, extra=1):
    rng = np.random.default_rng(seed)
    own_pages = [(n + ps - 1) // ps + extra for n in own_lens]
    num_pages = n_prefix_pages + sum(own_pages) + 8
    pool = paged.PagedKVPool(1, num_pages, ps, hkv, d, device="cuda")
    perm = rng.permutation(num_pages).astype(np.int32)
    prefix = perm[:n_prefix_pages]
    own, off = [], n_prefix_pages
    for k in own_pages:
        own.append(perm[off:off + k])
        off += k
    plen = n_prefix_pages * ps
    kp = rng.standard_normal((plen, hkv, d)).astype(np.float32)
    vp = rng.standard_normal((plen, hkv, d)).astype(np.float32)
    ko = [rng.standard_normal((n, hkv, d)).astype(np.float32) for n in own_lens]
    vo = [rng.standard_normal((n, hkv, d)).astype(np.float32) for n in own_lens]
    slots = [prefix[t // ps] * ps + t % ps for t in range(plen)]
    for r, n in enumerate(own_lens):
        slots += [own[r][t // ps] * ps + t % ps for t in range(n)]
    k_all = np.concatenate([kp] + ko)
    v_all = np.concatenate([vp] + vo)
    pool.append(0, torch.from_numpy(k_all).cuda(), torch.from_numpy(v_all).cuda(),
                torch.tensor(slots, dtype=torch.int64, device="cuda"))
    indptr = np.concatenate([[0], np.cumsum([len(o) for o in own])]).astype(np.int32)
    return {"pool": pool, "prefix": prefix, "own": own, "kp": kp, "vp": vp, "ko": ko, "vo": vo,
            "indptr": torch.from_numpy(indptr).cuda(),
            "indices": torch.from_numpy(np.concatenate(own).astype(np.int32)).cuda(),
            "lens": torch.tensor(own_lens, dtype=torch.int32, device="cuda"),
            "prefix_t": torch.from_numpy(prefix.copy()).cuda(), "own_lens": list(own_lens), "ps": ps}


def _full_tables(c):
    """The same sequences as plain block tables: prefix pages ++ own pages."""
    tabs = [np.concatenate([c["prefix"], o]) for o in c["own"]]
    indptr = np.concatenate([[0], np.cumsum([len(t) for t in tabs])]).astype(np.int32)
    lens = [len(c["prefix"]) * c["ps"] + n for n in c["own_lens"]]
    return (torch.from_numpy(indptr).cuda(), torch.from_numpy(np.concatenate(tabs).astype(np.int32)).cuda(),
            torch.tensor(lens, dtype=torch.int32, device="cuda"))


def _check(c, q, q_used, out, phantom, d):
    e_spec = e_kern = 0.0
    for r in range(len(c["own_lens"])):
        k = np.concatenate([c["kp"], c["ko"][r]]).transpose(1, 0, 2)
        v = np.concatenate([c["vp"], c["vo"][r]]).transpose(1, 0, 2)
        kb, vb = oracle.round_bf16(k), oracle.round_bf16(v)
        if phantom:
            z = np.zeros((k.shape[0], 1, d), np.float32)
            k, v, kb, vb = (np.concatenate([z, x], axis=1) for x in (k, v, kb, vb))
        e_spec = max(e_spec, float(np.abs(out[r] - oracle.attention(q[r:r + 1], k, v, d ** -0.5)[0]).max()))
        e_kern = max(e_kern, float(np.abs(out[r] - oracle.attention(q_used[r:r + 1], kb, vb, d ** -0.5)[0]).max()))
    assert e_spec <= TOL_SPEC, e_spec
    assert e_kern <= TOL_KERNEL, e_kern


@pytest.mark.parametrize("hq,hkv,d,phantom", [(28, 4, 128, False), (14, 2, 64, True), (8, 1, 256, False),
                                              (14, 2, 64, False)])
def test_shared_prefix_matches_oracle_and_full_tables(cuda_device, hq, hkv, d, phantom):
    rng = np.random.default_rng(hq + d)
    own_lens = [0, 1, 15, 16, 17, 130] + [int(x) for x in rng.integers(1, 600, size=34)]
    c = _case(hkv, d, 24, own_lens, seed=hq * 3 + d)
    n = len(own_lens)
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    ws = paged.shared_prefix_workspace(c["pool"], n, hq)
    outs = []
    for _ in range(2):  # two calls in a row on one workspace
        outs.append(paged.paged_decode_shared_prefix(c["pool"], 0, qt, c["prefix_t"], c["indptr"], c["indices"],
                                                     c["lens"], phantom=phantom, out_dtype=torch.float32,
                                                     workspace=ws).cpu().numpy())
    np.testing.assert_array_equal(outs[0], outs[1])
    _check(c, q, oracle.round_bf16(qt.float().cpu().numpy()), outs[0], phantom, d)
    ip, idx, lens = _full_tables(c)
    full = paged.paged_decode(c["pool"], 0, qt, ip, idx, lens, phantom=phantom, out_dtype=torch.float32)
    assert float(np.abs(full.cpu().numpy() - outs[0]).max()) <= TOL_KERNEL
    assert paged.device_error(0) == (0, 0)


@pytest.mark.parametrize("hq,hkv,d", [(28, 4, 128), (8, 1, 256)])
def test_shared_prefix_fused_append_cfg3_shape(cuda_device, hq, hkv, d):
    """A config-3-like batch: 128 sequences over a 64-page (1024-token) shared
    prefix, own parts of U[1, 520] tokens, the step's K/V appended at each own
    part's last position (bit-exact in the pool) and attended to."""
    rng = np.random.default_rng(7)
    own_lens = [int(x) for x in rng.integers(1, 521, size=128)]
    c = _case(hkv, d, 64, own_lens, seed=8)
    n = len(own_lens)
    kn = rng.standard_normal((n, hkv, d)).astype(np.float32)
    vn = rng.standard_normal((n, hkv, d)).astype(np.float32)
    for r in range(n):
        c["ko"][r][-1] = kn[r]
        c["vo"][r][-1] = vn[r]
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    out = paged.paged_decode_shared_prefix(c["pool"], 0, qt, c["prefix_t"], c["indptr"], c["indices"], c["lens"],
                                           k_new=torch.from_numpy(kn).cuda().to(torch.bfloat16),
                                           v_new=torch.from_numpy(vn).cuda().to(torch.bfloat16),
                                           out_dtype=torch.float32).cpu().numpy()
    ks, vs = c["pool"].gather(0, c["indptr"], c["indices"], c["lens"])
    for r in range(n):
        np.testing.assert_array_equal(ks[r].contiguous().view(torch.int16).cpu().numpy().view(np.uint16),
                                      oracle.rne_bf16_bits(c["ko"][r].transpose(1, 0, 2)))
        np.testing.assert_array_equal(vs[r].contiguous().view(torch.int16).cpu().numpy().view(np.uint16),
                                      oracle.rne_bf16_bits(c["vo"][r].transpose(1, 0, 2)))
    _check(c, q, oracle.round_bf16(qt.float().cpu().numpy()), out, False, d)
    assert paged.device_error(0) == (0, 0)


def test_shared_prefix_rejects_empty_prefix(cuda_device):
    c = _case(2, 64, 2, [5, 6], seed=1)
    q = torch.zeros(2, 14, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_lib.MittenError):
        paged.paged_decode_shared_prefix(c["pool"], 0, q, c["prefix_t"][:0], c["indptr"], c["indices"], c["lens"])
