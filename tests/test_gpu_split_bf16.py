"""MTN_ATTN_SPLIT_BF16 on the GPU: Q and P reach the tensor cores as bf16
hi + lo pairs, so decode and prefill match the reference's f32 products
(qwen model.rs:413-416) on f32 queries far more tightly than the default
bf16 operands.

Tolerance: max |out - oracle| <= 2e-4 against the f32 oracle fed the f32
queries and the bf16 K/V the pool holds (the pool stores bf16 either way).
The default mode's own bound on the same comparison is 1e-2 (P is rounded
to bf16); the test also shows split mode is at least 20x closer on each
case.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import _lib, paged
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu

TOL_SPLIT = 2e-4


def _decode(case, q, split, k_new=None, v_new=None):
    out = paged.paged_decode(case.pool, 0, q, case.kv_indptr, case.kv_indices, case.seq_lens, phantom=True,
                             out_dtype=torch.float32, split_bf16=split, k_new=k_new, v_new=v_new)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _decode_err(case, q_np, out, d):
    err = 0.0
    for r in range(len(case.lens)):
        kb, vb = case.oracle_cache(r, layer_round=True, phantom=True)
        want = oracle.attention(q_np[r:r + 1], kb, vb, d ** -0.5)[0]
        err = max(err, float(np.abs(out[r] - want).max()))
    return err


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256), (16, 2, 64), (3, 3, 128)])
def test_decode_split_f32_queries(cuda_device, hq, hkv, d):
    lens = [1, 17, 130, 700, 2500]
    case = make_case(lens, hkv, d, seed=hq + d)
    rng = np.random.default_rng(d)
    q = rng.standard_normal((len(lens), hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).cuda()
    e_split = _decode_err(case, q, _decode(case, qt, True), d)
    e_plain = _decode_err(case, q, _decode(case, qt, False), d)
    assert e_split <= TOL_SPLIT, e_split
    assert e_split * 20 <= e_plain, (e_split, e_plain)
    assert paged.device_error(0) == (0, 0)


def test_decode_split_with_fused_append(cuda_device):
    """The step's K/V row stored by the kernel itself, then attended, in split mode."""
    lens = [64, 300, 1025]
    hq, hkv, d = 14, 2, 64
    case = make_case(lens, hkv, d, seed=3)
    rng = np.random.default_rng(4)
    kn = rng.standard_normal((len(lens), hkv, d)).astype(np.float32)
    vn = rng.standard_normal((len(lens), hkv, d)).astype(np.float32)
    # the appended token is the last of each sequence: the case's cache holds
    # len - 1 earlier tokens plus this row
    for r in range(len(lens)):
        case.k[r][-1] = kn[r]
        case.v[r][-1] = vn[r]
    q = rng.standard_normal((len(lens), hq, d)).astype(np.float32)
    out = _decode(case, torch.from_numpy(q).cuda(), True, torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
    assert _decode_err(case, q, out, d) <= TOL_SPLIT


def test_decode_split_bf16_queries(cuda_device):
    """bf16 queries have no remainder: split mode still splits P."""
    lens = [200, 900]
    case = make_case(lens, 2, 64, seed=8)
    q = torch.randn((2, 14, 64), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    out = _decode(case, q.cuda(), True)
    assert _decode_err(case, q.float().numpy(), out, 64) <= TOL_SPLIT


def _prefill(case, q, q_lens, split, one_tile=False):
    qo = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32), device="cuda")
    out = paged.paged_prefill(case.pool, 0, q, qo, case.kv_indptr, case.kv_indices, case.seq_lens, max(q_lens),
                              phantom=True, out_dtype=torch.float32, split_bf16=split, one_tile=one_tile)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _prefill_err(case, q_np, q_lens, out, d):
    off, err = 0, 0.0
    for r, ql in enumerate(q_lens):
        kb, vb = case.oracle_cache(r, layer_round=True, phantom=True)
        want = oracle.attention(q_np[off:off + ql], kb, vb, d ** -0.5)
        err = max(err, float(np.abs(out[off:off + ql] - want).max()))
        off += ql
    return err


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (4, 4, 64)])
def test_prefill_split_f32_queries(cuda_device, hq, hkv, d):
    kv_lens, q_lens = [200, 77, 812, 1, 640], [72, 77, 300, 1, 130]
    case = make_case(kv_lens, hkv, d, seed=hq * 3 + d)
    rng = np.random.default_rng(hq)
    q = rng.standard_normal((sum(q_lens), hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).cuda()
    e_split = _prefill_err(case, q, q_lens, _prefill(case, qt, q_lens, True), d)
    e_plain = _prefill_err(case, q, q_lens, _prefill(case, qt, q_lens, False), d)
    assert e_split <= TOL_SPLIT, e_split
    assert e_split * 20 <= e_plain, (e_split, e_plain)
    assert paged.device_error(0) == (0, 0)


def test_prefill_split_long_chunk_pieces(cuda_device):
    """One long chunk (few units: the split of long units into pieces runs) in split mode."""
    kv_lens, q_lens = [4096 + 512], [512]
    case = make_case(kv_lens, 2, 64, seed=12)
    q = np.random.default_rng(13).standard_normal((512, 14, 64)).astype(np.float32)
    out = _prefill(case, torch.from_numpy(q).cuda(), q_lens, True)
    assert _prefill_err(case, q, q_lens, out, 64) <= TOL_SPLIT


def test_prefill_f32_queries_unsplit_match_bf16(cuda_device):
    """f32 queries without the flag are rounded to bf16 on load: the same
    result as passing the rounded bf16 queries."""
    kv_lens, q_lens = [300, 129], [300, 2]
    case = make_case(kv_lens, 2, 64, seed=5)
    q = torch.randn((302, 14, 64), generator=torch.Generator().manual_seed(2))
    a = _prefill(case, q.cuda(), q_lens, False)
    b = _prefill(case, q.to(torch.bfloat16).cuda(), q_lens, False, one_tile=True)
    np.testing.assert_array_equal(a, b)


def test_prefill_split_rejects_head_dim_256(cuda_device):
    case = make_case([64], 1, 256, seed=1)
    q = torch.zeros((64, 8, 256), device="cuda")
    with pytest.raises(_lib.MittenError, match="SPLIT_BF16 needs head_dim <= 128"):
        _prefill(case, q, [64], True)
