"""Paged decode attention on the GPU against the f32 oracle.

Tolerance (stated by the spec): max |out - oracle| <= 2e-2 against the
reference's f32 path fed the unrounded f32 Q/K/V.  A second, tighter check
(1e-2) feeds the oracle the bf16 values the kernel reads (Q and K/V as
stored; P is rounded to bf16 before P.V on the tensor cores), which
isolates the kernel's own arithmetic from storage rounding.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import _lib, paged
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu

TOL_SPEC = 2e-2
TOL_KERNEL = 1e-2


def run_decode(case, hq, d, phantom=True, q_dtype=torch.bfloat16, out_dtype=torch.float32, seed=1, ws=None):
    n = len(case.lens)
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).to("cuda").to(q_dtype)
    out = paged.paged_decode(case.pool, 0, qt, case.kv_indptr, case.kv_indices, case.seq_lens, phantom=phantom,
                             out_dtype=out_dtype, workspace=ws)
    torch.cuda.synchronize()
    q_used = oracle.round_bf16(qt.float().cpu().numpy())
    return q, q_used, out.float().cpu().numpy()


def check(case, hq, d, q, q_used, out, phantom=True):
    err_spec, err_kernel = 0.0, 0.0
    for r, n in enumerate(case.lens):
        if n == 0 and not phantom:
            assert np.all(out[r] == 0)
            continue
        k32, v32 = case.oracle_cache(r, layer_round=False, phantom=phantom)
        want = oracle.attention(q[r:r + 1], k32, v32, d ** -0.5)[0]
        err_spec = max(err_spec, float(np.abs(out[r] - want).max()))
        kb, vb = case.oracle_cache(r, layer_round=True, phantom=phantom)
        want_b = oracle.attention(q_used[r:r + 1], kb, vb, d ** -0.5)[0]
        err_kernel = max(err_kernel, float(np.abs(out[r] - want_b).max()))
    assert err_spec <= TOL_SPEC, err_spec
    assert err_kernel <= TOL_KERNEL, err_kernel
    return err_spec, err_kernel


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256), (2, 2, 64), (16, 2, 64),
                                      (6, 2, 128), (5, 1, 64)])
def test_decode_shapes(cuda_device, hq, hkv, d):
    lens = [1, 16, 17, 129, 300, 1000]
    case = make_case(lens, hkv, d, seed=hq * 7 + d)
    q, qu, out = run_decode(case, hq, d)
    check(case, hq, d, q, qu, out)
    assert paged.device_error(0) == (0, 0)


def test_decode_head_dim_256_many_tiles_per_cta(cuda_device):
    # ~700 tiles of 128 tokens over the persistent grid: every CTA streams
    # several tiles, so the 6-slot ring of head-dim halves wraps many times.
    rng = np.random.default_rng(31)
    lens = [int(x) for x in rng.integers(1500, 2600, size=40)]
    case = make_case(lens, 1, 256, seed=32)
    q, qu, out = run_decode(case, 8, 256)
    check(case, 8, 256, q, qu, out)
    assert paged.device_error(0) == (0, 0)


def test_decode_one_long_sequence_split_over_many_ctas(cuda_device):
    # 79 tiles x 2 kv heads < the CTA count: every CTA holds a piece of a
    # segment, so the cross-CTA merge runs for both segments.
    case = make_case([10000], 2, 64, seed=21)
    q, qu, out = run_decode(case, 14, 64)
    check(case, 14, 64, q, qu, out)


def test_decode_many_sequences_mixed_lengths(cuda_device):
    rng = np.random.default_rng(5)
    lens = rng.integers(1, 4097, size=96).tolist()
    case = make_case(lens, 2, 64, seed=23)
    q, qu, out = run_decode(case, 14, 64)
    check(case, 14, 64, q, qu, out)


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256)])
def test_decode_many_short_segments_per_cta(cuda_device, hq, hkv, d):
    """Several one- or two-tile segments per CTA, some cut by CTA boundaries:
    the softmax warps hand each segment to the epilogue warps through
    per-O^T-buffer barriers while the next segments stream, so every
    buffer's barriers go through many phases in one launch."""
    rng = np.random.default_rng(d + hq)
    lens = [int(x) for x in rng.integers(1, 260, size=600 if d == 64 else 300)]
    lens[::37] = [1] * len(lens[::37])
    case = make_case(lens, hkv, d, seed=d + 3)
    q, qu, out = run_decode(case, hq, d)
    check(case, hq, d, q, qu, out)
    assert paged.device_error(0) == (0, 0)


def test_decode_deterministic_and_workspace_reuse(cuda_device):
    lens = [3000, 2000, 1000, 50, 7000]
    case = make_case(lens, 2, 64, seed=4)
    ws = paged.DecodeWorkspace.for_shape(case.pool, len(lens), 14)
    outs = [run_decode(case, 14, 64, out_dtype=torch.float32, ws=ws)[2] for _ in range(3)]
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])


def test_decode_without_phantom_and_empty_sequences(cuda_device):
    lens = [0, 5, 0, 64]
    case = make_case(lens, 2, 64, seed=6)
    q, qu, out = run_decode(case, 14, 64, phantom=False)
    check(case, 14, 64, q, qu, out, phantom=False)
    q, qu, out = run_decode(case, 14, 64, phantom=True)
    check(case, 14, 64, q, qu, out, phantom=True)
    assert np.all(out[0] == 0) and np.all(out[2] == 0)  # phantom only: softmax on a zero value


def test_decode_all_empty(cuda_device):
    case = make_case([0, 0, 0], 2, 64, seed=7)
    _, _, out = run_decode(case, 14, 64, phantom=True)
    assert np.all(out == 0)


def test_decode_reserved_pages_f32_q_bf16_out(cuda_device):
    # Block tables longer than the sequence (config 2 pre-reserves pages).
    lens = [100, 256, 257]
    case = make_case(lens, 2, 64, seed=8, extra_pages=7)
    q, qu, out = run_decode(case, 14, 64, out_dtype=torch.bfloat16, q_dtype=torch.float32)
    check(case, 14, 64, q, qu, out)


def test_decode_page_size_8_and_32(cuda_device):
    for ps in (8, 32):
        case = make_case([40, 500, 33], 2, 64, page_size=ps, seed=ps)
        q, qu, out = run_decode(case, 14, 64)
        check(case, 14, 64, q, qu, out)


@pytest.mark.parametrize("hq,hkv,d,new_dtype", [(14, 2, 64, torch.bfloat16), (28, 4, 128, torch.float32),
                                                (8, 1, 256, torch.bfloat16)])
def test_decode_fused_append(cuda_device, hq, hkv, d, new_dtype):
    """k_new/v_new are stored at position len-1 (bit-exact) and attended to."""
    lens = [1, 16, 17, 300, 129]
    case = make_case(lens, hkv, d, seed=31)
    n = len(lens)
    rng = np.random.default_rng(32)
    kn = rng.standard_normal((n, hkv, d)).astype(np.float32)
    vn = rng.standard_normal((n, hkv, d)).astype(np.float32)
    # The new token is the last of each sequence: overwrite the case's last row.
    for r in range(n):
        case.k[r][-1] = kn[r]
        case.v[r][-1] = vn[r]
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    out = paged.paged_decode(case.pool, 0, qt, case.kv_indptr, case.kv_indices, case.seq_lens, phantom=True,
                             k_new=torch.from_numpy(kn).cuda().to(new_dtype),
                             v_new=torch.from_numpy(vn).cuda().to(new_dtype), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ks, vs = case.pool.gather(0, case.kv_indptr, case.kv_indices, case.seq_lens)
    for r in range(n):
        want_k = oracle.rne_bf16_bits(case.k[r].transpose(1, 0, 2))
        np.testing.assert_array_equal(ks[r].contiguous().view(torch.int16).cpu().numpy().view(np.uint16), want_k)
        want_v = oracle.rne_bf16_bits(case.v[r].transpose(1, 0, 2))
        np.testing.assert_array_equal(vs[r].contiguous().view(torch.int16).cpu().numpy().view(np.uint16), want_v)
    check(case, hq, d, q, oracle.round_bf16(q), out.cpu().numpy())
    assert paged.device_error(0) == (0, 0)


def test_decode_rejects_bad_arguments(cuda_device):
    case = make_case([10], 2, 64)
    q = torch.zeros(1, 13, 64, device="cuda", dtype=torch.bfloat16)  # 13 not a multiple of 2
    with pytest.raises(_lib.MittenError):
        paged.paged_decode(case.pool, 0, q, case.kv_indptr, case.kv_indices, case.seq_lens)
    q = torch.zeros(1, 14, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_lib.MittenError):
        paged.paged_decode(case.pool, 5, q, case.kv_indptr, case.kv_indices, case.seq_lens)
    ws = paged.DecodeWorkspace(256, "cuda")
    with pytest.raises(_lib.MittenError):
        paged.paged_decode(case.pool, 0, q, case.kv_indptr, case.kv_indices, case.seq_lens, workspace=ws)


def test_decode_bad_page_id_is_flagged_not_faulted(cuda_device):
    case = make_case([40], 2, 64, seed=2)
    bad = case.kv_indices.clone()
    bad[1] = 10 ** 6
    paged.device_error(0, clear=True)
    q = torch.randn(1, 14, 64, device="cuda").to(torch.bfloat16)
    paged.paged_decode(case.pool, 0, q, case.kv_indptr, bad, case.seq_lens)
    code, detail = paged.device_error(0, clear=True)
    assert code == 1 and detail == 0
