"""Chunked-prefill attention (tcgen05 / TMEM) on the GPU against the f32 oracle.

Each case appends a chunk of q_len tokens after P cached tokens, then runs
the prefill kernel over the paged cache.  Tolerances as for decode: 2e-2
max-abs against the oracle fed unrounded f32 inputs (the spec's bar), and
a tighter bound against the oracle fed the bf16 values the kernel reads
(P is rounded to bf16 before the P.V product, hence 1e-2).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import paged
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu

TOL_SPEC = 2e-2
TOL_KERNEL = 1e-2


def run_prefill(kv_lens, q_lens, hq, hkv, d, phantom=True, seed=0, out_dtype=torch.float32, page_size=16,
                workspace=None, case=None, one_tile=False):
    case = case or make_case(kv_lens, hkv, d, page_size=page_size, seed=seed)
    rng = np.random.default_rng(seed + 100)
    total_q = sum(q_lens)
    q = rng.standard_normal((total_q, hq, d)).astype(np.float32)
    qt = torch.from_numpy(q).to("cuda").to(torch.bfloat16)
    qo = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32), device="cuda")
    out = paged.paged_prefill(case.pool, 0, qt, qo, case.kv_indptr, case.kv_indices, case.seq_lens,
                              max(q_lens), phantom=phantom, out_dtype=out_dtype, workspace=workspace,
                              one_tile=one_tile)
    torch.cuda.synchronize()
    return case, q, qt.float().cpu().numpy(), out.float().cpu().numpy()


def check(case, q_lens, q, q_used, out, d, phantom=True):
    off = 0
    e_spec = e_kernel = 0.0
    for r, ql in enumerate(q_lens):
        if ql == 0:
            continue
        k32, v32 = case.oracle_cache(r, layer_round=False, phantom=phantom)
        want = oracle.attention(q[off:off + ql], k32, v32, d ** -0.5)
        kb, vb = case.oracle_cache(r, layer_round=True, phantom=phantom)
        want_b = oracle.attention(q_used[off:off + ql], kb, vb, d ** -0.5)
        got = out[off:off + ql]
        e_spec = max(e_spec, float(np.abs(got - want).max()))
        e_kernel = max(e_kernel, float(np.abs(got - want_b).max()))
        off += ql
    assert e_spec <= TOL_SPEC, e_spec
    assert e_kernel <= TOL_KERNEL, e_kernel
    return e_spec, e_kernel


def test_prefill_single_tile(cuda_device):
    case, q, qu, out = run_prefill([128], [128], 14, 2, 64)
    check(case, [128], q, qu, out, 64)
    assert paged.device_error(0) == (0, 0)


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256), (4, 4, 64)])
def test_prefill_chunks_over_cached_prefix(cuda_device, hq, hkv, d):
    # (kv_len, q_len): chunk after a cached prefix, ragged and multi-tile.
    kv_lens = [200, 77, 512 + 300, 1, 640]
    q_lens = [72, 77, 300, 1, 130]
    case, q, qu, out = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=hq + d)
    check(case, q_lens, q, qu, out, d)
    assert paged.device_error(0) == (0, 0)


def test_prefill_without_phantom_bf16_out(cuda_device):
    kv_lens, q_lens = [300, 129], [300, 2]
    case, q, qu, out = run_prefill(kv_lens, q_lens, 14, 2, 64, phantom=False, out_dtype=torch.bfloat16, seed=5)
    check(case, q_lens, q, qu, out, 64, phantom=False)


def test_prefill_page_size_32(cuda_device):
    kv_lens, q_lens = [100, 257], [40, 257]
    case, q, qu, out = run_prefill(kv_lens, q_lens, 14, 2, 64, page_size=32, seed=9)
    check(case, q_lens, q, qu, out, 64)


def test_prefill_empty_chunk_rows(cuda_device):
    kv_lens, q_lens = [10, 50, 20], [0, 50, 0]
    case, q, qu, out = run_prefill(kv_lens, q_lens, 14, 2, 64, seed=3)
    check(case, q_lens, q, qu, out, 64)


@pytest.mark.parametrize("hq,hkv,d,kv_lens,q_lens", [
    (8, 1, 256, [8192], [512]),                      # one long chunk: every unit cut in 4
    (2, 1, 256, [6144, 2560, 2048, 8192], [512] * 4),  # 2, 2, 4 and 4 pieces
    (14, 2, 128, [5000, 300], [256, 300]),
    (14, 2, 64, [9000], [200]),
])
def test_prefill_split_long_units(cuda_device, hq, hkv, d, kv_lens, q_lens):
    """Few units, long contexts: pieces of kv tiles on separate CTAs, merged in
    piece order; matches the oracle, the unsplit launch (a workspace too small
    to split) within tolerance, and itself bit for bit on a reused workspace."""
    from mitten_b200 import _lib as L
    nb = L.lib().mtn_paged_prefill_workspace_bytes(len(q_lens), sum(q_lens), hq, hkv, d)
    assert nb > 0
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    case, q, qu, out = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=d + hq, workspace=ws)
    check(case, q_lens, q, qu, out, d)
    _, _, _, again = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=d + hq, workspace=ws, case=case)
    assert np.array_equal(out, again)
    units = (sum(q_lens) // 128 + len(q_lens)) * hq
    off = (units * 4 + 255) // 256 * 256
    assert int(ws[:off].count_nonzero()) == 0  # arrival counters left at zero
    assert int(ws[off:].count_nonzero()) > 0  # partials were written: the split ran
    small = torch.zeros(256, dtype=torch.uint8, device="cuda")
    _, _, _, unsplit = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=d + hq, workspace=small, case=case)
    check(case, q_lens, q, qu, unsplit, d)
    assert float(np.abs(out - unsplit).max()) <= 1e-3
    assert paged.device_error(0) == (0, 0)


@pytest.mark.parametrize("hq,hkv,d,page_size", [(28, 4, 128, 16), (14, 2, 64, 16), (28, 4, 128, 64)])
@pytest.mark.parametrize("phantom", [True, False])
def test_prefill_two_tiles_per_cta(cuda_device, hq, hkv, d, page_size, phantom):
    """At least two query tiles per SM at head_dim <= 128: two query tiles per
    CTA share each K/V tile.  Ragged chunks give pairs with and without a
    second tile and pairs whose tiles see different kv tile counts; the
    result matches the oracle and the one-tile kernel."""
    q_lens = [512, 300, 1, 777, 130, 1200, 128]
    kv_lens = [512 + 1000, 300, 1, 777 + 5000, 130 + 129, 1200 + 3, 128 + 64]
    assert (sum(q_lens) // 128) * hq >= 2 * torch.cuda.get_device_properties(0).multi_processor_count
    case, q, qu, out = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=hq + d + page_size, phantom=phantom,
                                   page_size=page_size)
    check(case, q_lens, q, qu, out, d, phantom=phantom)
    _, _, _, one = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=hq + d + page_size, phantom=phantom,
                               page_size=page_size, case=case, one_tile=True)
    check(case, q_lens, q, qu, one, d, phantom=phantom)
    assert float(np.abs(out - one).max()) <= 1e-3
    assert paged.device_error(0) == (0, 0)


@pytest.mark.parametrize("hq,hkv,d,page_size", [(14, 2, 64, 32), (28, 4, 128, 128)])
def test_prefill_two_tiles_page_sizes_bf16_out(cuda_device, hq, hkv, d, page_size):
    """The two-tile kernel at other page sizes (two pages and one page per
    128-key tile) with bf16 output."""
    q_lens = [384, 129, 1000, 256, 64, 900, 200]
    kv_lens = [384 + 2000, 129 + 7, 1000, 256 + 300, 64 + 4000, 900 + 128, 200 + 50]
    assert (sum(q_lens) // 128) * hq >= 2 * torch.cuda.get_device_properties(0).multi_processor_count
    case, q, qu, out = run_prefill(kv_lens, q_lens, hq, hkv, d, seed=3 * d + page_size, page_size=page_size,
                                   out_dtype=torch.bfloat16)
    check(case, q_lens, q, qu, out, d)
    assert paged.device_error(0) == (0, 0)


def test_prefill_split_head_dim_256_one_page_per_tile(cuda_device):
    """The split at head_dim 256 with 64-token pages (one page per 64-key kv
    tile) and a ragged second chunk."""
    from mitten_b200 import _lib as L
    q_lens, kv_lens = [300, 77], [6000, 77 + 2500]
    nb = L.lib().mtn_paged_prefill_workspace_bytes(len(q_lens), sum(q_lens), 4, 1, 256)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    case, q, qu, out = run_prefill(kv_lens, q_lens, 4, 1, 256, seed=11, page_size=64, workspace=ws)
    check(case, q_lens, q, qu, out, 256)
    units = (sum(q_lens) // 128 + len(q_lens)) * 4
    off = (units * 4 + 255) // 256 * 256
    assert int(ws[:off].count_nonzero()) == 0 and int(ws[off:].count_nonzero()) > 0
    assert paged.device_error(0) == (0, 0)
