"""The allocation-free decode entry point, through the C ABI.

mtn_paged_decode_noalloc serves callers that cannot call cudaMalloc: an
engine whose device memory is all handed out at start-up by its own arena
(the KV pool takes nearly all of HBM), or a serving loop that must not
allocate mid-step because an allocation can synchronise the device.  It
uses a static scratch array inside the library instead of a caller
workspace.  On two calls in a row that share that scratch (the second one
also appending the step's K/V row), at head_dim 64, 128 and 256 (each puts
the scratch's arrival counters at a different offset), its output must
match mtn_paged_decode's and the f32 oracle's (fed the bf16 values the
kernel reads), within the decode tests' 1e-2.  This file sorts last so a
run that stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import _lib, paged
from tests.paged_case import make_case

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _noalloc(case, q, out, phantom, k_new=None, v_new=None):
    lib = _lib.lib()
    n, hq, _ = q.shape
    flags = _lib.MTN_ATTN_PHANTOM_ZERO_SLOT if phantom else 0
    st = lib.mtn_paged_decode_noalloc(
        C.byref(case.pool.layout), 0, q.data_ptr(), _lib.MTN_DTYPE_BF16, out.data_ptr(), _lib.MTN_DTYPE_F32,
        None if k_new is None else k_new.data_ptr(), None if v_new is None else v_new.data_ptr(),
        _lib.MTN_DTYPE_BF16, n, hq, case.kv_indptr.data_ptr(), case.kv_indices.data_ptr(),
        case.seq_lens.data_ptr(), q.shape[-1] ** -0.5, flags, torch.cuda.current_stream().cuda_stream)
    _lib.check(st)


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256)])
def test_noalloc_matches_workspace_entry_point_and_oracle_twice(cuda_device, hq, hkv, d):
    # Long and short sequences, so segments are split across CTAs and the
    # scratch's partials and arrival counters are exercised on both calls.
    lens = [10000, 3000, 17, 1, 129, 0, 2048]
    case = make_case(lens, hkv, d, seed=41 + d)
    rng = np.random.default_rng(42 + d)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((len(lens), hq, d)).astype(np.float32)).cuda().to(torch.bfloat16)
        kn = vn = None
        if call == 1:  # the second call also stores each sequence's newest K/V row (fused append)
            kn32 = rng.standard_normal((len(lens), hkv, d)).astype(np.float32)
            vn32 = rng.standard_normal((len(lens), hkv, d)).astype(np.float32)
            kn = torch.from_numpy(kn32).cuda().to(torch.bfloat16)
            vn = torch.from_numpy(vn32).cuda().to(torch.bfloat16)
            for r, n in enumerate(lens):
                if n:
                    case.k[r][-1] = kn32[r]
                    case.v[r][-1] = vn32[r]
        got = torch.empty((len(lens), hq, d), dtype=torch.float32, device="cuda")
        _noalloc(case, q, got, phantom=True, k_new=kn, v_new=vn)
        # the workspace entry point on the same inputs (its append rewrites the same rows)
        want = paged.paged_decode(case.pool, 0, q, case.kv_indptr, case.kv_indices, case.seq_lens, phantom=True,
                                  out_dtype=torch.float32, k_new=kn, v_new=vn)
        torch.cuda.synchronize()
        got_h = got.cpu().numpy()
        np.testing.assert_allclose(got_h, want.cpu().numpy(), atol=TOL, rtol=0, err_msg=f"call {call}")
        q_used = q.float().cpu().numpy()
        for r in range(len(lens)):
            kb, vb = case.oracle_cache(r, layer_round=True, phantom=True)
            ref = oracle.attention(q_used[r:r + 1], kb, vb, d ** -0.5)[0]
            np.testing.assert_allclose(got_h[r], ref, atol=TOL, rtol=0, err_msg=f"call {call}, sequence {r}")
    assert paged.device_error(0) == (0, 0)


def test_noalloc_rejects_batches_beyond_the_scratch(cuda_device):
    # 4 million sequence x kv-head pairs need more than the 8 MiB scratch;
    # the call is refused before anything is launched.
    case = make_case([4], 2, 64, seed=43)
    q = torch.zeros(1, 14, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, 14, 64, dtype=torch.float32, device="cuda")
    lib = _lib.lib()
    st = lib.mtn_paged_decode_noalloc(C.byref(case.pool.layout), 0, q.data_ptr(), _lib.MTN_DTYPE_BF16,
                                      out.data_ptr(), _lib.MTN_DTYPE_F32, None, None, 0, 2_000_000, 14,
                                      case.kv_indptr.data_ptr(), case.kv_indices.data_ptr(),
                                      case.seq_lens.data_ptr(), 0.125, 0, None)
    assert st == _lib.MTN_EINVAL
    assert b"static scratch" in lib.mtn_last_error()
