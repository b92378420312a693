"""Paged decode with a host-made work plan (mtn_paged_decode_with_plan) on the
GPU: the same oracle bounds as the unplanned kernel (tests/test_gpu_decode.py)
on GQA / MQA shapes, empty and short sequences, the fused append and a
config-2-sized batch; results within 2e-3 of the unplanned launch (the two
split the tiles differently, and each piece rounds its softmax weights to
bf16 against its own reference maximum: 2^-9 relative per weight);
deterministic; and a plan that does not fit the launch is reported as
device error 6 without a fault."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from mitten_b200 import paged
from tests.paged_case import make_case
from tests.test_gpu_decode import check

pytestmark = pytest.mark.gpu


def _plan_for(case):
    return paged.DecodePlan(case.pool.head_dim, "cuda").build(case.kv_indptr.cpu().numpy(), case.seq_lens.cpu().numpy(),
                                                              case.pool.page_size, case.pool.num_kv_heads)


def _run(case, q, plan=None, **kw):
    out = paged.paged_decode(case.pool, 0, q, case.kv_indptr, case.kv_indices, case.seq_lens, phantom=True,
                             out_dtype=torch.float32, plan=plan, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 1, 256), (16, 2, 64)])
def test_plan_matches_oracle_and_unplanned(cuda_device, hq, hkv, d):
    rng = np.random.default_rng(d + hq)
    lens = [0, 1, 16, 129, 3000, 0, 257] + rng.integers(1, 5000, size=40).tolist()
    case = make_case(lens, hkv, d, seed=hq)
    q32 = rng.standard_normal((len(lens), hq, d)).astype(np.float32)
    q = torch.from_numpy(q32).cuda().to(torch.bfloat16)
    plan = _plan_for(case)
    got = _run(case, q, plan)
    check(case, hq, d, q32, oracle.round_bf16(q32), got)
    np.testing.assert_allclose(got, _run(case, q), atol=2e-3, rtol=0)
    np.testing.assert_array_equal(got, _run(case, q, plan))  # deterministic
    assert paged.device_error(0) == (0, 0)


def test_plan_config2_batch_with_fused_append(cuda_device):
    rng = np.random.default_rng(2)
    lens = rng.integers(256, 4097, size=64).tolist()
    hq, hkv, d = 14, 2, 64
    case = make_case(lens, hkv, d, seed=3)
    kn = rng.standard_normal((64, hkv, d)).astype(np.float32)
    vn = rng.standard_normal((64, hkv, d)).astype(np.float32)
    for r in range(64):
        case.k[r][-1] = kn[r]
        case.v[r][-1] = vn[r]
    q32 = rng.standard_normal((64, hq, d)).astype(np.float32)
    q = torch.from_numpy(q32).cuda().to(torch.bfloat16)
    got = _run(case, q, _plan_for(case), k_new=torch.from_numpy(kn).cuda().to(torch.bfloat16),
               v_new=torch.from_numpy(vn).cuda().to(torch.bfloat16))
    check(case, hq, d, q32, oracle.round_bf16(q32), got)
    assert paged.device_error(0) == (0, 0)


def test_plan_one_long_sequence_many_pieces(cuda_device):
    case = make_case([20000], 2, 64, seed=9)
    q32 = np.random.default_rng(9).standard_normal((1, 14, 64)).astype(np.float32)
    got = _run(case, torch.from_numpy(q32).cuda().to(torch.bfloat16), _plan_for(case))
    check(case, 14, 64, q32, oracle.round_bf16(q32), got)


def test_mismatched_plan_is_flagged_not_faulted(cuda_device):
    case = make_case([300, 40], 2, 64, seed=4)
    q = torch.randn(2, 14, 64, device="cuda").to(torch.bfloat16)
    plan = _plan_for(case)
    paged.device_error(0, clear=True)
    bad = paged.DecodePlan(64, "cuda")
    bad.dev.zero_()  # not a plan
    _run(case, q, bad)
    assert paged.device_error(0, clear=True) == (6, -1)
    w = plan.words()
    w[2] += 1  # made for another grid
    bad.host.copy_(torch.from_numpy(w.view(np.uint8)))
    bad.dev.copy_(bad.host)
    _run(case, q, bad)
    assert paged.device_error(0, clear=True) == (6, int(w[2]))
    # the context is fine: a good plan still gives the oracle's result
    q32 = q.float().cpu().numpy()
    check(case, 14, 64, q32, q32, _run(case, q, plan))
