"""Failure detection without a GPU fault.

Every wait inside the kernels is bounded: a wait that nothing completes gives
up after ~1 s, records the timeout in the per-device error word and returns,
so the host sees an error status and the CUDA context stays usable.  The
self-test entry point runs exactly such a wait (an mbarrier nobody arrives
at); a decode on the same context right after must still match the oracle.
"""
from __future__ import annotations

import time

import pytest
import torch

from mitten_b200 import _lib, paged
from tests.paged_case import make_case
from tests.test_gpu_decode import check, run_decode

pytestmark = pytest.mark.gpu

TIMEOUT_CODE = 4  # kDevErrTimeout, the code MTN_ETIMEOUT mirrors
SELFTEST_DETAIL = 99


def test_bounded_wait_gives_up_and_context_survives(cuda_device):
    paged.device_error(0, clear=True)
    t0 = time.monotonic()
    _lib.check(_lib.lib().mtn_selftest_bounded_wait(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert paged.device_error(0, clear=True) == (TIMEOUT_CODE, SELFTEST_DETAIL)
    assert 0.5 < waited < 30.0, waited  # the ~1 s bound, not a hang
    # Same context, same device: a normal decode runs and is correct.
    case = make_case([1, 37, 300, 1000], 2, 64, seed=5)
    q, qu, out = run_decode(case, 14, 64)
    check(case, 14, 64, q, qu, out)
    assert paged.device_error(0) == (0, 0)
