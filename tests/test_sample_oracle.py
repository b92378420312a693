"""sample_token (inference-engine/src/scheduler.rs:186-223) restated three
times on the CPU must agree token for token: the C oracle with libm's expf
(oracle.sample_token, what Rust's f32::exp calls), the pure-Python
restatement (oracle.host_ref.sample_token) and the C++ scheduler mirror's
own sampler (reached through process_logits).  The device kernel is held to
the C oracle in tests/test_gpu_sampling.py.

Rows: N(0, s) logits at vocab sizes up to config 1's 151 936, at several
temperatures and greedy, the StubBackend's one-hot rows, rows with -inf
and NaN entries, and rows whose exponentials overflow (the reference then
returns the last index)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import oracle.host_ref as ref
from mitten_b200 import _lib, host


def _rows():
    rng = np.random.default_rng(17)
    rows = []
    for vocab, scale, temps in [(151936, 1.0, (0.0, 0.7, 1.0)), (4096, 3.0, (0.0, 0.5, 1.3)),
                                (100, 1.0, (1.0, 2.0)), (7, 1.0, (1.0,))]:
        for _ in range(3):
            x = (rng.standard_normal(vocab) * scale).astype(np.float32)
            rows += [(x, t) for t in temps]
    stub = np.zeros(100, np.float32)
    stub[42] = 10.0
    rows += [(stub, 1.0), (stub, 0.0)]
    neg = rng.standard_normal(500).astype(np.float32)
    neg[:250] = -np.inf
    rows += [(neg, 1.0), (neg, 0.0)]
    nan = rng.standard_normal(300).astype(np.float32)
    nan[[0, 17, 299]] = np.nan
    rows += [(nan, 0.0), (nan, 1.0)]
    big = (rng.standard_normal(1000) * 50).astype(np.float32)
    rows += [(big, 0.5)]  # exp overflows to inf: sum inf, every e/sum NaN -> last index
    return rows


def _mirror_sample(row, temperature):
    s = host.Scheduler(8, 4, mode=_lib.MTN_SCHED_REFERENCE)
    s.add_request(1, [1, 2, 3], temperature, 2)
    assert s.schedule() is not None
    s.process_logits(row[None, :])
    return s.request_output(1)[0]


@pytest.mark.filterwarnings("ignore::RuntimeWarning")  # the overflow row overflows on purpose
@pytest.mark.parametrize("k", range(len(_rows())))
def test_three_restatements_agree(k):
    row, t = _rows()[k]
    want = oracle.sample_token(row, t)
    assert 0 <= want < row.size
    assert ref.sample_token(row, t) == want
    assert _mirror_sample(row, t) == want


def test_overflow_row_returns_last_index():
    row, t = _rows()[-1]
    assert oracle.sample_token(row, t) == row.size - 1
