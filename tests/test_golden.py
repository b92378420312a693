"""The oracle against the committed golden fixtures (tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest

from tests.golden import make_golden as G


@pytest.fixture(scope="module")
def golden():
    return np.load(G.OUT)


@pytest.mark.parametrize("case", G.CASES, ids=[c["name"] for c in G.CASES])
def test_oracle_reproduces_golden(golden, case):
    q, ks, vs = G.inputs(case)
    assert bytes(golden[case["name"] + "/digest"]).hex() == G.digest(q, ks, vs)  # same inputs as when written
    out = G.oracle_outputs(case, q, ks, vs)
    np.testing.assert_allclose(out[G.kept_rows(out.shape[0], case.get("stride", 7))], golden[case["name"] + "/out"], rtol=0, atol=1e-6)
