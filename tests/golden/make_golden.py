"""Writes tests/golden/attention_golden.npz: seeded paged-attention cases and the
f32 oracle's outputs for them.

The reference computes attention inside Burn 0.16.1 (qwen model.rs:394-416),
which cannot be built here, so these fixtures pin the oracle's restatement
(oracle/attention_ref.c: GQA repeat, -1e10 causal mask, max-subtracted
softmax, optional all-zero first row) rather than the reference itself: the
CPU test re-runs the oracle on the same inputs and requires the stored
outputs, and the GPU test holds the kernels to them within the spec's 2e-2.
Inputs are regenerated from the seeds; their SHA-256 digests are stored so a
change in the generator is caught.

Run from the repo root:  python -m tests.golden.make_golden
"""
from __future__ import annotations

import hashlib
import pathlib

import numpy as np

import oracle

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "attention_golden.npz"

# decode: one query per sequence at position len-1 (the step's token already stored)
# prefill: q_lens[r] queries at the last positions of lens[r]
CASES = [
    dict(name="decode_gqa7_d64", kind="decode", hq=14, hkv=2, d=64, lens=[1, 17, 300], phantom=True, seed=101),
    dict(name="decode_mqa_d256", kind="decode", hq=8, hkv=1, d=256, lens=[100, 513], phantom=False, seed=102),
    dict(name="decode_gqa7_d128", kind="decode", hq=28, hkv=4, d=128, lens=[129, 1000], phantom=True, seed=105),
    dict(name="prefill_gqa7_d64", kind="prefill", hq=14, hkv=2, d=64, lens=[200, 77], q_lens=[72, 77],
         phantom=True, seed=103),
    dict(name="prefill_gqa4_d128", kind="prefill", hq=8, hkv=2, d=128, lens=[300], q_lens=[300], phantom=True,
         seed=104),
    dict(name="prefill_mqa_d256", kind="prefill", hq=8, hkv=1, d=256, lens=[640], q_lens=[130], phantom=False,
         seed=106),
    # Launches with at least two query tiles per SM (148): the two-query-tile
    # kernel.  Every 97th output row is stored.
    dict(name="prefill_pair_gqa7_d128", kind="prefill", hq=28, hkv=4, d=128, lens=[1412, 512, 2384],
         q_lens=[512, 512, 384], phantom=True, seed=107, stride=97),
    dict(name="prefill_pair_gqa7_d64", kind="prefill", hq=14, hkv=2, d=64, lens=[1324, 1024, 2268],
         q_lens=[1024, 1024, 768], phantom=False, seed=108, stride=97),
]


def inputs(case: dict):
    """q [rows, hq, d] and per-sequence k, v [len, hkv, d], f32 N(0, 1)."""
    rng = np.random.default_rng(case["seed"])
    ks = [rng.standard_normal((n, case["hkv"], case["d"])).astype(np.float32) for n in case["lens"]]
    vs = [rng.standard_normal((n, case["hkv"], case["d"])).astype(np.float32) for n in case["lens"]]
    rows = sum(case["q_lens"]) if case["kind"] == "prefill" else len(case["lens"])
    q = rng.standard_normal((rows, case["hq"], case["d"])).astype(np.float32)
    return q, ks, vs


def digest(q, ks, vs) -> str:
    h = hashlib.sha256()
    for a in [q, *ks, *vs]:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def oracle_outputs(case: dict, q, ks, vs) -> np.ndarray:
    d, out = case["d"], []
    q_lens = case["q_lens"] if case["kind"] == "prefill" else [1] * len(case["lens"])
    off = 0
    for r, ql in enumerate(q_lens):
        kc, vc = ks[r].transpose(1, 0, 2), vs[r].transpose(1, 0, 2)
        if case["phantom"]:
            z = np.zeros((kc.shape[0], 1, d), np.float32)
            kc, vc = np.concatenate([z, kc], axis=1), np.concatenate([z, vc], axis=1)
        out.append(oracle.attention(q[off:off + ql], kc, vc, d ** -0.5))
        off += ql
    return np.concatenate(out)


def kept_rows(n_rows: int, stride: int = 7) -> np.ndarray:
    """The output rows stored (every `stride`-th and the last), to keep the fixture small."""
    return np.unique(np.concatenate([np.arange(0, n_rows, stride), [n_rows - 1]]))


def main() -> None:
    arrays = {}
    for case in CASES:
        q, ks, vs = inputs(case)
        out = oracle_outputs(case, q, ks, vs)
        arrays[case["name"] + "/out"] = out[kept_rows(out.shape[0], case.get("stride", 7))]
        arrays[case["name"] + "/digest"] = np.frombuffer(bytes.fromhex(digest(q, ks, vs)), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
