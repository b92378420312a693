"""Pin the CPU oracle itself before trusting it (CPU only).

The attention restatement is checked against an independent torch-CPU f32
evaluation of the same reference op sequence (model.rs:394-416 with the
-1e10 mask of model.rs:542-555 and the GQA repeat of model.rs:398-408),
and the bf16 rounding against torch's own f32->bf16 conversion.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle


def torch_reference(q, kc, vc, scale):
    """The reference's tensor program written with torch ops, f32 on CPU."""
    q = torch.from_numpy(q)        # [S, Hq, D]
    kc = torch.from_numpy(kc)      # [Hkv, T, D]
    vc = torch.from_numpy(vc)
    S, Hq, D = q.shape
    Hkv, T, _ = kc.shape
    n_rep = Hq // Hkv
    k_ext = kc.reshape(Hkv, 1, T, D).repeat(1, n_rep, 1, 1).reshape(Hq, T, D)
    v_ext = vc.reshape(Hkv, 1, T, D).repeat(1, n_rep, 1, 1).reshape(Hq, T, D)
    i = torch.arange(S).view(S, 1)
    j = torch.arange(T).view(1, T)
    mask = torch.where(j > (T - S + i), torch.tensor(-1e10), torch.tensor(0.0))
    qh = q.transpose(0, 1)  # [Hq, S, D]
    attn = torch.softmax(qh @ k_ext.transpose(1, 2) * scale + mask, dim=-1)
    return (attn @ v_ext).transpose(0, 1).numpy()


@pytest.mark.parametrize("S,T,Hq,Hkv,D", [(1, 1, 2, 1, 64), (1, 37, 14, 2, 64), (5, 40, 14, 2, 64),
                                          (16, 16, 8, 1, 256), (7, 200, 28, 4, 128)])
def test_attention_matches_torch(S, T, Hq, Hkv, D):
    rng = np.random.default_rng(S * 1000 + T)
    q = rng.standard_normal((S, Hq, D)).astype(np.float32)
    kc = rng.standard_normal((Hkv, T, D)).astype(np.float32)
    vc = rng.standard_normal((Hkv, T, D)).astype(np.float32)
    kc[:, 0] = 0.0  # phantom zero row (model.rs:207-220)
    vc[:, 0] = 0.0
    got = oracle.attention(q, kc, vc, D ** -0.5)
    want = torch_reference(q, kc, vc, D ** -0.5)
    np.testing.assert_allclose(got, want, atol=2e-5, rtol=1e-4)


def test_phantom_row_only_adds_to_denominator():
    # One real key with score s: softmax over {0 (phantom), s} puts
    # 1/(1+exp(-s)) on the real value.
    D = 64
    q = np.zeros((1, 1, D), np.float32)
    q[0, 0, 0] = 8.0
    kc = np.zeros((1, 2, D), np.float32)
    vc = np.zeros((1, 2, D), np.float32)
    kc[0, 1, 0] = 1.0
    vc[0, 1, :] = 3.0
    out = oracle.attention(q, kc, vc, D ** -0.5)
    s = 8.0 * D ** -0.5
    np.testing.assert_allclose(out[0, 0], 3.0 / (1.0 + np.exp(-s)), rtol=1e-6)


def test_rne_matches_torch():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1.0, np.inf, -np.inf, 1e-40, 3.3895314e38], np.float32)])
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(oracle.rne_bf16_bits(x), want)


def test_catgrown_step_equals_attention():
    rng = np.random.default_rng(3)
    Hq, Hkv, D, n = 14, 2, 64, 3
    lens = [5, 17, 33]
    kp, vp = [], []
    for L_ in lens:
        k = rng.standard_normal((Hkv, L_, D)).astype(np.float32)
        v = rng.standard_normal((Hkv, L_, D)).astype(np.float32)
        k[:, 0] = 0
        v[:, 0] = 0
        kp.append(k)
        vp.append(v)
    dec = oracle.CatGrownDecode(kp, vp, Hq, D ** -0.5)
    q = rng.standard_normal((n, Hq, D)).astype(np.float32)
    kn = rng.standard_normal((n, Hkv, D)).astype(np.float32)
    vn = rng.standard_normal((n, Hkv, D)).astype(np.float32)
    out = dec.step(q, kn, vn)
    for r in range(n):
        kc = np.concatenate([kp[r], kn[r][:, None]], axis=1)
        vc = np.concatenate([vp[r], vn[r][:, None]], axis=1)
        np.testing.assert_allclose(out[r], oracle.attention(q[r:r + 1], kc, vc, D ** -0.5)[0], atol=1e-6)
    dec.close()
