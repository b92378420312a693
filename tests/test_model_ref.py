"""The numpy Qwen3_5Model restatement (oracle/model_ref.py) on CPU."""
from __future__ import annotations

import numpy as np

from oracle import model_ref as R

TINY = R.QwenShape(hidden=64, layers=2, hq=4, hkv=2, head_dim=16, inter=96, vocab=300)


def test_weight_map_matches_config1_names():
    names = dict(R.weight_names(R.CONFIG1))
    assert len(names) == 2 + 24 * 11
    assert names["layers.0.mixer.q_proj.weight"] == (1792, 896)  # q and gate per head (model.rs:289)
    assert names["embedding.weight"] == (151936, 896)
    assert "output.weight" not in names  # tied LM head


def test_chunked_prefill_matches_one_shot():
    w = R.random_weights(TINY, seed=0)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, TINY.vocab, 23)
    a, b = R.RefModel(TINY, w), R.RefModel(TINY, w)
    la = a.forward(0, ids, np.arange(23))
    lb = None
    for s in range(0, 23, 5):
        lb = b.forward(0, ids[s:s + 5], np.arange(s, min(23, s + 5)))
    np.testing.assert_allclose(la, lb, rtol=0, atol=1e-5)


def test_phantom_row_is_a_zero_key_and_value():
    # One token: softmax over {phantom (score 0, value 0), the token itself}.
    w = R.random_weights(TINY, seed=2)
    m = R.RefModel(TINY, w)
    m.init_cache(0)
    x = w["embedding.weight"][[7]]
    h = R.rms_norm(x, w["layers.0.norm.weight"], TINY.eps)
    m.attention(0, 0, h, np.array([0]))
    o = m.last_attn[0][0].reshape(TINY.hq, TINY.head_dim)
    k = R.rms_norm((h @ w["layers.0.mixer.k_proj.weight"].T).reshape(1, TINY.hkv, TINY.head_dim),
                   w["layers.0.mixer.k_norm.weight"], TINY.eps)
    v = (h @ w["layers.0.mixer.v_proj.weight"].T).reshape(TINY.hkv, TINY.head_dim)
    qg = (h @ w["layers.0.mixer.q_proj.weight"].T).reshape(TINY.hq, 2, TINY.head_dim)
    q = R.rms_norm(qg[:, 0], w["layers.0.mixer.q_norm.weight"], TINY.eps)
    for hh in range(TINY.hq):
        g = hh // (TINY.hq // TINY.hkv)
        s = float(q[hh] @ k[0, g]) * TINY.head_dim ** -0.5  # position 0: RoPE is the identity
        p = np.exp(s) / (np.exp(s) + 1.0)
        np.testing.assert_allclose(o[hh], p * v[g], rtol=1e-5, atol=1e-6)


def test_rne_bf16_ties_to_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], np.float32)
    np.testing.assert_array_equal(R.rne_bf16(x), np.array([1.0, 1.0 + 2 ** -6, -2.5, 0.0], np.float32))


def test_greedy_first_max_takes_the_first_of_ties():
    assert R.greedy_first_max(np.array([0.5, 2.0, 2.0, 1.0], np.float32)) == 1
