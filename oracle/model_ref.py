"""TEST INFRASTRUCTURE -- numpy f32 restatement of Qwen3_5Model::forward.

Follows inference-model-qwen/src/model.rs with every layer a full-attention
layer (config 1 sets layer_types so; GatedDeltaNet is out of scope):

  RmsNorm::forward / forward4   model.rs:98-108   x / sqrt(mean(x^2) + eps) * (1 + w)
  embedding splits               model.rs:159-183  numerically a plain row lookup
  Qwen3_5Layer::forward          model.rs:348-365  pre-norm attention + SwiGLU MLP
  GatedAttention::forward        model.rs:369-422  q/gate interleaved per head, q/k norm,
                                                   RoPE, cat-grown cache, GQA repeat,
                                                   softmax(S * scale + mask), sigmoid gate
  init_cache                     model.rs:207-220  caches start with one zero row
  apply_rope                     model.rs:508-540  rotate-half over rotary_dim, f32 powf
  generate_causal_mask           model.rs:542-555  -1e10 where j > T - s + i
  tied LM head                   model.rs:185-205, 262-276

Each request has its own contiguous cache (the reference backend keeps one
per request, burn_backend.rs:44-71).  `kv_round` optionally rounds each
appended K/V row to bf16 (round-to-nearest-even), the storage precision of
the paged pool, so that a comparison isolates the kernels' arithmetic.

Only tests and __graft_entry__.smoke() use this module, as the checker.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class QwenShape:
    hidden: int
    layers: int
    hq: int
    hkv: int
    head_dim: int
    inter: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6
    partial_rotary: float = 1.0
    gated_q: bool = True    # q_proj carries a sigmoid gate per head (model.rs:372-375, 417)
    qk_norm: bool = True    # RMSNorm (1 + w) over each head of q and k (model.rs:380-381)
    phantom: bool = True    # caches start with one zero row (model.rs:207-220)
    mlp: str = "swiglu"     # silu(gate) * up; "geglu": gelu_tanh(gate) * up

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)  # config.rs:39-42


# Qwen2.5-0.5B-shaped decoder.
CONFIG1 = QwenShape(hidden=896, layers=24, hq=14, hkv=2, head_dim=64, inter=4864, vocab=151936)
# Gemma-2B shapes.  The reference Gemma model has no attention
# (inference-model-gemma/src/model.rs:82-94) and empty caches (:96-105); this is the
# attention layer above at these shapes, without the Qwen gate and q/k norms, RoPE theta 1e4,
# GeGLU MLP and no phantom row.
GEMMA_2B = QwenShape(hidden=2048, layers=18, hq=8, hkv=1, head_dim=256, inter=16384, vocab=256000, theta=1e4,
                     gated_q=False, qk_norm=False, phantom=False, mlp="geglu")


def weight_names(cfg: QwenShape) -> list[tuple[str, tuple[int, ...]]]:
    """The name -> shape map new_with_weights consumes (model.rs:224-344), in a fixed order."""
    h, d = cfg.hidden, cfg.head_dim
    names = [("embedding.weight", (cfg.vocab, h)), ("norm.weight", (h,))]
    for i in range(cfg.layers):
        p = f"layers.{i}"
        m = f"{p}.mixer"
        names += [
            (f"{p}.norm.weight", (h,)),
            (f"{m}.q_proj.weight", (cfg.hq * d * (2 if cfg.gated_q else 1), h)),
            (f"{m}.k_proj.weight", (cfg.hkv * d, h)),
            (f"{m}.v_proj.weight", (cfg.hkv * d, h)),
            (f"{m}.o_proj.weight", (h, cfg.hq * d)),
        ]
        if cfg.qk_norm:
            names += [(f"{m}.q_norm.weight", (d,)), (f"{m}.k_norm.weight", (d,))]
        names += [
            (f"{p}.ffn_norm.weight", (h,)),
            (f"{p}.mlp.gate_proj.weight", (cfg.inter, h)),
            (f"{p}.mlp.up_proj.weight", (cfg.inter, h)),
            (f"{p}.mlp.down_proj.weight", (h, cfg.inter)),
        ]
    return names


def random_weights(cfg: QwenShape, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Every weight N(0, std) in f32 from one seeded generator, in weight_names order."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in weight_names(cfg):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(std)
        out[name] = a
    return out


def rne_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even), returned as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(x)
    out = r.view(np.float32).copy()
    out[nan] = np.float32(np.nan)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """model.rs:98-108, over the last axis."""
    var = np.mean(np.square(x, dtype=np.float32), axis=-1, keepdims=True, dtype=np.float32)
    y = x * (np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32))
    return (y * (w + np.float32(1.0))).astype(np.float32)


def rope_freqs(cfg: QwenShape) -> np.ndarray:
    """1 / theta^(2i / rotary_dim) in f32 (model.rs:511-514)."""
    half = cfg.rotary_dim // 2
    i = np.arange(half, dtype=np.float32)
    return (np.float32(1.0) / np.power(np.float32(cfg.theta), np.float32(2.0) * i / np.float32(cfg.rotary_dim),
                                       dtype=np.float32)).astype(np.float32)


def apply_rope(x: np.ndarray, pos: np.ndarray, cfg: QwenShape) -> np.ndarray:
    """x [seq, heads, head_dim], pos [seq]: rotate-half over the first rotary_dim (model.rs:508-540)."""
    rd, half = cfg.rotary_dim, cfg.rotary_dim // 2
    ang = pos.astype(np.float32)[:, None, None] * rope_freqs(cfg)[None, None, :]
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x1, x2 = x[..., :half], x[..., half:rd]
    out = np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)
    if rd < x.shape[-1]:
        out = np.concatenate([out, x[..., rd:]], axis=-1)
    return out


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(np.float32(0.7978845608028654) *
                                                            (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


class RefModel:
    """Qwen3_5Model::forward over per-request contiguous caches (f32)."""

    def __init__(self, cfg: QwenShape, weights: dict[str, np.ndarray], kv_round: bool = False,
                 p_round: bool = False, q_round_prefill: bool = False, q_round: bool = False):
        # p_round / q_round_prefill round the probabilities (and the queries of multi-token calls) to
        # bf16 the way the tensor-core kernels do: diagnostics that attribute differences, not the
        # reference's arithmetic.
        self.cfg, self.w, self.kv_round = cfg, weights, kv_round
        self.p_round, self.q_round_prefill, self.q_round = p_round, q_round_prefill, q_round
        self.caches: dict[int, list[tuple[np.ndarray, np.ndarray]]] = {}
        self.last_attn: dict[int, list[np.ndarray]] = {}  # per request, per layer: the last call's attention output

    def init_cache(self, rid: int) -> None:
        """model.rs:207-220: every layer's K and V start as one zero row per kv head."""
        c = self.cfg
        z = np.zeros((c.hkv, 1 if c.phantom else 0, c.head_dim), np.float32)
        self.caches[rid] = [(z.copy(), z.copy()) for _ in range(c.layers)]

    def attention(self, li: int, rid: int, x: np.ndarray, pos: np.ndarray) -> np.ndarray:
        """GatedAttention::forward (model.rs:369-422) for one request's `seq` rows."""
        c, w = self.cfg, self.w
        m = f"layers.{li}.mixer"
        seq = x.shape[0]
        if c.gated_q:
            qg = (x @ w[f"{m}.q_proj.weight"].T).reshape(seq, c.hq, 2, c.head_dim)
            q, gate = qg[:, :, 0, :], qg[:, :, 1, :].reshape(seq, c.hq * c.head_dim)
        else:
            q, gate = (x @ w[f"{m}.q_proj.weight"].T).reshape(seq, c.hq, c.head_dim), None
        k = (x @ w[f"{m}.k_proj.weight"].T).reshape(seq, c.hkv, c.head_dim)
        v = (x @ w[f"{m}.v_proj.weight"].T).reshape(seq, c.hkv, c.head_dim)
        if c.qk_norm:
            q = rms_norm(q, w[f"{m}.q_norm.weight"], c.eps)
            k = rms_norm(k, w[f"{m}.k_norm.weight"], c.eps)
        q, k = apply_rope(q, pos, c), apply_rope(k, pos, c)
        if self.q_round or (self.q_round_prefill and seq > 1):
            q = rne_bf16(q)
        if self.kv_round:
            k, v = rne_bf16(k), rne_bf16(v)
        kc, vc = self.caches[rid][li]
        kc = np.concatenate([kc, k.transpose(1, 0, 2)], axis=1)  # Tensor::cat along the sequence axis
        vc = np.concatenate([vc, v.transpose(1, 0, 2)], axis=1)
        self.caches[rid][li] = (kc, vc)
        total = kc.shape[1]
        n_rep = c.hq // c.hkv
        kx = np.repeat(kc, n_rep, axis=0)  # q head h reads kv head h // n_rep
        vx = np.repeat(vc, n_rep, axis=0)
        i = np.arange(seq)[:, None]
        j = np.arange(total)[None, :]
        mask = np.where(j > total - seq + i, np.float32(-1e10), np.float32(0.0)).astype(np.float32)
        qh = q.transpose(1, 0, 2)  # [hq, seq, d]
        s = np.matmul(qh, kx.transpose(0, 2, 1)) * np.float32(c.head_dim ** -0.5) + mask[None]
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        l = p.sum(axis=-1, keepdims=True)
        if self.p_round:
            p = rne_bf16(p)
        p = p / l
        o = np.matmul(p, vx).transpose(1, 0, 2).reshape(seq, c.hq * c.head_dim).astype(np.float32)
        self.last_attn.setdefault(rid, [None] * c.layers)[li] = o
        if gate is not None:
            o = sigmoid(gate) * o
        return (o @ w[f"{m}.o_proj.weight"].T).astype(np.float32)

    def forward(self, rid: int, ids: np.ndarray, pos: np.ndarray) -> np.ndarray:
        """Qwen3_5Model::forward for one request's new tokens; returns the logits of its last row."""
        c, w = self.cfg, self.w
        if rid not in self.caches:
            self.init_cache(rid)
        x = w["embedding.weight"][np.asarray(ids, dtype=np.int64)].astype(np.float32)
        for li in range(c.layers):
            p = f"layers.{li}"
            x = x + self.attention(li, rid, rms_norm(x, w[f"{p}.norm.weight"], c.eps), pos)
            h = rms_norm(x, w[f"{p}.ffn_norm.weight"], c.eps)
            g = h @ w[f"{p}.mlp.gate_proj.weight"].T
            u = h @ w[f"{p}.mlp.up_proj.weight"].T
            act = silu(g) if c.mlp == "swiglu" else gelu_tanh(g)
            x = x + (act * u) @ w[f"{p}.mlp.down_proj.weight"].T
        last = rms_norm(x[-1:], w["norm.weight"], c.eps)
        return (last @ w["embedding.weight"].T)[0].astype(np.float32)


def greedy_first_max(logits: np.ndarray) -> int:
    """sample_token with temperature <= 0 (scheduler.rs:186-199): the first strict maximum."""
    best, arg = -np.inf, 0
    for i, v in enumerate(logits.tolist()):
        if v > best:
            best, arg = v, i
    return arg


def generate(model: RefModel, prompts: list[np.ndarray], steps: int, chunk: int | None = None,
             logits_out: list | None = None) -> list[list[int]]:
    """Prefill every prompt (in chunks of `chunk` tokens if given), then greedy tokens until each request
    has `steps` of them (the first comes from the prompt's last logits).  `logits_out`, if given,
    receives per request the logits every token was chosen from."""
    out = []
    for rid, prompt in enumerate(prompts):
        n = len(prompt)
        c = chunk or n
        logits = None
        for a in range(0, n, c):
            b = min(n, a + c)
            logits = model.forward(rid, prompt[a:b], np.arange(a, b))
        seen = [logits]
        toks = [greedy_first_max(logits)]
        for s in range(1, steps):
            pos = n + s - 1
            logits = model.forward(rid, np.array([toks[-1]]), np.array([pos]))
            seen.append(logits)
            toks.append(greedy_first_max(logits))
        out.append(toks)
        if logits_out is not None:
            logits_out.append(seen)
    return out
