"""Model call sites over the paged KV pool: the CUDA backend's forward.

`QwenPagedModel.forward(batch)` is the B200 form of
`BackendHandle::forward` (inference-backend/src/backend.rs:16-21) for
Qwen3_5Model with full-attention layers (inference-model-qwen/src/model.rs):
one call serves the scheduler's whole CSR batch (prefill rows first, then
decode rows) instead of the reference's per-request loop with private
contiguous caches (burn_backend.rs:31-80), and returns one logits row per
request (the last token of its rows), like `Logits` (backend.rs:8-12).

Per layer, the dense work stays on the device's BLAS in f32 (q/k/v/o
projections, q/k RMSNorm (1 + w), RoPE, SwiGLU); the paged-KV path is this
library's kernels:
  prefill rows  mtn_build_slot_mapping + mtn_kv_append, then
                mtn_paged_prefill (causal over the pool, phantom zero key)
  decode rows   mtn_paged_decode with the step's K/V appended in the same
                launch (phantom zero key)
The reference's cache starts with one all-zero K/V row per layer
(model.rs:207-220); MTN_ATTN_PHANTOM_ZERO_SLOT reproduces that key without
storing it, so position p of a sequence lives in pool slot p.

The same class is the attention call site the Gemma crate lacks
(inference-model-gemma/src/model.rs:82-94 has none): `GEMMA_2B` runs the
layer at Gemma-2B shapes (MQA, head_dim 256, GeGLU MLP, theta 1e4) without
the Qwen gate, q/k norms or phantom row (Gemma's caches start empty,
model.rs:96-105).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from . import paged


@dataclass(frozen=True)
class DecoderShape:
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
    gated_q: bool = True      # Qwen3.5 q_proj carries a sigmoid gate per head
    qk_norm: bool = True      # RMSNorm (1 + w) over each head of q and k
    phantom: bool = True      # Qwen caches start with one zero row; Gemma's start empty
    mlp: str = "swiglu"       # "swiglu" (Qwen) or "geglu" (Gemma)

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)


QWEN_CONFIG1 = DecoderShape(hidden=896, layers=24, hq=14, hkv=2, head_dim=64, inter=4864, vocab=151936)
GEMMA_2B = DecoderShape(hidden=2048, layers=18, hq=8, hkv=1, head_dim=256, inter=16384, vocab=256000, theta=1e4,
                        gated_q=False, qk_norm=False, phantom=False, mlp="geglu")


def _rms(x: torch.Tensor, w1: torch.Tensor, eps: float) -> torch.Tensor:
    """RmsNorm::forward (model.rs:98-108): x / sqrt(mean(x^2) + eps) * (1 + w), last axis; w1 = 1 + w."""
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), w1, eps)


class QwenPagedModel:
    """Qwen3_5Model (all layers full attention) over a PagedKVPool."""

    def __init__(self, shape: DecoderShape, weights: dict, num_pages: int, page_size: int = 16,
                 device: torch.device | str = "cuda", split_bf16: bool = True, dtype: torch.dtype = torch.float32,
                 fused_prologue: bool = True, decode_plan: bool = True):
        self.s = shape
        # Dense weights and activations in `dtype` (f32: the reference's CPU
        # path; bf16: the random-bf16 configs 3-5).  RoPE is applied in f32 and
        # the attention kernels take f32 q/k/v either way.
        # The dense path is f32, like the reference's (model.rs:413-416
        # multiplies in f32): q and the softmax weights reach the tensor cores
        # as bf16 hi + lo pairs (MTN_ATTN_SPLIT_BF16) unless split_bf16=False;
        # prefill can split only at head_dim <= 128.
        self.split_dec = split_bf16
        self.split_pre = split_bf16 and shape.head_dim <= 128
        self.dev = torch.device(device)
        self.dt = dtype
        # fused_prologue: q/k RMSNorm + RoPE + the K/V store in one kernel
        # (mtn_qkv_prologue) instead of torch ops and a separate append.
        self.fused = fused_prologue and shape.rotary_dim % 64 == 0
        self.w = {k: torch.as_tensor(v).to(self.dev, dtype) for k, v in weights.items()}
        # RMSNorm scales (1 + w), formed once
        for k in [k for k in self.w if k.endswith("norm.weight")]:
            self.w[k] = self.w[k] + 1.0
        self.pool = paged.PagedKVPool(shape.layers, num_pages, page_size, shape.hkv, shape.head_dim, device=self.dev)
        half = shape.rotary_dim // 2
        i = np.arange(half, dtype=np.float32)
        # 1 / theta^(2i / rotary_dim) in f32, as model.rs:511-514 computes it
        inv = np.float32(1.0) / np.power(np.float32(shape.theta), np.float32(2.0) * i / np.float32(shape.rotary_dim),
                                         dtype=np.float32)
        self.inv_freq = torch.from_numpy(inv.astype(np.float32)).to(self.dev)
        # (1 + w) of the q/k norms in f32 for the fused prologue
        self.w32 = {k: v.float().contiguous() for k, v in self.w.items() if k.endswith(("q_norm.weight", "k_norm.weight"))}
        self.scale = shape.head_dim ** -0.5
        self._ws = None
        self._ws_seqs = 0
        self._pws = None
        self._plan = None
        # decode_plan: pass the decode kernel a host-made work plan
        # (mtn_paged_decode_plan) instead of letting it split the tiles itself.
        self.use_plan = decode_plan
        self._graphs: dict[int, _DecodeGraph] = {}

    # ------------------------------------------------------------ pieces
    def _rope_tables(self, pos: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """cos and sin of pos * inv_freq [T, 1, rotary_dim/2], shared by q, k and every layer."""
        ang = pos.to(torch.float32)[:, None, None] * self.inv_freq[None, None, :]
        return torch.cos(ang), torch.sin(ang)

    def _rope(self, x: torch.Tensor, cs: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
        """apply_rope (model.rs:508-540): rotate-half over the first rotary_dim of each head."""
        rd, half = self.s.rotary_dim, self.s.rotary_dim // 2
        c, s = cs
        x1, x2 = x[..., :half], x[..., half:rd]
        out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
        if rd < x.shape[-1]:
            out = torch.cat([out, x[..., rd:]], dim=-1)
        return out

    def _prefill_ws(self, n: int, total_q: int) -> torch.Tensor | None:
        """Split workspace for mtn_paged_prefill (zeroed once, grown on demand; None when not used)."""
        nb = paged.L.lib().mtn_paged_prefill_workspace_bytes(n, total_q, self.s.hq, self.s.hkv, self.s.head_dim)
        if nb == 0:
            return None
        if self._pws is None or self._pws.numel() < nb:
            self._pws = torch.zeros(nb, dtype=torch.uint8, device=self.dev)
        return self._pws

    def reset_workspaces(self) -> None:
        """Zero every attention workspace (after a launch that gave up on a bounded wait)."""
        for ws in [self._ws] + [g.meta["ws"] for g in self._graphs.values()]:
            if ws is not None:
                ws.reset()
        if self._pws is not None:
            self._pws.zero_()

    def _decode_ws(self, n: int) -> paged.DecodeWorkspace:
        if self._ws is None or n > self._ws_seqs:
            self._ws = paged.DecodeWorkspace.for_shape(self.pool, n, self.s.hq)
            self._ws_seqs = n
        return self._ws

    def _mlp(self, h: torch.Tensor, p: str) -> torch.Tensor:
        g = h @ self.w[f"{p}.mlp.gate_proj.weight"].T
        u = h @ self.w[f"{p}.mlp.up_proj.weight"].T
        act = torch.nn.functional.silu(g) if self.s.mlp == "swiglu" else torch.nn.functional.gelu(g, approximate="tanh")
        return (act * u) @ self.w[f"{p}.mlp.down_proj.weight"].T

    def _attention(self, li: int, h: torch.Tensor, cs: tuple[torch.Tensor, torch.Tensor], meta: dict) -> torch.Tensor:
        """GatedAttention::forward (model.rs:369-422) for every row of the batch."""
        s, w = self.s, self.w
        m = f"layers.{li}.mixer"
        T = h.shape[0]
        qp = h @ w[f"{m}.q_proj.weight"].T
        if s.gated_q:
            qg = qp.view(T, s.hq, 2, s.head_dim)  # per head: q then gate (model.rs:372-375)
            q, gate = qg[:, :, 0, :], qg[:, :, 1, :].reshape(T, s.hq * s.head_dim)
        else:
            q, gate = qp.view(T, s.hq, s.head_dim), None
        k = (h @ w[f"{m}.k_proj.weight"].T).view(T, s.hkv, s.head_dim)
        v = (h @ w[f"{m}.v_proj.weight"].T).view(T, s.hkv, s.head_dim)
        attn = torch.empty((T, s.hq, s.head_dim), dtype=torch.float32, device=self.dev)
        tp = meta["tp"]
        if self.fused:
            # q/k norms, RoPE and every row's K/V store in one launch; the
            # attention kernels then find the step's rows in the pool
            q = torch.empty((T, s.hq, s.head_dim), dtype=torch.float32, device=self.dev)
            qp = qp.contiguous()
            kc, vc = k.contiguous(), v.contiguous()
            qw, kw = (self.w32.get(f"{m}.q_norm.weight"), self.w32.get(f"{m}.k_norm.weight")) if s.qk_norm else (None, None)
            L.check(L.lib().mtn_qkv_prologue(
                paged.C.byref(self.pool.layout), li, qp.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                paged._dtype_code(self.dt), qp.shape[1], s.hkv * s.head_dim, s.hkv * s.head_dim, int(s.gated_q), s.hq,
                None if qw is None else qw.data_ptr(), None if kw is None else kw.data_ptr(), s.eps,
                self.inv_freq.data_ptr(), s.rotary_dim, meta["pos"].data_ptr(), meta["slots_all"].data_ptr(), T,
                q.data_ptr(), paged._stream(None)))
            k_new = v_new = None
        else:
            v = v.float()
            if s.qk_norm:
                q = _rms(q, w[f"{m}.q_norm.weight"], s.eps)
                k = _rms(k, w[f"{m}.k_norm.weight"], s.eps)
            q, k = self._rope(q.float(), cs), self._rope(k.float(), cs)
            if tp:
                self.pool.append(li, k[:tp].contiguous(), v[:tp].contiguous(), meta["slots"])
            k_new, v_new = (k[tp:].contiguous(), v[tp:].contiguous()) if T > tp else (None, None)
        if tp:
            paged.paged_prefill(self.pool, li, q[:tp].contiguous(), meta["qo_p"], meta["kv_p"],
                                meta["kv_indices"], meta["len_p"], meta["max_q"], scale=self.scale, phantom=s.phantom,
                                out=attn[:tp], workspace=meta["pws"], split_bf16=self.split_pre)
        if T > tp:
            paged.paged_decode(self.pool, li, q[tp:].contiguous(), meta["kv_d"], meta["kv_indices"], meta["len_d"],
                               scale=self.scale, phantom=s.phantom, k_new=k_new, v_new=v_new,
                               out=attn[tp:], workspace=meta["ws"], split_bf16=self.split_dec, plan=meta.get("plan"))
        o = attn.view(T, s.hq * s.head_dim).to(self.dt)
        if gate is not None:
            o = torch.sigmoid(gate) * o
        return o @ w[f"{m}.o_proj.weight"].T

    # ------------------------------------------------------------ forward
    def batch_meta(self, b) -> dict:
        """Device copies of the batch's CSR metadata, split into prefill and decode rows."""
        dev = self.dev
        n, npf = b.n_reqs, b.n_prefill
        qo = b.qo_indptr
        tp = int(qo[npf])
        meta = {"tp": tp, "kv_indices": torch.from_numpy(np.ascontiguousarray(b.kv_indices, np.int32)).to(dev),
                "qo_all": torch.from_numpy(np.ascontiguousarray(qo, np.int32)).to(dev),
                "kv_all": torch.from_numpy(np.ascontiguousarray(b.kv_indptr, np.int32)).to(dev)}
        if npf:
            meta["qo_p"] = torch.from_numpy(np.ascontiguousarray(qo[:npf + 1], np.int32)).to(dev)
            meta["kv_p"] = torch.from_numpy(np.ascontiguousarray(b.kv_indptr[:npf + 1], np.int32)).to(dev)
            meta["len_p"] = torch.from_numpy(np.ascontiguousarray(b.seq_lens[:npf], np.int32)).to(dev)
            meta["max_q"] = int(np.max(np.diff(qo[:npf + 1])))
            meta["pws"] = self._prefill_ws(npf, tp)
            pos_p = torch.from_numpy(np.ascontiguousarray(b.position_ids[:tp], np.int32)).to(dev)
            meta["slots"] = paged.build_slot_mapping(meta["qo_p"], pos_p, meta["kv_p"], meta["kv_indices"],
                                                     self.pool.page_size)
        if n > npf:
            meta["kv_d"] = torch.from_numpy(np.ascontiguousarray(b.kv_indptr[npf:], np.int32)).to(dev)
            meta["len_d"] = torch.from_numpy(np.ascontiguousarray(b.seq_lens[npf:], np.int32)).to(dev)
            meta["ws"] = self._decode_ws(n - npf)
            # one host-made work plan serves the decode rows of every layer
            if self.use_plan:
                if self._plan is None:
                    self._plan = paged.DecodePlan(self.s.head_dim, dev)
                meta["plan"] = self._plan.build(b.kv_indptr[npf:], b.seq_lens[npf:], self.pool.page_size,
                                                self.s.hkv)
        return meta

    def _cow(self, b) -> None:
        if len(b.cow_src):
            self.pool.page_copy(torch.from_numpy(np.ascontiguousarray(b.cow_src, np.int32)).to(self.dev),
                                torch.from_numpy(np.ascontiguousarray(b.cow_dst, np.int32)).to(self.dev))

    def _forward_rows(self, ids: torch.Tensor, pos: torch.Tensor, meta: dict, last: torch.Tensor) -> torch.Tensor:
        """The device part of the forward: every launch depends only on tensors, so it can be captured."""
        s, w = self.s, self.w
        x = w["embedding.weight"][ids]  # the vocab-split lookup of model.rs:159-183 is a plain lookup
        if self.fused:
            # every row's pool slot (prefill chunks and decode tokens alike)
            meta = dict(meta, pos=pos, slots_all=paged.build_slot_mapping(meta["qo_all"], pos, meta["kv_all"],
                                                                         meta["kv_indices"], self.pool.page_size))
            cs = None
        else:
            cs = self._rope_tables(pos)
        for li in range(s.layers):
            p = f"layers.{li}"
            x = x + self._attention(li, _rms(x, w[f"{p}.norm.weight"], s.eps), cs, meta)
            x = x + self._mlp(_rms(x, w[f"{p}.ffn_norm.weight"], s.eps), p)
        h = _rms(x[last], w["norm.weight"], s.eps)
        return (h @ w["embedding.weight"].T).float().contiguous()  # tied LM head (model.rs:262-276)

    @torch.no_grad()
    def forward(self, b) -> torch.Tensor:
        """Logits [n_reqs, vocab] (f32, on the device) of each request's last row."""
        self._cow(b)
        meta = self.batch_meta(b)
        ids = torch.from_numpy(b.input_ids.astype(np.int64)).to(self.dev)
        pos = torch.from_numpy(np.ascontiguousarray(b.position_ids, np.int32)).to(self.dev)
        last = torch.from_numpy(b.qo_indptr[1:].astype(np.int64) - 1).to(self.dev)
        return self._forward_rows(ids, pos, meta, last)

    @torch.no_grad()
    def decode_step(self, b) -> torch.Tensor:
        """forward() for a decode-only batch through a CUDA graph per batch size.

        The first batch of a size runs eagerly, then its forward is captured;
        later batches of that size copy their token ids, positions and CSR
        metadata into the graph's static buffers and replay it.  The graph
        holds the paged kernels' launches like any other, so the whole step
        (every layer's projections, norms, RoPE, fused append + decode
        attention, MLP and the LM head) replays without per-launch overhead."""
        if b.n_prefill:
            return self.forward(b)
        self._cow(b)
        n = b.n_reqs
        g = self._graphs.get(n)
        if g is None:
            g = _DecodeGraph(self, n)
            self._graphs[n] = g
        return g.run(b)


class _DecodeGraph:
    """Static buffers and the captured decode forward of one batch size."""

    def __init__(self, model: QwenPagedModel, n: int):
        dev = model.dev
        self.model, self.n = model, n
        self.ids = torch.zeros(n, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(n, dtype=torch.int32, device=dev)
        self.kv_indptr = torch.zeros(n + 1, dtype=torch.int32, device=dev)
        # Page-table entries of the batch: with shared prefix pages a batch
        # lists more entries than the pool has pages, so this grows on demand.
        self.kv_indices = torch.zeros(max(model.pool.num_pages, 1), dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros(n, dtype=torch.int32, device=dev)
        self.last = torch.arange(n, dtype=torch.int64, device=dev)
        self.plan = paged.DecodePlan(model.s.head_dim, dev) if model.use_plan else None
        self.meta = {"tp": 0, "kv_indices": self.kv_indices, "kv_d": self.kv_indptr, "len_d": self.seq_lens,
                     "qo_all": torch.arange(n + 1, dtype=torch.int32, device=dev), "kv_all": self.kv_indptr,
                     "ws": paged.DecodeWorkspace.for_shape(model.pool, n, model.s.hq), "plan": self.plan}
        self.graph = None
        self.out = None

    def _fill(self, b) -> None:
        nk = int(b.kv_indptr[-1])
        if nk > self.kv_indices.numel():
            # A bigger static table: the captured graph holds the old one's
            # address, so it is dropped and captured again on this batch.
            self.kv_indices = torch.zeros(2 * nk, dtype=torch.int32, device=self.model.dev)
            self.meta["kv_indices"] = self.kv_indices
            self.graph = None
            self.out = None
        self.ids.copy_(torch.from_numpy(b.input_ids.astype(np.int64)))
        self.pos.copy_(torch.from_numpy(np.ascontiguousarray(b.position_ids, np.int32)))
        self.kv_indptr.copy_(torch.from_numpy(np.ascontiguousarray(b.kv_indptr, np.int32)))
        self.kv_indices[:nk].copy_(torch.from_numpy(np.ascontiguousarray(b.kv_indices[:nk], np.int32)))
        self.seq_lens.copy_(torch.from_numpy(np.ascontiguousarray(b.seq_lens, np.int32)))
        if self.plan is not None:
            self.plan.build(b.kv_indptr, b.seq_lens, self.model.pool.page_size, self.model.s.hkv)

    def run(self, b) -> torch.Tensor:
        self._fill(b)
        if self.graph is not None:
            self.graph.replay()
            return self.out
        # First batch of this size: run it eagerly on a side stream (its result
        # is this step's), then capture the same launches (capture does not run them).
        m = self.model
        side = torch.cuda.Stream(device=m.dev)
        side.wait_stream(torch.cuda.current_stream(m.dev))
        with torch.cuda.stream(side):
            res = m._forward_rows(self.ids, self.pos, self.meta, self.last)
        torch.cuda.current_stream(m.dev).wait_stream(side)
        torch.cuda.synchronize(m.dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = m._forward_rows(self.ids, self.pos, self.meta, self.last)
        return res


class Engine:
    """engine_loop.rs:28-107 over the scheduler mirror and a paged model.

    Each iteration: schedule a batch, run its copy-on-write page copies and
    the model forward, sample every row on the device with its request's
    temperature (sample_token, scheduler.rs:186-223: greedy first strict max
    or the reference's hash-of-logits pick) and hand the tokens back to the
    scheduler.  A backend error aborts every request of the batch
    (engine_loop.rs:47-57).
    """

    def __init__(self, model: QwenPagedModel, sched, cuda_graphs: bool = True):
        self.model, self.sched = model, sched
        self.cuda_graphs = cuda_graphs
        self.iterations = 0
        self._sample_ws = None

    def step(self) -> bool:
        b = self.sched.schedule()
        if b is None:
            return False
        try:
            logits = self.model.decode_step(b) if self.cuda_graphs else self.model.forward(b)
            if np.any(b.temperatures > 0):
                nb = L.lib().mtn_sample_rows_workspace_bytes(*logits.shape)
                if self._sample_ws is None or self._sample_ws.numel() < nb:
                    self._sample_ws = torch.empty(nb, dtype=torch.uint8, device=logits.device)
                temps = torch.from_numpy(b.temperatures).to(logits.device)
                tokens = paged.sample_rows(logits, temps, workspace=self._sample_ws).cpu().numpy().astype(np.uint32)
            else:
                tokens = paged.argmax_rows(logits).cpu().numpy().astype(np.uint32)
            code, detail = paged.device_error(self.model.dev.index or 0)
            if code:
                timeout = code == paged.DEV_ERR_TIMEOUT
                if timeout:
                    self.model.reset_workspaces()
                raise L.MittenError(L.MTN_ETIMEOUT if timeout else L.MTN_EDEVICE,
                                    f"device error {code} (detail {detail}) in the step's kernels")
        except (L.MittenError, RuntimeError):
            self.sched.abort_batch()
            raise
        self.sched.process_tokens(tokens)
        self.iterations += 1
        return True

    def run(self, max_iterations: int = 1 << 20) -> None:
        while self.sched.num_active() and self.iterations < max_iterations:
            if not self.step():
                break
