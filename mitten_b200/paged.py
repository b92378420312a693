"""Device side of the paged-KV path, over torch CUDA tensors.

Thin wrappers over the C ABI (include/mitten_kv.h): torch supplies device
memory and the current stream; every computation runs in libmitten_kv.so.
There is no fallback: a missing library or a CPU tensor raises.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import _lib as L


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor (the paged-KV path has no CPU implementation)")
    return t.data_ptr()


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise ValueError(f"expected a contiguous int32 tensor, got {t.dtype}")
    return t


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return L.MTN_DTYPE_BF16
    if dt == torch.float32:
        return L.MTN_DTYPE_F32
    raise ValueError(f"unsupported dtype {dt}")


class PagedKVPool:
    """The device KV pool: bf16 [layers][2][pages][kv_heads][page_size][head_dim].

    Each (page, kv head) slab is a [page_size, head_dim] slice of the
    reference's per-request KVCacheState::Attention [1, heads, seq, head_dim]
    (inference-model-common/src/lib.rs:5-13).
    """

    def __init__(self, num_layers: int, num_pages: int, page_size: int, num_kv_heads: int, head_dim: int,
                 device: torch.device | str | int = "cuda"):
        self.num_layers, self.num_pages, self.page_size = num_layers, num_pages, page_size
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.device = torch.device(device)
        self.storage = torch.zeros((num_layers, 2, num_pages, num_kv_heads, page_size, head_dim),
                                   dtype=torch.bfloat16, device=self.device)
        self.layout = L.KvLayout(self.storage.data_ptr(), num_pages, num_layers, page_size, num_kv_heads, head_dim)

    @staticmethod
    def required_bytes(num_pages, page_size, num_layers, num_kv_heads, head_dim, dtype_bytes=2) -> int:
        """KvCachePool::required_bytes (kv_pool.rs:58-68)."""
        return int(L.lib().mtn_kv_required_bytes(num_pages, page_size, num_layers, num_kv_heads, head_dim,
                                                  dtype_bytes))

    def k_pages(self, layer: int) -> torch.Tensor:
        return self.storage[layer, 0]

    def v_pages(self, layer: int) -> torch.Tensor:
        return self.storage[layer, 1]

    # -- kernels ---------------------------------------------------------
    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor, stream=None) -> None:
        """Scatter k/v [n_tokens, kv_heads, head_dim] (or row-strided 2-D views) to `slots`."""
        if slots.dtype != torch.int64:
            raise ValueError("slots must be int64")
        n = slots.numel()
        k2 = k.reshape(n, -1) if k.dim() != 2 else k
        v2 = v.reshape(n, -1) if v.dim() != 2 else v
        if k2.stride(1) != 1 or v2.stride(1) != 1 or k2.stride(0) != v2.stride(0):
            raise ValueError("k/v rows must be unit-stride with a common row stride")
        if k2.dtype != v2.dtype:
            raise ValueError("k and v dtypes differ")
        L.check(L.lib().mtn_kv_append(C.byref(self.layout), layer, _ptr(k2), _ptr(v2), _dtype_code(k2.dtype),
                                      k2.stride(0), _ptr(slots), n, _stream(stream)))

    def page_copy(self, src: torch.Tensor, dst: torch.Tensor, stream=None) -> None:
        """Copy page src[i] onto dst[i] in every layer (copy-on-write / fork)."""
        L.check(L.lib().mtn_page_copy(C.byref(self.layout), _ptr(_i32(src)), _ptr(_i32(dst)), src.numel(),
                                      _stream(stream)))

    def gather(self, layer: int, kv_indptr: torch.Tensor, kv_indices: torch.Tensor, seq_lens: torch.Tensor,
               stream=None) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
        """Contiguous per-sequence [kv_heads, seq_len, head_dim] bf16 copies (KVCacheState layout)."""
        lens = seq_lens.to("cpu").tolist()
        offs = [0]
        for x in lens:
            offs.append(offs[-1] + x)
        total = offs[-1]
        ok = torch.empty((max(total, 1) * self.num_kv_heads * self.head_dim,), dtype=torch.bfloat16,
                         device=self.device)
        ov = torch.empty_like(ok)
        off_t = torch.tensor(offs[:-1] or [0], dtype=torch.int64, device=self.device)
        L.check(L.lib().mtn_kv_gather(C.byref(self.layout), layer, _ptr(_i32(kv_indptr)), _ptr(_i32(kv_indices)),
                                      _ptr(_i32(seq_lens)), _ptr(off_t), len(lens), _ptr(ok), _ptr(ov), total,
                                      _stream(stream)))
        ks, vs = [], []
        hd = self.num_kv_heads * self.head_dim
        for r, n in enumerate(lens):
            ks.append(ok[offs[r] * hd:(offs[r] + n) * hd].view(self.num_kv_heads, n, self.head_dim))
            vs.append(ov[offs[r] * hd:(offs[r] + n) * hd].view(self.num_kv_heads, n, self.head_dim))
        return ks, vs


def build_slot_mapping(qo_indptr, positions, kv_indptr, kv_indices, page_size: int, stream=None) -> torch.Tensor:
    """Per-token pool slots for a CSR batch (device kernel)."""
    n_tok = positions.numel()
    slots = torch.empty(n_tok, dtype=torch.int64, device=positions.device)
    L.check(L.lib().mtn_build_slot_mapping(_ptr(_i32(qo_indptr)), _ptr(_i32(positions)), _ptr(_i32(kv_indptr)),
                                           _ptr(_i32(kv_indices)), qo_indptr.numel() - 1, n_tok, page_size,
                                           _ptr(slots), _stream(stream)))
    return slots


class DecodeWorkspace:
    """Partials + arrival counters for mtn_paged_decode (zeroed once, reusable).

    A launch that gives up on a bounded wait (device error code 4) can leave
    arrival counters non-zero: call reset() before the next launch."""

    def __init__(self, nbytes: int, device):
        self.nbytes = max(int(nbytes), 256)
        self.buf = torch.zeros(self.nbytes, dtype=torch.uint8, device=device)

    def reset(self) -> None:
        self.buf.zero_()

    @classmethod
    def for_shape(cls, pool: PagedKVPool, n_seqs: int, num_q_heads: int):
        nb = L.lib().mtn_paged_decode_workspace_bytes(n_seqs, num_q_heads, pool.num_kv_heads, pool.head_dim)
        return cls(nb, pool.device)


class DecodePlan:
    """Host-made work plan for paged_decode (mtn_paged_decode_plan): each CTA's tile range and start,
    balanced by cost, from host copies of the batch's kv_indptr and seq_lens.  build() fills the pinned
    host copy and queues its upload on `stream`; one plan serves every layer of a step."""

    def __init__(self, head_dim: int, device):
        self.head_dim = head_dim
        self.nbytes = int(L.lib().mtn_paged_decode_plan_bytes(head_dim))
        if self.nbytes == 0:
            raise ValueError(f"head_dim {head_dim} has no decode plan")
        self.host = torch.empty(self.nbytes, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(self.nbytes, dtype=torch.uint8, device=device)

    def build(self, kv_indptr, seq_lens, page_size: int, num_kv_heads: int, stream=None) -> "DecodePlan":
        ip = np.ascontiguousarray(np.asarray(kv_indptr), dtype=np.int32)
        ln = np.ascontiguousarray(np.asarray(seq_lens), dtype=np.int32)
        if ip.size != ln.size + 1:
            raise ValueError("kv_indptr must have n_seqs + 1 entries")
        i32 = C.POINTER(C.c_int32)
        L.check(L.lib().mtn_paged_decode_plan(ip.ctypes.data_as(i32), ln.ctypes.data_as(i32), ln.size, page_size,
                                              num_kv_heads, self.head_dim, self.host.data_ptr(), self.nbytes))
        s = stream if stream is not None else torch.cuda.current_stream(self.dev.device)
        with torch.cuda.stream(s):
            self.dev.copy_(self.host, non_blocking=True)
        return self

    def words(self) -> np.ndarray:
        """The host copy as int32 words (for tests)."""
        return self.host.numpy().view(np.int32).copy()


def paged_decode(pool: PagedKVPool, layer: int, q: torch.Tensor, kv_indptr: torch.Tensor,
                 kv_indices: torch.Tensor, seq_lens: torch.Tensor, scale: float | None = None,
                 phantom: bool = False, k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
                 workspace: DecodeWorkspace | None = None, stream=None, split_bf16: bool = False,
                 plan: DecodePlan | None = None) -> torch.Tensor:
    """Decode attention for q [n_seqs, num_q_heads, head_dim] over the paged cache.

    With k_new/v_new [n_seqs, kv_heads, head_dim] the step's token is first
    stored at position seq_lens[r]-1 of each sequence (fused KV append).
    `split_bf16` passes Q and P to the tensor cores as bf16 hi + lo pairs
    (MTN_ATTN_SPLIT_BF16): f32-level products at no extra tensor-core work.
    `plan` (DecodePlan built for these kv_indptr / seq_lens) replaces the
    kernel's own scan and even split of the tiles.
    """
    if q.dim() != 3 or not q.is_contiguous():
        raise ValueError("q must be a contiguous [n_seqs, heads, head_dim] tensor")
    n, hq, d = q.shape
    if d != pool.head_dim:
        raise ValueError("head_dim mismatch")
    if scale is None:
        scale = d ** -0.5
    if out is None:
        out = torch.empty((n, hq, d), dtype=out_dtype, device=q.device)
    if workspace is None:
        workspace = DecodeWorkspace.for_shape(pool, n, hq)
    new_code = 0
    if k_new is not None or v_new is not None:
        if k_new is None or v_new is None or not k_new.is_contiguous() or not v_new.is_contiguous():
            raise ValueError("k_new and v_new must both be contiguous [n_seqs, kv_heads, head_dim] tensors")
        if k_new.dtype != v_new.dtype or k_new.numel() != n * pool.num_kv_heads * d:
            raise ValueError("k_new/v_new shape or dtype mismatch")
        new_code = _dtype_code(k_new.dtype)
    flags = (L.MTN_ATTN_PHANTOM_ZERO_SLOT if phantom else 0) | (L.MTN_ATTN_SPLIT_BF16 if split_bf16 else 0)
    L.check(L.lib().mtn_paged_decode_with_plan(C.byref(pool.layout), layer, _ptr(q), _dtype_code(q.dtype),
                                               _ptr(out), _dtype_code(out.dtype), _ptr(k_new), _ptr(v_new), new_code,
                                               n, hq, _ptr(_i32(kv_indptr)), _ptr(_i32(kv_indices)),
                                               _ptr(_i32(seq_lens)), float(scale), flags,
                                               None if plan is None else plan.dev.data_ptr(), _ptr(workspace.buf),
                                               workspace.nbytes, _stream(stream)))
    return out


def shared_prefix_workspace(pool: PagedKVPool, n_seqs: int, num_q_heads: int) -> torch.Tensor:
    """Zeroed workspace for paged_decode_shared_prefix (reusable; zero it again after a device timeout)."""
    nb = L.lib().mtn_paged_decode_shared_prefix_workspace_bytes(n_seqs, num_q_heads, pool.num_kv_heads,
                                                                 pool.head_dim)
    if nb == 0:
        raise ValueError("no shared-prefix decode for this shape")
    return torch.zeros(nb, dtype=torch.uint8, device=pool.device)


def paged_decode_shared_prefix(pool: PagedKVPool, layer: int, q: torch.Tensor, prefix_pages: torch.Tensor,
                               kv_indptr: torch.Tensor, kv_indices: torch.Tensor, seq_lens: torch.Tensor,
                               scale: float | None = None, phantom: bool = False, k_new: torch.Tensor | None = None,
                               v_new: torch.Tensor | None = None, out: torch.Tensor | None = None,
                               out_dtype: torch.dtype = torch.bfloat16, workspace: torch.Tensor | None = None,
                               stream=None, split_bf16: bool = False) -> torch.Tensor:
    """paged_decode for sequences that all start with the same full pages `prefix_pages`.

    Sequence r attends over the prefix pages followed by its own pages
    kv_indices[kv_indptr[r]:kv_indptr[r+1]] holding seq_lens[r] tokens (the
    step's token, with k_new/v_new, at own position seq_lens[r] - 1); the
    prefix is read once for the whole batch instead of once per sequence.
    """
    if q.dim() != 3 or not q.is_contiguous():
        raise ValueError("q must be a contiguous [n_seqs, heads, head_dim] tensor")
    n, hq, d = q.shape
    if d != pool.head_dim:
        raise ValueError("head_dim mismatch")
    if scale is None:
        scale = d ** -0.5
    if out is None:
        out = torch.empty((n, hq, d), dtype=out_dtype, device=q.device)
    if workspace is None:
        workspace = shared_prefix_workspace(pool, n, hq)
    new_code = 0
    if k_new is not None or v_new is not None:
        if k_new is None or v_new is None or not k_new.is_contiguous() or not v_new.is_contiguous():
            raise ValueError("k_new and v_new must both be contiguous [n_seqs, kv_heads, head_dim] tensors")
        new_code = _dtype_code(k_new.dtype)
    pp = _i32(prefix_pages)
    flags = (L.MTN_ATTN_PHANTOM_ZERO_SLOT if phantom else 0) | (L.MTN_ATTN_SPLIT_BF16 if split_bf16 else 0)
    L.check(L.lib().mtn_paged_decode_shared_prefix(C.byref(pool.layout), layer, _ptr(q), _dtype_code(q.dtype),
                                                   _ptr(out), _dtype_code(out.dtype), _ptr(k_new), _ptr(v_new),
                                                   new_code, n, hq, _ptr(pp), pp.numel(), _ptr(_i32(kv_indptr)),
                                                   _ptr(_i32(kv_indices)), _ptr(_i32(seq_lens)), float(scale), flags,
                                                   _ptr(workspace), workspace.numel(), _stream(stream)))
    return out


def paged_prefill(pool: PagedKVPool, layer: int, q: torch.Tensor, qo_indptr: torch.Tensor,
                  kv_indptr: torch.Tensor, kv_indices: torch.Tensor, seq_lens: torch.Tensor, max_q_len: int,
                  scale: float | None = None, phantom: bool = False, out: torch.Tensor | None = None,
                  out_dtype: torch.dtype = torch.bfloat16, workspace: torch.Tensor | None = None,
                  stream=None, one_tile: bool = False, split_bf16: bool = False) -> torch.Tensor:
    """Chunked-prefill attention for q [total_q, num_q_heads, head_dim] (bf16 or f32) over the paged cache.

    f32 queries are rounded to bf16 as they are loaded; `split_bf16`
    (MTN_ATTN_SPLIT_BF16, head_dim <= 128) instead passes Q and P to the
    tensor cores as bf16 hi + lo pairs, twice the tensor-core work.

    Launches with few (query tile, head) units cut long ones into pieces over
    more CTAs; that needs `workspace` (mtn_paged_prefill_workspace_bytes,
    zeroed once, reusable, one stream at a time; zero it again after a call
    that reported a device timeout).  A fresh zeroed one is made
    when none is given; a smaller one runs the launch unsplit.  Launches with
    many query tiles at head_dim <= 128 run two query tiles per CTA;
    `one_tile` forces the one-tile kernel (same results).
    """
    if q.dim() != 3 or not q.is_contiguous() or q.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("q must be a contiguous bf16 or f32 [total_q, heads, head_dim] tensor")
    tq, hq, d = q.shape
    if scale is None:
        scale = d ** -0.5
    if out is None:
        out = torch.empty((tq, hq, d), dtype=out_dtype, device=q.device)
    n = qo_indptr.numel() - 1
    nb = L.lib().mtn_paged_prefill_workspace_bytes(n, tq, hq, pool.num_kv_heads, d)
    if workspace is None and nb > 0:
        workspace = torch.zeros(nb, dtype=torch.uint8, device=q.device)
    flags = (L.MTN_ATTN_PHANTOM_ZERO_SLOT if phantom else 0) | (L.MTN_ATTN_PREFILL_ONE_TILE if one_tile else 0) \
        | (L.MTN_ATTN_SPLIT_BF16 if split_bf16 else 0)
    L.check(L.lib().mtn_paged_prefill(C.byref(pool.layout), layer, _ptr(q), _dtype_code(q.dtype), _ptr(out),
                                      _dtype_code(out.dtype), n,
                                      tq, hq, _ptr(_i32(qo_indptr)), _ptr(_i32(kv_indptr)), _ptr(_i32(kv_indices)),
                                      _ptr(_i32(seq_lens)), max_q_len, float(scale), flags, _ptr(workspace),
                                      0 if workspace is None else workspace.numel(), _stream(stream)))
    return out


def pack_pages(pool: PagedKVPool, pages: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Pages (every layer, K and V) into a flat [n_pages, layers, 2, kv_heads, page_size, head_dim] bf16
    buffer (mtn_kv_pages_pack): device memory, or pinned host memory for offload."""
    n = pages.numel()
    shape = (n, pool.num_layers, 2, pool.num_kv_heads, pool.page_size, pool.head_dim)
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=pool.device)
    if out.numel() * 2 < L.lib().mtn_kv_pages_bytes(C.byref(pool.layout), n) or not out.is_contiguous():
        raise ValueError("out must be a contiguous buffer of mtn_kv_pages_bytes bytes")
    L.check(L.lib().mtn_kv_pages_pack(C.byref(pool.layout), _ptr(_i32(pages)), n, out.data_ptr(), _stream(stream)))
    return out


def unpack_pages(pool: PagedKVPool, src: torch.Tensor, pages: torch.Tensor, stream=None) -> None:
    """The reverse of pack_pages: src's pages into the listed pool pages (mtn_kv_pages_unpack)."""
    n = pages.numel()
    if src.numel() * src.element_size() < L.lib().mtn_kv_pages_bytes(C.byref(pool.layout), n) or not src.is_contiguous():
        raise ValueError("src must be a contiguous buffer of mtn_kv_pages_bytes bytes")
    L.check(L.lib().mtn_kv_pages_unpack(C.byref(pool.layout), src.data_ptr(), _ptr(_i32(pages)), n, _stream(stream)))


def argmax_rows(logits: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Greedy sample_token (scheduler.rs:186-199) on the device: first strict max per row."""
    if logits.dtype != torch.float32 or not logits.is_contiguous() or logits.dim() != 2:
        raise ValueError("logits must be a contiguous f32 [rows, vocab] tensor")
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    L.check(L.lib().mtn_argmax_rows(_ptr(logits), logits.shape[0], logits.shape[1], _ptr(out), _stream(stream)))
    return out


def sample_rows(logits: torch.Tensor, temperatures: torch.Tensor, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """sample_token (scheduler.rs:186-223) on the device: greedy rows (temperature <= 0) take the
    first strict max, the others the reference's hash-of-logits pick, bit-exact with its f32 order."""
    if logits.dtype != torch.float32 or not logits.is_contiguous() or logits.dim() != 2:
        raise ValueError("logits must be a contiguous f32 [rows, vocab] tensor")
    n, vocab = logits.shape
    t = temperatures.to(device=logits.device, dtype=torch.float32).contiguous()
    if t.numel() != n:
        raise ValueError("one temperature per row")
    if out is None:
        out = torch.empty(n, dtype=torch.int32, device=logits.device)
    nb = L.lib().mtn_sample_rows_workspace_bytes(n, vocab)
    if workspace is None or workspace.numel() < nb:
        workspace = torch.empty(max(nb, 4), dtype=torch.uint8, device=logits.device)
    L.check(L.lib().mtn_sample_rows(_ptr(logits), _ptr(t), n, vocab, _ptr(out), _ptr(workspace), workspace.numel(),
                                    _stream(stream)))
    return out


DEV_ERR_TIMEOUT = 4  # a bounded device wait ran out


def device_error(device: int = 0, clear: bool = True) -> tuple[int, int]:
    """(code, detail) of the first metadata error a kernel recorded; (0, 0) if none.
    After DEV_ERR_TIMEOUT, reset() every DecodeWorkspace (and zero every prefill split
    workspace) the failed launches used."""
    code, detail = C.c_int32(0), C.c_int32(0)
    L.check(L.lib().mtn_device_error(device, int(clear), C.byref(code), C.byref(detail)))
    return code.value, detail.value


def log2e() -> float:
    return 1.0 / math.log(2.0)
