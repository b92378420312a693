"""Host page bookkeeping and scheduler, backed by the C++ mirror in libmitten_kv.so.

Names and semantics follow the reference engine so that the reference's own
tests read the same against this module:
  KvCachePool  -> inference-engine/src/kv_pool.rs:4-69
  RadixCache   -> inference-engine/src/radix_cache.rs:37-303
  Scheduler    -> prefill.rs / decode.rs / scheduler.rs (schedule_batch,
                  process_and_transition) producing a CSR Batch.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L


def _u32(a) -> tuple[np.ndarray, C.POINTER(C.c_uint32)]:
    arr = np.ascontiguousarray(np.asarray(a, dtype=np.uint32))
    return arr, arr.ctypes.data_as(C.POINTER(C.c_uint32))


def _owner_halves(owner) -> tuple[int, int]:
    v = int(getattr(owner, "int", owner))  # uuid.UUID or int
    return (v >> 64) & 0xFFFFFFFFFFFFFFFF, v & 0xFFFFFFFFFFFFFFFF


class KvCachePool:
    """KvCachePool (kv_pool.rs:4-69).  `free` of a page not in use raises
    (the reference's debug_assert!); refcounts are an extension."""

    def __init__(self, num_pages: int, page_size: int):
        h = C.c_void_p()
        L.check(L.lib().mtn_page_pool_create(num_pages, page_size, C.byref(h)))
        self._h = h
        self._destroy = L.lib().mtn_page_pool_destroy
        self.num_pages, self.page_size = num_pages, page_size

    def __del__(self):
        # the destroy function is bound at construction: module globals may
        # already be gone when the interpreter shuts down
        if getattr(self, "_h", None) and getattr(self, "_destroy", None):
            self._destroy(self._h)
            self._h = None

    def allocate(self, owner) -> int | None:
        hi, lo = _owner_halves(owner)
        p = C.c_uint32()
        st = L.lib().mtn_page_pool_allocate(self._h, hi, lo, C.byref(p))
        if st == L.MTN_ENOMEM:
            return None
        L.check(st)
        return p.value

    def free(self, page: int) -> None:
        L.check(L.lib().mtn_page_pool_free(self._h, page))

    def free_pages(self) -> int:
        return int(L.lib().mtn_page_pool_free_pages(self._h))

    def total_pages(self) -> int:
        return int(L.lib().mtn_page_pool_total_pages(self._h))

    def state(self, page: int):
        """None if Free, else the owner as an int (PageState::InUse)."""
        iu, hi, lo = C.c_int32(), C.c_uint64(), C.c_uint64()
        L.check(L.lib().mtn_page_pool_state(self._h, page, C.byref(iu), C.byref(hi), C.byref(lo)))
        return (hi.value << 64 | lo.value) if iu.value else None

    def retain(self, page: int) -> None:
        L.check(L.lib().mtn_page_pool_retain(self._h, page))

    def release(self, page: int) -> bool:
        freed = C.c_int32()
        L.check(L.lib().mtn_page_pool_release(self._h, page, C.byref(freed)))
        return bool(freed.value)

    def refcount(self, page: int) -> int:
        return int(L.lib().mtn_page_pool_refcount(self._h, page))

    @staticmethod
    def required_bytes(num_pages, page_size, num_layers, num_kv_heads, head_dim, dtype_bytes) -> int:
        return int(L.lib().mtn_kv_required_bytes(num_pages, page_size, num_layers, num_kv_heads, head_dim,
                                                  dtype_bytes))


class RadixCache:
    """RadixCache (radix_cache.rs:37-303)."""

    def __init__(self, page_size: int, max_pages: int):
        h = C.c_void_p()
        L.check(L.lib().mtn_radix_create(page_size, max_pages, C.byref(h)))
        self._h = h
        self._destroy = L.lib().mtn_radix_destroy
        self.page_size = page_size

    def __del__(self):
        # the destroy function is bound at construction: module globals may
        # already be gone when the interpreter shuts down
        if getattr(self, "_h", None) and getattr(self, "_destroy", None):
            self._destroy(self._h)
            self._h = None

    def match_prefix(self, tokens) -> tuple[int, list[int], list[int]]:
        arr, tp = _u32(tokens)
        cap = max(1, len(arr) // max(1, self.page_size) + 1)
        pages = (C.c_uint32 * cap)()
        nodes = (C.c_uint64 * cap)()
        matched, npg, nnd = C.c_int64(), C.c_int64(cap), C.c_int64(cap)
        L.check(L.lib().mtn_radix_match_prefix(self._h, tp, len(arr), C.byref(matched), pages, C.byref(npg),
                                               nodes, C.byref(nnd)))
        return matched.value, list(pages[:npg.value]), list(nodes[:nnd.value])

    def insert_prefix(self, tokens, pages) -> list[int]:
        """Returns the pages evicted to make room (the reference drops them)."""
        ta, tp = _u32(tokens)
        pa, pp = _u32(pages)
        cap = max(1, self.total_cached_pages() + len(pa))
        ev = (C.c_uint32 * cap)()
        nev = C.c_int64(cap)
        L.check(L.lib().mtn_radix_insert_prefix(self._h, tp, len(ta), pp, len(pa), ev, C.byref(nev)))
        return list(ev[:min(nev.value, cap)])

    def unlock_nodes(self, nodes) -> None:
        arr = np.ascontiguousarray(np.asarray(nodes, dtype=np.uint64))
        L.check(L.lib().mtn_radix_unlock_nodes(self._h, arr.ctypes.data_as(C.POINTER(C.c_uint64)), len(arr)))

    def evict_pages(self, target: int) -> list[int]:
        cap = max(1, self.total_cached_pages())
        out = (C.c_uint32 * cap)()
        n = C.c_int64(cap)
        L.check(L.lib().mtn_radix_evict_pages(self._h, target, out, C.byref(n)))
        return list(out[:n.value])

    def promote_request(self, input_ids, device_len: int, kv_pages) -> None:
        ia, ip = _u32(input_ids)
        pa, pp = _u32(kv_pages)
        L.check(L.lib().mtn_radix_promote(self._h, ip, len(ia), device_len, pp, len(pa)))

    def total_cached_pages(self) -> int:
        return int(L.lib().mtn_radix_total_cached_pages(self._h))

    def num_nodes(self) -> int:
        return int(L.lib().mtn_radix_num_nodes(self._h))


@dataclass
class Batch:
    """A scheduled batch (batch.rs:7-36) in CSR form; numpy copies of the view."""
    phase: int
    req_ids: np.ndarray
    n_prefill: int
    input_ids: np.ndarray
    position_ids: np.ndarray
    qo_indptr: np.ndarray
    kv_indptr: np.ndarray
    kv_indices: np.ndarray
    seq_lens: np.ndarray
    cow_src: np.ndarray
    cow_dst: np.ndarray
    temperatures: np.ndarray  # per row, SamplingParams::temperature

    @property
    def n_reqs(self) -> int:
        return len(self.req_ids)

    def page_table(self) -> list[list[int]]:
        return [self.kv_indices[self.kv_indptr[i]:self.kv_indptr[i + 1]].tolist() for i in range(self.n_reqs)]


def _arr(ptr, n, dtype):
    if n == 0:
        return np.zeros(0, dtype=dtype)
    return np.ctypeslib.as_array(ptr, shape=(n,)).astype(dtype, copy=True)


class Scheduler:
    """EngineContext + schedule_batch / process_and_transition over the C++ mirror."""

    def __init__(self, num_pages: int, page_size: int, max_prefill_tokens_per_iter: int = 512,
                 max_decode_batch_size: int = 8, radix_max_pages: int | None = None,
                 mode: int = L.MTN_SCHED_REFCOUNT, eos_token_ids=(99,)):
        self._eos = np.ascontiguousarray(np.asarray(list(eos_token_ids), dtype=np.uint32))
        cfg = L.SchedConfig(num_pages, page_size, max_prefill_tokens_per_iter, max_decode_batch_size,
                            num_pages if radix_max_pages is None else radix_max_pages, mode, len(self._eos),
                            self._eos.ctypes.data_as(C.POINTER(C.c_uint32)))
        h = C.c_void_p()
        L.check(L.lib().mtn_sched_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self._destroy = L.lib().mtn_sched_destroy
        self.page_size = page_size

    def __del__(self):
        # the destroy function is bound at construction: module globals may
        # already be gone when the interpreter shuts down
        if getattr(self, "_h", None) and getattr(self, "_destroy", None):
            self._destroy(self._h)
            self._h = None

    def add_request(self, req_id: int, input_ids, temperature: float = 0.0, max_new_tokens: int = 512) -> None:
        a, p = _u32(input_ids)
        L.check(L.lib().mtn_sched_add_request(self._h, req_id, p, len(a), temperature, max_new_tokens))

    def schedule(self) -> Batch | None:
        v = L.BatchView()
        has = C.c_int32()
        L.check(L.lib().mtn_sched_schedule(self._h, C.byref(v), C.byref(has)))
        if not has.value:
            return None
        n = v.n_reqs
        nkv = v.kv_indptr[n] if n else 0
        return Batch(v.phase, _arr(v.req_ids, n, np.uint64), v.n_prefill, _arr(v.input_ids, v.n_tokens, np.uint32),
                     _arr(v.position_ids, v.n_tokens, np.int32), _arr(v.qo_indptr, n + 1, np.int32),
                     _arr(v.kv_indptr, n + 1, np.int32), _arr(v.kv_indices, nkv, np.int32),
                     _arr(v.seq_lens, n, np.int32), _arr(v.cow_src, v.n_cow, np.int32),
                     _arr(v.cow_dst, v.n_cow, np.int32), _arr(v.temperatures, n, np.float32))

    def process_logits(self, logits: np.ndarray) -> None:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        L.check(L.lib().mtn_sched_process_logits(self._h, lg.ctypes.data_as(C.POINTER(C.c_float)), lg.shape[0],
                                                 lg.shape[1]))

    def process_tokens(self, tokens) -> None:
        a, p = _u32(tokens)
        L.check(L.lib().mtn_sched_process_tokens(self._h, p, len(a)))

    def abort_batch(self) -> None:
        L.check(L.lib().mtn_sched_abort_batch(self._h))

    def request_info(self, req_id: int) -> dict:
        st, dl, cl, npg, nout = C.c_int32(), C.c_int64(), C.c_int64(), C.c_int64(), C.c_int64()
        L.check(L.lib().mtn_sched_request_info(self._h, req_id, C.byref(st), C.byref(dl), C.byref(cl),
                                               C.byref(npg), C.byref(nout)))
        return {"state": st.value, "device_len": dl.value, "cached_len": cl.value, "n_pages": npg.value,
                "n_output": nout.value}

    def request_pages(self, req_id: int) -> list[int]:
        n = self.request_info(req_id)["n_pages"]
        buf = (C.c_uint32 * max(n, 1))()
        cnt = C.c_int64(max(n, 1))
        L.check(L.lib().mtn_sched_request_pages(self._h, req_id, buf, C.byref(cnt)))
        return list(buf[:cnt.value])

    def request_output(self, req_id: int) -> list[int]:
        n = self.request_info(req_id)["n_output"]
        buf = (C.c_uint32 * max(n, 1))()
        cnt = C.c_int64(max(n, 1))
        L.check(L.lib().mtn_sched_request_output(self._h, req_id, buf, C.byref(cnt)))
        return list(buf[:cnt.value])

    def fork(self, parent_id: int, child_id: int, suffix, temperature: float = 0.0, max_new_tokens: int = 512) -> None:
        """Queue child_id = parent's prompt + suffix, sharing the parent's prompt pages (refcount mode)."""
        a, p = _u32(suffix)
        L.check(L.lib().mtn_sched_fork(self._h, parent_id, child_id, p, len(a), temperature, max_new_tokens))

    def export_request(self, req_id: int) -> dict:
        """Hand a decoding request over (KvHandoff): its pages, device_len and generated tokens."""
        info = self.request_info(req_id)
        npg, nout = max(info["n_pages"], 1), max(info["n_output"], 1)
        pages, outs = (C.c_uint32 * npg)(), (C.c_uint32 * nout)()
        n_p, n_o, dl = C.c_int64(npg), C.c_int64(nout), C.c_int64()
        L.check(L.lib().mtn_sched_export(self._h, req_id, pages, C.byref(n_p), C.byref(dl), outs, C.byref(n_o)))
        return {"pages": list(pages[:n_p.value]), "device_len": dl.value, "outputs": list(outs[:n_o.value])}

    def import_request(self, req_id: int, input_ids, outputs, device_len: int, temperature: float = 0.0,
                       max_new_tokens: int = 512) -> list[int]:
        """Admit a handed-over request as Decoding; returns the pages to unpack its KV into."""
        a, ap = _u32(input_ids)
        o, op = _u32(outputs)
        cap = (device_len + self.page_size - 1) // self.page_size
        pages = (C.c_uint32 * max(cap, 1))()
        n = C.c_int64(max(cap, 1))
        L.check(L.lib().mtn_sched_import(self._h, req_id, ap, len(a), op, len(o), device_len, temperature,
                                         max_new_tokens, pages, C.byref(n)))
        return list(pages[:n.value])

    def page_refcount(self, page: int) -> int:
        return int(L.lib().mtn_sched_page_refcount(self._h, page))

    def tree_pages(self) -> list[int]:
        # the tree lists exactly cached_pages() pages
        cap = max(1, self.cached_pages())
        buf = (C.c_uint32 * cap)()
        cnt = C.c_int64(cap)
        L.check(L.lib().mtn_sched_tree_pages(self._h, buf, C.byref(cnt)))
        return list(buf[:cnt.value])

    def free_pages(self) -> int:
        return int(L.lib().mtn_sched_free_pages(self._h))

    def cached_pages(self) -> int:
        return int(L.lib().mtn_sched_cached_pages(self._h))

    def num_active(self) -> int:
        return int(L.lib().mtn_sched_num_active(self._h))
