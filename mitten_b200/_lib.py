"""ctypes binding of libmitten_kv.so (the C ABI in include/mitten_kv.h).

The library is built in-tree (``python -m mitten_b200.build``).  Loading
fails loudly when it is missing: there is no Python or CPU fallback for any
device entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmitten_kv.so"

MTN_OK, MTN_EINVAL, MTN_ENOMEM, MTN_ECUDA, MTN_ETIMEOUT, MTN_EDEVICE = range(6)
MTN_DTYPE_BF16, MTN_DTYPE_F32 = 0, 1
MTN_ATTN_PHANTOM_ZERO_SLOT = 1
MTN_ATTN_PREFILL_ONE_TILE = 2
MTN_ATTN_SPLIT_BF16 = 4
MTN_SCHED_REFERENCE, MTN_SCHED_REFCOUNT = 0, 1
MTN_REQ_WAITING, MTN_REQ_PREFILLING, MTN_REQ_DECODING, MTN_REQ_DONE, MTN_REQ_ABORTED = range(5)
MTN_PHASE_PREFILL_ONLY, MTN_PHASE_DECODE_ONLY, MTN_PHASE_MIXED = range(3)

c_i32p = C.POINTER(C.c_int32)
c_i64p = C.POINTER(C.c_int64)
c_u32p = C.POINTER(C.c_uint32)
c_u64p = C.POINTER(C.c_uint64)
c_f32p = C.POINTER(C.c_float)


class KvLayout(C.Structure):
    _fields_ = [
        ("base", C.c_void_p),
        ("num_pages", C.c_int64),
        ("num_layers", C.c_int32),
        ("page_size", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
    ]


class SchedConfig(C.Structure):
    _fields_ = [
        ("num_pages", C.c_int64),
        ("page_size", C.c_int32),
        ("max_prefill_tokens_per_iter", C.c_int32),
        ("max_decode_batch_size", C.c_int32),
        ("radix_max_pages", C.c_int64),
        ("mode", C.c_int32),
        ("n_eos", C.c_int32),
        ("eos_token_ids", c_u32p),
    ]


class BatchView(C.Structure):
    _fields_ = [
        ("phase", C.c_int32),
        ("n_reqs", C.c_int32),
        ("n_prefill", C.c_int32),
        ("n_tokens", C.c_int64),
        ("req_ids", c_u64p),
        ("input_ids", c_u32p),
        ("position_ids", c_i32p),
        ("qo_indptr", c_i32p),
        ("kv_indptr", c_i32p),
        ("kv_indices", c_i32p),
        ("seq_lens", c_i32p),
        ("n_cow", C.c_int64),
        ("cow_src", c_i32p),
        ("cow_dst", c_i32p),
        ("temperatures", c_f32p),
    ]


# name -> (restype, argtypes).  Mirrors include/mitten_kv.h one to one; the
# test suite checks that every declared symbol is exported and listed here.
SIGNATURES: dict[str, tuple] = {
    "mtn_last_error": (C.c_char_p, []),
    "mtn_version": (C.c_char_p, []),
    "mtn_device_error": (C.c_int, [C.c_int, C.c_int, c_i32p, c_i32p]),
    "mtn_selftest_bounded_wait": (C.c_int, [C.c_void_p]),
    "mtn_kv_required_bytes": (C.c_size_t, [C.c_int64] * 6),
    "mtn_kv_pool_alloc": (C.c_int, [C.c_int, C.POINTER(KvLayout)]),
    "mtn_kv_pool_free": (C.c_int, [C.POINTER(KvLayout)]),
    "mtn_kv_page_offset": (C.c_int64, [C.POINTER(KvLayout), C.c_int32, C.c_int32, C.c_int64]),
    "mtn_build_slot_mapping": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int64,
                                         C.c_int32, C.c_void_p, C.c_void_p]),
    "mtn_kv_append": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int64,
                                C.c_void_p, C.c_int64, C.c_void_p]),
    "mtn_page_copy": (C.c_int, [C.POINTER(KvLayout), C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "mtn_kv_gather": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "mtn_paged_decode_workspace_bytes": (C.c_size_t, [C.c_int32] * 4),
    "mtn_paged_decode": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_float, C.c_uint32, C.c_void_p, C.c_size_t,
                                   C.c_void_p]),
    "mtn_paged_decode_plan_bytes": (C.c_size_t, [C.c_int32]),
    "mtn_paged_decode_plan": (C.c_int, [c_i32p, c_i32p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                        C.c_size_t]),
    "mtn_paged_decode_with_plan": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                             C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                             C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_uint32, C.c_void_p,
                                             C.c_void_p, C.c_size_t, C.c_void_p]),
    "mtn_paged_decode_noalloc": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                           C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_uint32, C.c_void_p]),
    "mtn_paged_decode_shared_prefix_workspace_bytes": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "mtn_paged_decode_shared_prefix": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_int32, C.c_void_p,
                                                 C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                                 C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                                 C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p]),
    "mtn_paged_prefill_workspace_bytes": (C.c_size_t, [C.c_int32, C.c_int64, C.c_int32, C.c_int32, C.c_int32]),
    "mtn_paged_prefill": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32,
                                    C.c_int32,
                                    C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_int32, C.c_float, C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p]),
    "mtn_qkv_prologue": (C.c_int, [C.POINTER(KvLayout), C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                   C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                   C.c_float, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                   C.c_void_p]),
    "mtn_kv_pages_bytes": (C.c_size_t, [C.POINTER(KvLayout), C.c_int64]),
    "mtn_kv_pages_pack": (C.c_int, [C.POINTER(KvLayout), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "mtn_kv_pages_unpack": (C.c_int, [C.POINTER(KvLayout), C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "mtn_argmax_rows": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]),
    "mtn_sample_rows_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int64]),
    "mtn_sample_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_size_t,
                                  C.c_void_p]),
    # host mirror: page pool
    "mtn_page_pool_create": (C.c_int, [C.c_int64, C.c_int32, C.POINTER(C.c_void_p)]),
    "mtn_page_pool_destroy": (None, [C.c_void_p]),
    "mtn_page_pool_allocate": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, c_u32p]),
    "mtn_page_pool_free": (C.c_int, [C.c_void_p, C.c_uint32]),
    "mtn_page_pool_free_pages": (C.c_int64, [C.c_void_p]),
    "mtn_page_pool_total_pages": (C.c_int64, [C.c_void_p]),
    "mtn_page_pool_page_size": (C.c_int32, [C.c_void_p]),
    "mtn_page_pool_state": (C.c_int, [C.c_void_p, C.c_uint32, c_i32p, c_u64p, c_u64p]),
    "mtn_page_pool_retain": (C.c_int, [C.c_void_p, C.c_uint32]),
    "mtn_page_pool_release": (C.c_int, [C.c_void_p, C.c_uint32, c_i32p]),
    "mtn_page_pool_refcount": (C.c_int32, [C.c_void_p, C.c_uint32]),
    # host mirror: radix
    "mtn_radix_create": (C.c_int, [C.c_int32, C.c_int64, C.POINTER(C.c_void_p)]),
    "mtn_radix_destroy": (None, [C.c_void_p]),
    "mtn_radix_match_prefix": (C.c_int, [C.c_void_p, c_u32p, C.c_int64, c_i64p, c_u32p, c_i64p, c_u64p, c_i64p]),
    "mtn_radix_insert_prefix": (C.c_int, [C.c_void_p, c_u32p, C.c_int64, c_u32p, C.c_int64, c_u32p, c_i64p]),
    "mtn_radix_unlock_nodes": (C.c_int, [C.c_void_p, c_u64p, C.c_int64]),
    "mtn_radix_evict_pages": (C.c_int, [C.c_void_p, C.c_int64, c_u32p, c_i64p]),
    "mtn_radix_promote": (C.c_int, [C.c_void_p, c_u32p, C.c_int64, C.c_int64, c_u32p, C.c_int64]),
    "mtn_radix_total_cached_pages": (C.c_int64, [C.c_void_p]),
    "mtn_radix_num_nodes": (C.c_int64, [C.c_void_p]),
    # host mirror: scheduler
    "mtn_sched_create": (C.c_int, [C.POINTER(SchedConfig), C.POINTER(C.c_void_p)]),
    "mtn_sched_destroy": (None, [C.c_void_p]),
    "mtn_sched_add_request": (C.c_int, [C.c_void_p, C.c_uint64, c_u32p, C.c_int64, C.c_float, C.c_int32]),
    "mtn_sched_schedule": (C.c_int, [C.c_void_p, C.POINTER(BatchView), c_i32p]),
    "mtn_sched_process_logits": (C.c_int, [C.c_void_p, c_f32p, C.c_int64, C.c_int64]),
    "mtn_sched_process_tokens": (C.c_int, [C.c_void_p, c_u32p, C.c_int64]),
    "mtn_sched_abort_batch": (C.c_int, [C.c_void_p]),
    "mtn_sched_request_info": (C.c_int, [C.c_void_p, C.c_uint64, c_i32p, c_i64p, c_i64p, c_i64p, c_i64p]),
    "mtn_sched_request_pages": (C.c_int, [C.c_void_p, C.c_uint64, c_u32p, c_i64p]),
    "mtn_sched_request_output": (C.c_int, [C.c_void_p, C.c_uint64, c_u32p, c_i64p]),
    "mtn_sched_export": (C.c_int, [C.c_void_p, C.c_uint64, c_u32p, c_i64p, c_i64p, c_u32p, c_i64p]),
    "mtn_sched_import": (C.c_int, [C.c_void_p, C.c_uint64, c_u32p, C.c_int64, c_u32p, C.c_int64, C.c_int64, C.c_float,
                                   C.c_int32, c_u32p, c_i64p]),
    "mtn_sched_fork": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, c_u32p, C.c_int64, C.c_float, C.c_int32]),
    "mtn_sched_page_refcount": (C.c_int32, [C.c_void_p, C.c_uint32]),
    "mtn_sched_tree_pages": (C.c_int, [C.c_void_p, c_u32p, c_i64p]),
    "mtn_sched_free_pages": (C.c_int64, [C.c_void_p]),
    "mtn_sched_cached_pages": (C.c_int64, [C.c_void_p]),
    "mtn_sched_num_active": (C.c_int32, [C.c_void_p]),
}


class MittenError(RuntimeError):
    """A non-zero status from the C ABI; ``code`` is the MTN_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class OutOfKvPages(MittenError):
    """MTN_ENOMEM: EngineError::OutOfKvPages (inference-backend/src/error.rs:7-8)."""


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load libmitten_kv.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m mitten_b200.build` "
                "(there is no CPU fallback for the paged-KV path)")
        handle = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    """Raise the matching exception for a non-zero MTN_* status."""
    if status != MTN_OK:
        msg = (lib().mtn_last_error() or b"").decode(errors="replace")
        if status == MTN_ENOMEM:
            raise OutOfKvPages(status, msg)
        raise MittenError(status, msg)
