"""TEST INFRASTRUCTURE -- CPU oracle for the paged-KV hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this package, and only as the checker (or the timed CPU baseline); the
product path in mitten_b200/ never imports it.

  attention_ref.c  f32 restatement of the reference attention core
                   (inference-model-qwen/src/model.rs:394-416), of the
                   reference's cat-grown CPU decode step (the timed baseline)
                   and of sample_token (scheduler.rs:186-223).
  host_ref.py      pure-Python restatement of kv_pool.rs / radix_cache.rs /
                   prefill.rs / decode.rs / scheduler.rs.
  model_ref.py     numpy f32 restatement of Qwen3_5Model::forward with
                   full-attention layers (model.rs:98-205, 348-422, 508-555).

Parity status: host page-id logic is pinned by the reference's own unit
tests (ported in tests/test_reference_kats.py).  Attention and forward
numerics are "parity unpinned": the reference computes them inside Burn
0.16.1 / ndarray 0.16.1 / matrixmultiply 0.3.10 (not vendored, no Rust
toolchain here) and no reference test pins a value.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB = BUILD / "liboracle.so"
SRC = HERE / "attention_ref.c"

_lib = None


def build(force: bool = False) -> Path:
    """Compile attention_ref.c (gcc, OpenMP) into oracle/_build/liboracle.so."""
    BUILD.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", str(SRC), "-o", str(LIB), "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        f32p, i64p = C.POINTER(C.c_float), C.POINTER(C.c_int64)
        h.ref_attention.argtypes = [f32p, f32p, f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                    C.c_float, f32p]
        h.ref_attention.restype = None
        h.ref_catgrown_step.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), i64p, f32p, f32p, f32p,
                                        C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_float, f32p]
        h.ref_catgrown_step.restype = None
        h.ref_rne_bf16.argtypes = [f32p, C.c_int64, C.POINTER(C.c_uint16)]
        h.ref_rne_bf16.restype = None
        h.ref_sample_token.argtypes = [f32p, C.c_int64, C.c_float, f32p]
        h.ref_sample_token.restype = C.c_int64
        h.ref_num_threads.argtypes = []
        h.ref_num_threads.restype = C.c_int
        _lib = h
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def attention(q, kc, vc, scale: float) -> np.ndarray:
    """model.rs:394-416 over a contiguous cache.

    q [S, Hq, D]; kc, vc [Hkv, T, D] (row 0 is the phantom zero row when the
    caller models Qwen3_5Model::init_cache).  Returns [S, Hq, D] f32.
    """
    q, qp = _f32(q)
    kc, kp = _f32(kc)
    vc, vp = _f32(vc)
    S, Hq, D = q.shape
    Hkv, T, _ = kc.shape
    out = np.empty((S, Hq, D), dtype=np.float32)
    lib().ref_attention(qp, kp, vp, T, S, Hq, Hkv, D, scale, out.ctypes.data_as(C.POINTER(C.c_float)))
    return out


def rne_bf16_bits(x) -> np.ndarray:
    """IEEE f32 -> bf16 round-to-nearest-even, returned as uint16 bit patterns."""
    x, xp = _f32(x)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ref_rne_bf16(xp, x.size, out.ctypes.data_as(C.POINTER(C.c_uint16)))
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def sample_token(row, temperature: float) -> int:
    """sample_token (scheduler.rs:186-223) of one logits row, in C with libm expf (ref_sample_token)."""
    r, rp = _f32(np.asarray(row).reshape(-1))
    scratch = np.empty(max(r.size, 1), np.float32)
    return int(lib().ref_sample_token(rp, r.size, float(temperature), scratch.ctypes.data_as(C.POINTER(C.c_float))))


def round_bf16(x) -> np.ndarray:
    """f32 values rounded to bf16 and widened back to f32."""
    return bf16_bits_to_f32(rne_bf16_bits(x))


class CatGrownDecode:
    """The reference CPU decode step (cat-grown caches), timed as the CPU baseline.

    Holds one contiguous [Hkv, T, D] f32 K and V cache per request, each
    starting with the phantom zero row plus `lens[r]` prior rows.
    """

    def __init__(self, k_prior, v_prior, Hq: int, scale: float):
        self.n = len(k_prior)
        self.Hkv, _, self.D = k_prior[0].shape
        self.Hq = Hq
        self.scale = scale
        libc = C.CDLL("libc.so.6")
        libc.malloc.restype = C.c_void_p
        libc.malloc.argtypes = [C.c_size_t]
        self._libc = libc
        self.kptr = (C.c_void_p * self.n)()
        self.vptr = (C.c_void_p * self.n)()
        self.lens = np.zeros(self.n, dtype=np.int64)
        for r in range(self.n):
            for src, dst in ((k_prior[r], self.kptr), (v_prior[r], self.vptr)):
                a = np.ascontiguousarray(src, dtype=np.float32)
                p = libc.malloc(a.nbytes)
                C.memmove(p, a.ctypes.data, a.nbytes)
                dst[r] = p
            self.lens[r] = k_prior[r].shape[1]

    def step(self, q, knew, vnew) -> np.ndarray:
        q, qp = _f32(q)
        knew, kp = _f32(knew)
        vnew, vp = _f32(vnew)
        out = np.empty((self.n, self.Hq, self.D), dtype=np.float32)
        lib().ref_catgrown_step(self.kptr, self.vptr, self.lens.ctypes.data_as(C.POINTER(C.c_int64)), kp, vp, qp,
                                self.n, self.Hq, self.Hkv, self.D, self.scale,
                                out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def close(self):
        libc = C.CDLL("libc.so.6")
        libc.free.argtypes = [C.c_void_p]
        for arr in (self.kptr, self.vptr):
            for r in range(self.n):
                if arr[r]:
                    libc.free(arr[r])
                    arr[r] = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def num_threads() -> int:
    return int(lib().ref_num_threads())
