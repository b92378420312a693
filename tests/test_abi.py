"""The C-ABI library loads and exports every symbol include/mitten_kv.h declares
(no compute: these run on CPU)."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

from mitten_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "mitten_kv.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^MTN_API [^(]*?\b(mtn_\w+)\(", text, flags=re.M))


def test_header_declares_symbols():
    syms = declared_symbols()
    assert "mtn_paged_decode" in syms and "mtn_kv_append" in syms and "mtn_sched_schedule" in syms
    assert len(syms) >= 40


def test_every_declared_symbol_is_exported():
    lib = _lib.lib()
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, missing


def test_bindings_cover_header():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_only_c_abi_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert declared_symbols() <= exported
    stray = [s for s in exported if not s.startswith("mtn_") and not s.startswith("_")]
    assert not stray, stray[:10]


def test_version_and_error_string():
    lib = _lib.lib()
    assert b"sm_100a" in lib.mtn_version()
    # An invalid call returns MTN_EINVAL and sets the thread's message, launching nothing.
    st = lib.mtn_kv_append(None, 0, None, None, 0, 0, None, 1, None)
    assert st == _lib.MTN_EINVAL
    assert b"null pool" in lib.mtn_last_error()


def test_required_bytes_kat():
    lib = _lib.lib()
    # kv_pool.rs:129-136
    assert lib.mtn_kv_required_bytes(1, 16, 1, 1, 1, 1) == 32
    assert lib.mtn_kv_required_bytes(512, 16, 28, 4, 128, 2) == 2 * 512 * 16 * 28 * 4 * 128 * 2


def test_shared_prefix_decode_argument_checks():
    """mtn_paged_decode_shared_prefix rejects bad arguments with MTN_EINVAL and a
    message before it launches anything (the layout is never dereferenced)."""
    import ctypes as C

    lib = _lib.lib()
    pool = _lib.KvLayout(0x100000, 64, 1, 16, 4, 128)  # aligned fake base
    fake = C.c_void_p(0x200000)  # 16-byte aligned, never dereferenced

    def call(prefix=fake, n_prefix=4, o=fake, o_dtype=_lib.MTN_DTYPE_BF16, flags=0, n_seqs=8, hq=28):
        return lib.mtn_paged_decode_shared_prefix(C.byref(pool), 0, fake, _lib.MTN_DTYPE_BF16, o, o_dtype, None, None,
                                                  _lib.MTN_DTYPE_BF16, n_seqs, hq, prefix, n_prefix, fake, fake, fake,
                                                  0.1, flags, fake, 1 << 20, None)

    cases = [
        (dict(prefix=None), b"at least one page"),
        (dict(n_prefix=0), b"at least one page"),
        (dict(o_dtype=7), b"bad o dtype"),
        (dict(o=C.c_void_p(0x200008)), b"16-byte aligned"),
        (dict(flags=_lib.MTN_ATTN_SPLIT_BF16), b"MTN_ATTN_SPLIT_BF16"),
        (dict(hq=0), b"num_q_heads"),
    ]
    for kw, msg in cases:
        assert call(**kw) == _lib.MTN_EINVAL, kw
        assert msg in lib.mtn_last_error(), (kw, lib.mtn_last_error())
    assert call(n_seqs=0) == _lib.MTN_OK  # nothing to do
