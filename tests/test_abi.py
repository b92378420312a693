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
