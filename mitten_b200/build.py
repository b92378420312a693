"""Build libmitten_kv.so in-tree for sm_100a.

    python -m mitten_b200.build            # incremental
    python -m mitten_b200.build --force    # rebuild everything

CUDA sources go through nvcc with ``-gencode arch=compute_100a,code=sm_100a``;
the host mirror (.cpp) through g++.  Objects land in ``mitten_b200/_build``
and the shared library in ``mitten_b200/lib`` (both git-ignored, both carried
to the GPU box with the tree).  No GPU is needed: nvcc cross-compiles.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmitten_kv.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE),
]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-I", str(INCLUDE)]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmitten_kv.so")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _compile(src: Path, obj: Path, verbose: bool, extra: list[str]) -> str:
    if src.suffix == ".cu":
        cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [os.environ.get("CXX", "g++"), *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False, jobs: int | None = None) -> Path:
    """Compile every source under csrc/ and link libmitten_kv.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    deps = _headers()
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    work = []
    for src in srcs:
        obj = BUILD / (src.name + ".o")
        if force or ptxas_info or _stale(obj, src, deps):
            work.append((src, obj))
    if work:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose, extra): s for s, o in work}
            for f in cf.as_completed(futs):
                msg = f.result()
                if ptxas_info and msg:
                    print(f"== {futs[f].name}\n{msg}")
    objs = [BUILD / (s.name + ".o") for s in srcs]
    if force or work or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
