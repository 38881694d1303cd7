"""Build libfrag.so (the C-ABI library of CUDA kernels) in-tree for sm_100a.

Usage: ``python -m kernelproblems_b200._build [--force] [--verbose]``.

nvcc cross-compiles without a GPU, so this runs on CPU-only hosts too.  The
shared library lands next to this file, where ``_lib.py`` loads it; objects go
to ``<repo>/_build/``.  The CUDA runtime is linked statically so the library
only needs the driver (``libcuda.so.1``) at the first CUDA call.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_PATH = PKG_DIR / "libfrag.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfrag.so")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files)


def _compile(src: Path, verbose: bool, ptxas_verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if ptxas_verbose:
        print(res.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libfrag.so.  Returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    dep_t = _deps_mtime()
    stale = []
    for s in srcs:
        obj = BUILD_DIR / (s.stem + ".o")
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, dep_t):
            stale.append(s)
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(stale), os.cpu_count() or 1))) as ex:
        list(ex.map(lambda s: _compile(s, verbose, ptxas_verbose), stale))
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if stale or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static",
               # keep the static CUDA runtime private to this library: its
               # calls must not bind to another libcudart already loaded
               "-Xlinker", "-Bsymbolic", "-Xlinker", "--exclude-libs,ALL",
               "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/spill report")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
