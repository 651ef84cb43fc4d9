"""Build the sm_100a kernels and the C-ABI into ``shadow_infer_b200/_lib/libshadowkv_b200.so``.

``python -m shadow_infer_b200.build [--force] [--ptxas-verbose]``

The library is compiled in-tree with nvcc only (no torch extension machinery):
every ``csrc/*.cu`` becomes an object with ``-gencode arch=compute_100a,code=sm_100a``
and the objects are linked into one shared library with the static CUDA runtime.
Quantisers must match the reference's IEEE arithmetic, so ``--use_fast_math`` is
never used.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from typing import List

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJ_DIR = os.path.join(REPO, "_build", "obj")
LIB_DIR = os.path.join(PKG, "_lib")
LIB_NAME = "libshadowkv_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build shadow_infer_b200")
    return cand


def _sources() -> List[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers() -> List[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, ptxas_verbose: bool = False, verbose: bool = False) -> str:
    """Compile every kernel source for sm_100a and link the C-ABI library; returns its path."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    headers = _headers()
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for src in _sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(obj, [src] + headers):
            cmd = [nvcc()] + ARCH_FLAGS + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc()] + ARCH_FLAGS + ["-shared", "-o", LIB_PATH] + objs + ["-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, ptxas_verbose=args.ptxas_verbose, verbose=True)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
