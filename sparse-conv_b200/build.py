"""Build recipe for the sm_100a CUDA library behind the ``sparseconv`` package.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only (``-gencode
arch=compute_100a,code=sm_100a``) and links ``sparseconv/lib/libsparseconv_b200.so``
in-tree, with the CUDA runtime linked statically so the library depends only on the
driver. Rebuilds only what changed (object files under ``_build/``).

    python sparse-conv_b200/build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJ_DIR = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "sparseconv", "lib")
LIB_PATH = os.path.join(LIB_DIR, "libsparseconv_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _deps_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    dep_t = _deps_mtime()
    objs = []
    changed = force or not os.path.exists(LIB_PATH)
    flags = NVCC_FLAGS + list(extra_flags or [])
    for src in sources:
        sp = os.path.join(CSRC, src)
        op = os.path.join(OBJ_DIR, src[:-3] + ".o")
        objs.append(op)
        if (not force and os.path.exists(op) and os.path.getmtime(op) >= os.path.getmtime(sp)
                and os.path.getmtime(op) >= dep_t):
            continue
        cmd = [nvcc()] + flags + ["-I", INCLUDE, "-c", sp, "-o", op]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        changed = True
    if changed or any(os.path.getmtime(o) > os.path.getmtime(LIB_PATH) for o in objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-cudart", "static", "-o", tmp] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register/smem usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else None
    print(build(force=args.force or args.ptxas_info, verbose=args.verbose, extra_flags=extra))
    sys.exit(0)
