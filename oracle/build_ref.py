"""ORACLE -- test infrastructure only.

Compiles the reference's own CUDA kernel-map extension from its sources where they lie
(``/root/reference/src/sparseconv/kernels/cuda/{hash/hash.cu, neighbor_map/neighbor_map.cu,
ext.cpp}``) into ``oracle/_ref/sparseconv_ref_cuda.so`` with nvcc/g++ directly (the
reference's setup.py is not run). The module exposes the reference's four pybind11
bindings (``ext.cpp:5-10``); GPU tests call its
``hashmap_build_submanifold_conv_neighbor_map_cuda_naive`` to pin the kernel map of the
oracle and of the new library against the reference itself, and
``tests/golden/make_ref_maps.py`` uses it to write golden map fixtures.

Flags follow the reference's build (``setup.py:22,28-31``: ``-O3 -std=c++17
--use_fast_math``) with the architecture fixed to sm_100a. The sources are only read.

    python oracle/build_ref.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OBJ_DIR = os.path.join(OUT_DIR, "obj")
MODULE = "sparseconv_ref_cuda"
OUT = os.path.join(OUT_DIR, MODULE + ".so")
REF_ROOT = "/root/reference/src/sparseconv/kernels/cuda"
SOURCES = ["hash/hash.cu", "neighbor_map/neighbor_map.cu", "ext.cpp"]


def available() -> bool:
    return os.path.isdir(REF_ROOT)


def build(force: bool = False, verbose: bool = True) -> str:
    if not available():
        raise RuntimeError("reference sources not present; cannot build oracle/_ref")
    if os.path.exists(OUT) and not force:
        return OUT
    import torch
    from torch.utils import cpp_extension as ce
    os.makedirs(OBJ_DIR, exist_ok=True)
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    inc_flags = [f"-I{p}" for p in incs]
    abi = "1" if torch.compiled_with_cxx11_abi() else "0"
    defs = ["-DTORCH_API_INCLUDE_EXTENSION_H", f"-DTORCH_EXTENSION_NAME={MODULE}",
            "-DPYBIND11_COMPILER_TYPE=\"_gcc\"", "-DPYBIND11_STDLIB=\"_libstdcpp\"",
            "-DPYBIND11_BUILD_ABI=\"_cxxabi1018\"", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    objs = []
    for rel in SOURCES:
        src = os.path.join(REF_ROOT, rel)
        obj = os.path.join(OBJ_DIR, os.path.basename(rel) + ".o")
        objs.append(obj)
        if rel.endswith(".cu"):
            cmd = ["/usr/local/cuda/bin/nvcc", "-c", src, "-o", obj, "-O3", "-std=c++17",
                   "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a",
                   "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                   "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                   "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__"] + inc_flags + defs
        else:
            cmd = ["g++", "-c", src, "-o", obj, "-O3", "-std=c++17", "-fPIC"] + inc_flags + defs
        if verbose:
            print("[build_ref]", os.path.basename(src), flush=True)
        subprocess.check_call(cmd)
    libdirs = ce.library_paths(device_type="cuda")
    link = ["g++", "-shared", "-o", OUT + ".tmp"] + objs + [f"-L{p}" for p in libdirs] + [
        "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
        "-lcudart"]
    subprocess.check_call(link)
    os.replace(OUT + ".tmp", OUT)
    return OUT


def load():
    """Import the built reference extension module (needs torch imported first)."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (provides the symbols the module links against)
    loader = importlib.machinery.ExtensionFileLoader(MODULE, OUT)
    spec = importlib.util.spec_from_file_location(MODULE, OUT, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
