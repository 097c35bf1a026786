"""ORACLE -- test infrastructure only.

Compiles the reference's own CUDA kernel-map extension from its sources where they lie
(``src/sparseconv/kernels/cuda/{hash/hash.cu, neighbor_map/neighbor_map.cu, ext.cpp}`` under
the reference checkout, ``$SPCONV_REFERENCE_ROOT``, default ``/root/reference``) into
``oracle/_ref/sparseconv_ref_cuda.so`` with nvcc/g++ directly (the reference's setup.py is not
run). The module exposes the reference's four pybind11 bindings (``ext.cpp:5-10``); GPU tests
call its ``hashmap_build_submanifold_conv_neighbor_map_cuda_naive`` to pin the kernel map of the
oracle and of the new library against the reference itself, and
``tests/golden/make_ref_maps.py`` uses it to write golden map fixtures.

It also stages the reference's unmodified Python package (``src/sparseconv/**/*.py``: the
front end, the ops and the Triton implicit-GEMM kernel ``kernels/triton/implicit_gemm.py``)
under ``oracle/_ref/py/`` next to a two-file stub of ``flex_gemm``, the un-vendored package
that ``implicit_gemm.py:5-6`` imports but never calls. ``oracle/ref_gpu.py`` runs the
reference's own GPU forward from there (its public ``sparse_submanifold_conv3d`` with
``Algorithm.IMPLICIT_GEMM``), so that the reference's B200 time can be measured beside this
library's. ``oracle/_ref/`` is not committed; it travels with the working tree.

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
REF_CHECKOUT = os.environ.get("SPCONV_REFERENCE_ROOT", "/root/reference")
REF_PKG = os.path.join(REF_CHECKOUT, "src", "sparseconv")
REF_ROOT = os.path.join(REF_PKG, "kernels", "cuda")
SOURCES = ["hash/hash.cu", "neighbor_map/neighbor_map.cu", "ext.cpp"]
PY_DIR = os.path.join(OUT_DIR, "py")          # staged reference Python package + flex_gemm stub

# flex_gemm is imported at module level by implicit_gemm.py:5-6 and never called; the stub
# makes the import succeed and fails loudly if anything does call it.
_FLEX_GEMM_STUB = {
    "flex_gemm/__init__.py": '"""Import stub: the reference imports flex_gemm but never calls it."""\n',
    "flex_gemm/ops/__init__.py": "",
    "flex_gemm/ops/spconv.py": (
        "def sparse_submanifold_conv3d(*args, **kwargs):\n"
        "    raise NotImplementedError('flex_gemm is not installed; the reference never calls it')\n"),
}


def available() -> bool:
    return os.path.isdir(REF_ROOT)


def stage_python(force: bool = False) -> str:
    """Copy the reference's Python package (``*.py`` only) and the flex_gemm stub into
    ``oracle/_ref/py``. Returns that directory."""
    import shutil
    marker = os.path.join(PY_DIR, "sparseconv", "__init__.py")
    if os.path.exists(marker) and not force:
        return PY_DIR
    if not os.path.isdir(REF_PKG):
        raise RuntimeError("reference Python package not present; cannot stage oracle/_ref/py")
    dst_pkg = os.path.join(PY_DIR, "sparseconv")
    if os.path.isdir(dst_pkg):
        shutil.rmtree(dst_pkg)
    for dirpath, _dirs, files in os.walk(REF_PKG):
        rel = os.path.relpath(dirpath, REF_PKG)
        for f in files:
            if f.endswith(".py"):
                os.makedirs(os.path.join(dst_pkg, rel), exist_ok=True)
                shutil.copyfile(os.path.join(dirpath, f), os.path.join(dst_pkg, rel, f))
    for rel, text in _FLEX_GEMM_STUB.items():
        path = os.path.join(PY_DIR, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as fh:
            fh.write(text)
    return PY_DIR


def build(force: bool = False, verbose: bool = True) -> str:
    if not available():
        raise RuntimeError("reference sources not present; cannot build oracle/_ref")
    stage_python(force)
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
