"""Builds and runs gather_bench.cu (nvcc, sm_100a) on GPU 0 and prints gathered rows/s for:
TMA tile::gather4 with 1, 2 or 4 issuing warps (one elected lane, or all lanes), and warp-local
cp.async pipelines with 4 or 8 warps per CTA; rows of 32, 64 and 128 bytes, 2M-row table
(256 MB at 128 B/row, larger than L2), 2M random indices, timed with CUDA events.

    python sparse-conv_b200/microbench/run_gather_bench.py
"""
import ctypes
import os
import subprocess

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libgather_bench.so")


def build():
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    subprocess.check_call([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-o", LIB,
                           os.path.join(HERE, "gather_bench.cu")])


def main():
    if not os.path.exists(LIB):
        build()
    lib = ctypes.CDLL(LIB)
    lib.gb_run.restype = ctypes.c_float
    lib.gb_run.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                           ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    dev = torch.device("cuda", 0)
    M, ntiles = 2 * 1024 * 1024, 16384
    g = torch.Generator(device="cpu").manual_seed(0)
    idx = torch.randint(0, M, (ntiles * 128,), dtype=torch.int32, generator=g).to(dev)
    names = {0: "TMA gather4, elected lane", 1: "TMA gather4, all lanes", 2: "cp.async warp-local"}
    for rb in (32, 64, 128):
        feats = torch.randint(0, 255, (M * rb,), dtype=torch.uint8, device=dev)
        print("row bytes %d" % rb)
        for mode, warps, ctas in [(0, 1, 1), (0, 2, 1), (0, 4, 1), (1, 1, 1), (1, 4, 1),
                                  (2, 4, 2), (2, 8, 1), (2, 8, 2)]:
            if rb == 128 and ctas == 2 and (mode < 2 or warps == 8):
                continue                       # does not fit two CTAs per SM
            ms = lib.gb_run(mode, rb, feats.data_ptr(), M, idx.data_ptr(), ntiles, warps, 148 * ctas)
            torch.cuda.synchronize()
            if lib.gb_err() != 0:
                raise RuntimeError("gather bench error %d" % lib.gb_err())
            rows = ntiles * 128
            print("  %-26s warps %d ctas/SM %d: %7.1f us  %6.0f GB/s" % (
                names[mode], warps, ctas, ms * 1e3, rows * rb / ms / 1e6))


if __name__ == "__main__":
    main()
