"""ORACLE -- test infrastructure only: times the reference's OWN GPU forward on a B200.

Runs in a process of its own (``bench.py --impl reference`` starts it), because the reference's
Python package is also called ``sparseconv``. It imports the reference's unmodified package
staged by ``oracle/build_ref.py`` under ``oracle/_ref/py`` (front end, ops, Triton kernel), binds
the reference's CUDA extension compiled from its sources (``oracle/_ref/sparseconv_ref_cuda.so``)
as ``sparseconv.kernels.cuda``, and times on ``cuda:0``, on the seeded synthetic workload of the
same name as the library's benchmark:

* ``step``: the reference's public call ``sparse_submanifold_conv3d(feats, coords, shape, weight,
  None, algorithm=Algorithm.IMPLICIT_GEMM)`` (``ops/submanifold_conv3d.py:208-236``), no cached
  map: ``init_hashmap`` (``ops/utils.py:3-16``) + ``hashmap_build_submanifold_conv_neighbor_map_cuda_naive``
  (``neighbor_map.cu:179-237``) + ``sparse_submanifold_conv_fwd_implicit_gemm``
  (``kernels/triton/implicit_gemm.py:59-86``);
* ``map`` and ``conv``: the same two stages on their own (``_compute_neighbor_cache`` and the
  Triton wrapper on that map).

Each timed step follows a 256 MB write that flushes the L2; times are CUDA events on the launch
stream (median and mean over the steps). A 1,024-row sample of the reference's output is checked
against the float64 oracle so the timed path is known to compute the convolution.

    python oracle/ref_gpu.py --workload indoor --steps 10 --warmup 3

prints one JSON line.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PY_DIR = os.path.join(HERE, "_ref", "py")
SYNTHETIC = os.path.join(ROOT, "sparse-conv_b200", "sparseconv", "synthetic.py")


def _load_synthetic():
    # The library's workload generator, loaded by path under another name: `sparseconv` here
    # is the reference's package.
    spec = importlib.util.spec_from_file_location("spconv_b200_synthetic", SYNTHETIC)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["spconv_b200_synthetic"] = mod
    spec.loader.exec_module(mod)
    return mod


def _reference_package():
    if not os.path.exists(os.path.join(PY_DIR, "sparseconv", "__init__.py")):
        raise RuntimeError("oracle/_ref/py was not staged (run oracle/build_ref.py where the reference is)")
    sys.path.insert(0, PY_DIR)
    sys.path.insert(0, HERE)      # build_ref.py and oracle.py import as top-level modules
    import torch  # noqa: F401  (the extension links against it)
    import build_ref
    if not os.path.exists(build_ref.OUT):
        raise RuntimeError("oracle/_ref/sparseconv_ref_cuda.so was not built")
    ext = build_ref.load()
    import sparseconv.kernels as kernels
    sys.modules["sparseconv.kernels.cuda"] = ext
    kernels.cuda = ext
    from sparseconv.ops import submanifold_conv3d as ops
    from sparseconv.kernels.triton import implicit_gemm
    return ops, implicit_gemm


def _stats(ms):
    ms = sorted(ms)
    return {"median": ms[len(ms) // 2], "mean": sum(ms) / len(ms), "min": ms[0], "n": len(ms)}


def run(workload: str, steps: int, warmup: int, device: int = 0) -> dict:
    import numpy as np
    import torch
    syn = _load_synthetic()
    ops, implicit_gemm = _reference_package()
    import oracle                 # oracle/oracle.py (this directory is on sys.path)
    w = syn.make(workload, seed=0)
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    coords = torch.from_numpy(w.coords).to(dev)
    feats = w.feats.to(dev)
    weight = w.weight.to(dev)
    shape = torch.Size(w.shape)
    Co, Kw, Kh, Kd, Ci = weight.shape
    V = Kw * Kh * Kd
    flush = torch.empty(256 << 18, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return ops.sparse_submanifold_conv3d(feats, coords, shape, weight, None,
                                             algorithm=ops.Algorithm.IMPLICIT_GEMM)

    def map_only():
        return ops.SubMConv3dFunction._compute_neighbor_cache(coords, shape, (Kw, Kh, Kd), tuple(w.dilation))

    t0 = time.time()
    out, cache = step()                          # Triton compiles its kernel here
    torch.cuda.synchronize()
    compile_s = time.time() - t0
    for _ in range(max(warmup - 1, 0)):
        step()
    torch.cuda.synchronize()

    def timed(fn, k):
        ms = []
        for i in range(k):
            flush.fill_(i)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            ms.append(a.elapsed_time(b))
        return ms

    step_ms = timed(step, steps)
    map_ms = timed(map_only, steps)
    nbr = cache.neighbor_map
    w3 = weight.reshape(Co, V, Ci)
    conv_ms = timed(lambda: implicit_gemm.sparse_submanifold_conv_fwd_implicit_gemm(feats, w3, None, nbr), steps)

    # The reference's output on a row sample against the float64 oracle over the oracle's map.
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(w.num_voxels, size=min(1024, w.num_voxels), replace=False))
    nbr_ref = oracle.neighbor_map(w.coords, w.shape, w.kernel_size, w.dilation)
    same_map = bool(np.array_equal(nbr.cpu().numpy().astype(np.uint32), nbr_ref))
    ref = oracle.conv_gather_f64(w.feats.double().numpy(), nbr_ref[rows], w.weight.double().numpy())
    got = out.float().cpu().numpy()[rows]
    err = float(np.abs(got - ref).max())
    s = _stats(step_ms)
    return {
        "workload": w.name, "voxels": int(w.num_voxels), "device": torch.cuda.get_device_name(dev),
        "path": "reference sparse_submanifold_conv3d(..., Algorithm.IMPLICIT_GEMM): its CUDA map "
                "builder (compiled from its sources, sm_100a) + its Triton implicit GEMM",
        "step_ms": s, "map_ms": _stats(map_ms), "conv_ms": _stats(conv_ms),
        "voxels_per_s": w.num_voxels / (s["median"] / 1e3),
        "triton_first_call_s": compile_s,
        "check": {"map_equals_oracle": same_map, "rows_checked": int(rows.size),
                  "max_abs_err_vs_f64": err},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="indoor")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    print(json.dumps(run(a.workload, a.steps, a.warmup, a.device)), flush=True)


if __name__ == "__main__":
    main()
