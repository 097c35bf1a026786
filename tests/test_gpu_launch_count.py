"""The benchmark's `gpu_launches` figure against the kernels this library really launches.

`bench.py` reports how many of the library's kernels one forward (map build without cache +
conv) launches, from `_launches_per_step`. Here the torch profiler records one forward through
the public API and the kernels of the library's `spconv` namespace are counted: the bucket
order (cube: prep, clear, insert, map, order, conv) and the radix order (one indoor sample of
250 k voxels on a sparse grid: prep, clear, insert, map, then a scan and a scatter per 8-bit
pass and a count for the second and third passes, conv).
"""
import importlib.util
import os

import pytest
import torch

from sparseconv import synthetic
from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _library_kernels(w):
    dev = torch.device("cuda", 0)
    coords = torch.from_numpy(w.coords).to(dev)
    feats, weight = w.feats.to(dev), w.weight.to(dev)
    shape = torch.Size(w.shape)
    sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)  # warm-up
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    return [n for n in names if "spconv::" in n]


@pytest.mark.parametrize("case", ["cube", "indoor_one_sample"])
def test_gpu_launches_claim_matches_profile(case):
    w = synthetic.cube(seed=0) if case == "cube" else synthetic.indoor(seed=0, batch=1)
    kernels = _library_kernels(w)
    claimed = _bench()._launches_per_step(w.num_voxels, w.kernel_size, w.shape)
    assert len(kernels) == claimed, kernels
    assert any("conv_tc_kernel" in n for n in kernels) and any("map_kernel" in n for n in kernels)
    if case == "indoor_one_sample":
        assert sum("sort_scatter_kernel" in n for n in kernels) == 3
