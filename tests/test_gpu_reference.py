"""The reference's own CUDA map builder (compiled from its sources by oracle/build_ref.py)
against the library and the oracle, on identical seeded inputs: bit-exact."""
import os

import numpy as np
import pytest
import torch

import gpu_cases
from oracle import build_ref, oracle
from sparseconv import _native

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def ref_module():
    if not os.path.exists(build_ref.OUT):
        pytest.skip("oracle/_ref was not built (reference sources absent where it was built)")
    return build_ref.load()


def _ref_map(mod, coords, shape, ks, dil):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_ref_maps", os.path.join(HERE, "golden", "make_ref_maps.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.reference_map(mod, coords, shape, ks, dil)


@pytest.mark.parametrize("name", sorted(gpu_cases.small_cases()))
def test_reference_cuda_map_equals_library_and_oracle(ref_module, name):
    coords, shape, ks, dil = gpu_cases.small_cases()[name]
    ref = _ref_map(ref_module, coords, shape, ks, dil)
    N, _C, W, H, D = shape
    nbr, _, _ = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    np.testing.assert_array_equal(nbr.cpu().numpy().view(np.uint32), ref)
    np.testing.assert_array_equal(oracle.neighbor_map(coords, shape, ks, dil), ref)


@pytest.mark.parametrize("name", ["cube", "lidar", "indoor", "wide3", "wide5", "indoor_shuffled"])
def test_reference_cuda_map_full_size(ref_module, name):
    """Full-size workloads. Their coordinates are sorted, so the 3x3x3 maps take the library's
    column path; `indoor_shuffled` permutes the indoor rows (seeded), which sends the 2M-voxel
    build down the hash path instead."""
    w = gpu_cases.workload(name.replace("_shuffled", ""))
    coords = w.coords
    if name.endswith("_shuffled"):
        coords = np.ascontiguousarray(coords[np.random.default_rng(5).permutation(coords.shape[0])])
    ref = _ref_map(ref_module, coords, w.shape, w.kernel_size, w.dilation)
    N, _C, W, H, D = w.shape
    nbr, _, _ = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D,
                                           w.kernel_size, w.dilation)
    np.testing.assert_array_equal(nbr.cpu().numpy().view(np.uint32), ref)
