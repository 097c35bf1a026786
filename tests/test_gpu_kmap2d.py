"""2-D submanifold map (the reference's hashmap_build_submanifold_conv2d_neighbor_map_cuda_naive,
neighbor_map.cu:10-111): bit-exact against the oracle (its 3-D map with D = 1, Kd = 1, z = 0)
and, when oracle/_ref was built, against the reference's own 2-D builder run live."""
import os

import numpy as np
import pytest
import torch

from oracle import build_ref, oracle
from sparseconv import _native

pytestmark = pytest.mark.gpu


def _cases():
    out = {}
    for name, seed, B, W, H, p, ks, dil in [
            ("rand3x3", 1, 2, 40, 36, 0.2, (3, 3), (1, 1)),
            ("rand5x5", 2, 1, 30, 30, 0.3, (5, 5), (1, 1)),
            ("even2x2", 3, 1, 20, 20, 0.4, (2, 2), (1, 1)),
            ("aniso3x5_dil", 4, 3, 17, 23, 0.25, (3, 5), (2, 1)),
            ("dense3x3", 5, 1, 64, 64, 0.9, (3, 3), (1, 1))]:
        rng = np.random.default_rng(seed)
        c = np.ascontiguousarray(np.argwhere(rng.random((B, W, H)) < p).astype(np.int32))
        out[name] = (c, (B, W, H), ks, dil)
    return out


def _ours(c, B, W, H, ks, dil):
    nbr, masks, order = _native.build_neighbor_map_2d(torch.from_numpy(c).cuda(), B, W, H, ks, dil)
    torch.cuda.synchronize()
    return nbr.cpu().numpy().view(np.uint32), masks.cpu().numpy().view(np.uint32), order.cpu().numpy()


@pytest.mark.parametrize("name", sorted(_cases()))
def test_2d_map_matches_oracle(name):
    c, (B, W, H), ks, dil = _cases()[name]
    nbr, masks, order = _ours(c, B, W, H, ks, dil)
    c4 = np.ascontiguousarray(np.concatenate([c, np.zeros((c.shape[0], 1), np.int32)], axis=1))
    ref = oracle.neighbor_map(c4, (B, 1, W, H, 1), (ks[0], ks[1], 1), (dil[0], dil[1], 1))
    np.testing.assert_array_equal(nbr, ref)
    V = ks[0] * ks[1]
    bits = np.zeros(c.shape[0], np.uint64)
    for v in range(V):
        bits |= (ref[:, v] != 0xFFFFFFFF).astype(np.uint64) << np.uint64(v)
    np.testing.assert_array_equal(masks[:, 0].astype(np.uint64), bits)
    assert np.array_equal(np.sort(order), np.arange(c.shape[0]))


@pytest.fixture(scope="module")
def ref_module():
    if not os.path.exists(build_ref.OUT):
        pytest.skip("oracle/_ref was not built (reference sources absent where it was built)")
    return build_ref.load()


@pytest.mark.parametrize("name", sorted(_cases()))
def test_2d_map_matches_reference_builder(ref_module, name):
    c, (B, W, H), ks, dil = _cases()[name]
    coords = torch.from_numpy(c).cuda()
    cap = int(2.0 * c.shape[0])
    keys = torch.full((cap,), torch.iinfo(torch.uint32).max, dtype=torch.uint32, device="cuda")
    vals = torch.empty((cap,), dtype=torch.uint32, device="cuda")
    ref = ref_module.hashmap_build_submanifold_conv2d_neighbor_map_cuda_naive(
        keys, vals, coords, W, H, ks[0], ks[1], dil[0], dil[1])
    torch.cuda.synchronize()
    nbr, _, _ = _ours(c, B, W, H, ks, dil)
    np.testing.assert_array_equal(nbr, ref.cpu().numpy().astype(np.uint32))


def test_2d_empty_and_bad_coords():
    nbr, masks, order = _native.build_neighbor_map_2d(torch.zeros((0, 3), dtype=torch.int32, device="cuda"),
                                                       1, 8, 8, (3, 3), (1, 1))
    assert nbr.shape == (0, 9) and order.shape == (0,)
    with pytest.raises(ValueError):
        _native.build_neighbor_map_2d(torch.zeros((4, 4), dtype=torch.int32, device="cuda"), 1, 8, 8, (3, 3), (1, 1))
