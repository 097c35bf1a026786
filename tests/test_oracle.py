"""The oracle, pinned: the C restatement of the reference's kernel-map build and the float64
conv oracles, checked against the reference's own outputs (golden fixtures), its known
answers, and an independent pure-Python restatement. CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _py_neighbor_map(coords, shape, ks, dil):
    """Pure-Python restatement of neighbor_map.cu:145-176 over a dict (small inputs only)."""
    N, _C, W, H, D = shape
    Kw, Kh, Kd = ks
    Dw, Dh, Dd = dil
    V = Kw * Kh * Kd
    table = {}
    for i, (b, x, y, z) in enumerate(coords.tolist()):
        table[b * W * H * D + x * H * D + y * D + z] = i   # hash.cu:384, last insert wins
    out = np.full((len(coords), V), 0xFFFFFFFF, dtype=np.uint32)
    for i, (b, x, y, z) in enumerate(coords.tolist()):
        x0, y0, z0 = x - Kw // 2 * Dw, y - Kh // 2 * Dh, z - Kd // 2 * Dd
        for v in range(V):
            if v == V // 2:
                out[i, v] = i
                continue
            kx = x0 + v // (Kh * Kd) * Dw
            ky = y0 + v // Kd % Kh * Dh
            kz = z0 + v % Kd * Dd
            if 0 <= kx < W and 0 <= ky < H and 0 <= kz < D:
                r = table.get(b * W * H * D + kx * H * D + ky * D + kz)
                if r is not None:
                    out[i, v] = r
    return out


def _random_coords(rng, B, W, H, D, p):
    occ = rng.random((B, W, H, D)) < p
    return np.ascontiguousarray(np.argwhere(occ).astype(np.int32))


def test_readme_toy_known_answer_map():
    g = np.load(os.path.join(GOLDEN, "readme_toy.npz"))
    nbr = oracle.neighbor_map(g["coords"], g["shape"], (3, 3, 3))
    np.testing.assert_array_equal(nbr, g["neighbor_map"])


def test_readme_toy_features_match_reference_explicit_gemm():
    """The reference's own EXPLICIT_GEMM (run on CPU to make the fixture) vs the oracle."""
    g = np.load(os.path.join(GOLDEN, "readme_toy.npz"))
    nbr = oracle.neighbor_map(g["coords"], g["shape"], (3, 3, 3))
    out = oracle.conv_gather_f64(g["feats"], nbr, g["weight"])
    np.testing.assert_allclose(out, g["reference_explicit_out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out, g["conv3d_f64_out"], rtol=1e-10, atol=1e-10)
    dense = oracle.conv_dense_f64(g["feats"], g["coords"], g["shape"], g["weight"])
    np.testing.assert_allclose(dense, g["conv3d_f64_out"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("ks,dil", [((3, 3, 3), (1, 1, 1)), ((5, 5, 5), (1, 1, 1)),
                                    ((3, 3, 3), (2, 2, 2)), ((2, 2, 2), (1, 1, 1)),
                                    ((4, 3, 2), (1, 2, 3)), ((1, 1, 1), (1, 1, 1))])
def test_c_restatement_matches_python_restatement(ks, dil):
    rng = np.random.default_rng(7)
    coords = _random_coords(rng, 2, 9, 7, 11, 0.2)
    shape = (2, 4, 9, 7, 11)
    np.testing.assert_array_equal(oracle.neighbor_map(coords, shape, ks, dil),
                                  _py_neighbor_map(coords, shape, ks, dil))


def test_c_restatement_uint64_keys():
    """N*W*H*D >= 2^32 switches the reference to uint64 keys (ops/utils.py:6-9)."""
    rng = np.random.default_rng(3)
    B, W, H, D = 2, 2048, 2048, 1024
    n = 3000
    c = np.stack([rng.integers(0, B, n), rng.integers(0, 8, n) + 1000,
                  rng.integers(0, 8, n) + 2000, rng.integers(0, 8, n) + 1010], 1)
    coords = np.unique(c, axis=0).astype(np.int32)
    shape = (B, 1, W, H, D)
    assert B * W * H * D >= 2 ** 32
    np.testing.assert_array_equal(oracle.neighbor_map(coords, shape, (3, 3, 3)),
                                  _py_neighbor_map(coords, shape, (3, 3, 3), (1, 1, 1)))


def test_duplicate_coordinates_last_row_wins():
    coords = np.array([[0, 1, 1, 1], [0, 1, 1, 2], [0, 1, 1, 1]], dtype=np.int32)
    nbr = oracle.neighbor_map(coords, (1, 1, 4, 4, 4), (3, 3, 3))
    # voxel (1,1,2) sees (1,1,1) at offset dz=-1 (v=12): the later duplicate, row 2
    assert nbr[1, 12] == 2
    assert nbr[0, 13] == 0 and nbr[2, 13] == 2


def test_gather_oracle_matches_dense_oracle():
    rng = np.random.default_rng(11)
    coords = _random_coords(rng, 2, 8, 9, 10, 0.25)
    shape = (2, 5, 8, 9, 10)
    feats = rng.standard_normal((coords.shape[0], 5))
    for ks, dil in [((3, 3, 3), (1, 1, 1)), ((5, 3, 3), (1, 2, 1))]:
        w = rng.standard_normal((4,) + ks + (5,))
        b = rng.standard_normal(4)
        nbr = oracle.neighbor_map(coords, shape, ks, dil)
        g = oracle.conv_gather_f64(feats, nbr, w, b)
        d = oracle.conv_dense_f64(feats, coords, shape, w, b, dil)
        np.testing.assert_allclose(g, d, rtol=1e-10, atol=1e-10)


def test_explicit_gemm_restatement_matches_gather_oracle():
    rng = np.random.default_rng(5)
    coords = _random_coords(rng, 1, 10, 10, 10, 0.3)
    shape = (1, 6, 10, 10, 10)
    feats = rng.standard_normal((coords.shape[0], 6)).astype(np.float32)
    w = rng.standard_normal((7, 3, 3, 3, 6)).astype(np.float32)
    b = rng.standard_normal(7).astype(np.float32)
    nbr = oracle.neighbor_map(coords, shape, (3, 3, 3))
    out = oracle.explicit_gemm_cpu(torch.from_numpy(feats), nbr, torch.from_numpy(w), torch.from_numpy(b))
    np.testing.assert_allclose(out.numpy(), oracle.conv_gather_f64(feats, nbr, w, b), rtol=1e-4, atol=1e-4)


def test_reference_map_fixtures():
    """Maps produced by the reference's own CUDA map builder on a B200
    (tests/golden/make_ref_maps.py) against the C restatement."""
    path = os.path.join(GOLDEN, "ref_maps.npz")
    if not os.path.exists(path):
        pytest.skip("ref_maps.npz has not been generated")
    d = np.load(path)
    names = sorted({k.split("__")[0] for k in d.files})
    assert names
    for name in names:
        coords, shape = d[f"{name}__coords"], d[f"{name}__shape"]
        ks, dil = d[f"{name}__kernel"], d[f"{name}__dilation"]
        np.testing.assert_array_equal(oracle.neighbor_map(coords, shape, ks, dil),
                                      d[f"{name}__map"], err_msg=name)


@pytest.mark.parametrize("dil", [(1, 1, 1), (1, 1, 2)])
def test_adjacent_rows_are_z_neighbours_of_sorted_unique_coords(dil):
    """The 3x3x3 map kernel takes offsets V/2 - 1 and V/2 + 1 (z - d, z + d) from the adjacent
    input rows when those rows hold exactly that coordinate and no coordinate repeats. For
    unique coordinates that is the reference's answer: check it on the oracle's maps."""
    rng = np.random.default_rng(3)
    shape = (2, 1, 12, 10, 40)
    cells = np.stack(np.meshgrid(np.arange(2), np.arange(12), np.arange(10), np.arange(40), indexing="ij"), -1)
    cells = cells.reshape(-1, 4)
    coords = cells[rng.random(len(cells)) < 0.35].astype(np.int32)   # sorted (b, x, y, z), unique
    nbr = oracle.neighbor_map(coords, shape, (3, 3, 3), dil).view(np.int32)
    V, d = 27, dil[2]
    up = np.nonzero(np.all(coords[1:] == coords[:-1] + np.array([0, 0, 0, d]), axis=1))[0]
    down = np.nonzero(np.all(coords[:-1] == coords[1:] - np.array([0, 0, 0, d]), axis=1))[0] + 1
    assert len(up) > 100 and len(down) > 100
    np.testing.assert_array_equal(nbr[up, V // 2 + 1], up + 1)
    np.testing.assert_array_equal(nbr[down, V // 2 - 1], down - 1)
