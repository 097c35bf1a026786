"""Seeded inputs shared by the GPU parity tests and the golden-map generator.

Small cases (oracle-sized) cover every kernel shape the reference accepts: 3^3 and 5^3,
even sizes (the centre rule v == V/2 of neighbor_map.cu:159-160 then is not the geometric
centre), anisotropic sizes and dilations, a 1^3 kernel, a 64-bit-key volume
(N*W*H*D >= 2^32, ops/utils.py:6-9), and a single voxel.
"""
import functools

import numpy as np


def random_coords(seed, B, W, H, D, p):
    rng = np.random.default_rng(seed)
    occ = rng.random((B, W, H, D)) < p
    return np.ascontiguousarray(np.argwhere(occ).astype(np.int32))


def key64_coords(seed, n=4000):
    rng = np.random.default_rng(seed)
    B, W, H, D = 2, 2048, 2048, 1024
    c = np.stack([rng.integers(0, B, n), rng.integers(0, 10, n) + 1000,
                  rng.integers(0, 10, n) + 2030, rng.integers(0, 10, n) + 1012], 1)
    return np.unique(c, axis=0).astype(np.int32), (B, 1, W, H, D)


def small_cases():
    """name -> (coords [M,4] int32, shape NCWHD, kernel, dilation)."""
    cases = {
        "rand3": (random_coords(1, 2, 20, 18, 16, 0.05), (2, 1, 20, 18, 16), (3, 3, 3), (1, 1, 1)),
        "dense3": (random_coords(2, 1, 12, 12, 12, 0.6), (1, 1, 12, 12, 12), (3, 3, 3), (1, 1, 1)),
        "rand5": (random_coords(3, 2, 16, 16, 16, 0.08), (2, 1, 16, 16, 16), (5, 5, 5), (1, 1, 1)),
        "dil2": (random_coords(4, 2, 16, 16, 16, 0.1), (2, 1, 16, 16, 16), (3, 3, 3), (2, 2, 2)),
        "even2": (random_coords(5, 1, 10, 10, 10, 0.3), (1, 1, 10, 10, 10), (2, 2, 2), (1, 1, 1)),
        "aniso": (random_coords(6, 3, 9, 14, 7, 0.2), (3, 1, 9, 14, 7), (4, 3, 2), (1, 2, 3)),
        "k1": (random_coords(7, 1, 8, 8, 8, 0.3), (1, 1, 8, 8, 8), (1, 1, 1), (1, 1, 1)),
        "single": (np.array([[0, 2, 3, 4]], dtype=np.int32), (1, 1, 5, 6, 7), (3, 3, 3), (1, 1, 1)),
    }
    c64, s64 = key64_coords(8)
    cases["key64"] = (c64, s64, (3, 3, 3), (1, 1, 1))
    return cases


def mixed_density_coords(seed=9):
    """Dense blocks (tiles with most of the 27 offsets active) beside scattered voxels (tiles
    with one or two): both index-staging modes of the tensor-core conv run in one launch."""
    rng = np.random.default_rng(seed)
    B, R = 2, 40
    occ = rng.random((B, R, R, R)) < 0.01
    occ[0, 4:16, 4:16, 4:16] |= rng.random((12, 12, 12)) < 0.9
    occ[1, 20:34, 10:20, 25:39] |= rng.random((14, 10, 14)) < 0.7
    return np.ascontiguousarray(np.argwhere(occ).astype(np.int32)), (B, 1, R, R, R)


@functools.lru_cache(maxsize=None)
def workload(name):
    from sparseconv import synthetic
    return synthetic.make(name)
