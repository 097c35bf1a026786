"""Seeded synthetic voxel workloads with the shapes, sizes and value distributions of the
five benchmark configurations of the submanifold-conv path.

No dataset ships with the reference; these generators stand in for its inputs. Every
generator returns coordinates that are unique and sorted by (b, x, y, z), which is the
order ``SparseConvTensor.from_dense`` produces (``core.py:56-63``).

=====  ===========================================================  ===========  =========
name   geometry                                                     channels     dtype
=====  ===========================================================  ===========  =========
toy    B=3, 5^3 grid, voxels (i,i,i), i=0..4                         3 -> 3       float32
cube   B=4, 128^3, i.i.d. occupancy p=0.02 (~42k voxels/sample)      32 -> 32     float16
indoor B=8, 512^3, 20 clipped planes + 30 spheres, <=250k/sample     64 -> 64     bfloat16
lidar  B=8, 41(z) x 1600 x 1408, 64 beams on a ground plane at z=2    16 -> 16     float16
       plus 200 boxes, ~120k voxels/sample
wide   B=16, 256^3, i.i.d. occupancy p=0.005 (~84k voxels/sample)    128 -> 128   bfloat16
=====  ===========================================================  ===========  =========

Weights are N(0, 1/(V*Cin)) except for the toy (N(0,1)); features are N(0,1).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional, Tuple

import numpy as np
import torch

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


@dataclasses.dataclass
class Workload:
    name: str
    coords: np.ndarray            # [M, 4] int32, (b, x, y, z), unique, sorted
    feats: torch.Tensor           # [M, Cin] CPU tensor in ``dtype``
    weight: torch.Tensor          # [Cout, Kw, Kh, Kd, Cin] CPU tensor in ``dtype``
    shape: Tuple[int, int, int, int, int]   # (B, Cin, W, H, D), the reference's NCWHD size
    kernel_size: Tuple[int, int, int]
    dilation: Tuple[int, int, int]
    dtype: torch.dtype

    @property
    def num_voxels(self) -> int:
        return int(self.coords.shape[0])

    @property
    def kernel_volume(self) -> int:
        return int(np.prod(self.kernel_size))

    def describe(self) -> dict:
        B, C, W, H, D = self.shape
        return {"workload": self.name, "batch": B, "grid": [W, H, D],
                "voxels": self.num_voxels, "cin": int(self.weight.shape[-1]),
                "cout": int(self.weight.shape[0]), "kernel": list(self.kernel_size),
                "dtype": str(self.dtype).replace("torch.", "")}


def _sort_unique(coords: np.ndarray, W: int, H: int, D: int) -> np.ndarray:
    flat = (((coords[:, 0].astype(np.int64) * W + coords[:, 1]) * H + coords[:, 2]) * D
            + coords[:, 3])
    flat = np.unique(flat)
    z = flat % D
    t = flat // D
    y = t % H
    t //= H
    x = t % W
    b = t // W
    return np.ascontiguousarray(np.stack([b, x, y, z], axis=1).astype(np.int32))


def _bernoulli_grid(rng: np.random.Generator, B: int, W: int, H: int, D: int,
                    p: float) -> np.ndarray:
    """i.i.d. occupancy: a Binomial count per sample, then a uniform subset of cells."""
    cells = W * H * D
    out = []
    for b in range(B):
        k = int(rng.binomial(cells, p))
        flat = np.sort(rng.choice(cells, size=k, replace=False))
        z = flat % D
        y = (flat // D) % H
        x = flat // (D * H)
        out.append(np.stack([np.full(k, b), x, y, z], axis=1))
    return _sort_unique(np.concatenate(out).astype(np.int64), W, H, D)


def _features(rng: np.random.Generator, M: int, C: int, dtype: torch.dtype) -> torch.Tensor:
    f = rng.standard_normal((M, C), dtype=np.float32)
    return torch.from_numpy(f).to(dtype)


def _weights(rng: np.random.Generator, Co: int, K: Tuple[int, int, int], Ci: int,
             dtype: torch.dtype, std: Optional[float] = None) -> torch.Tensor:
    V = K[0] * K[1] * K[2]
    s = math.sqrt(1.0 / (V * Ci)) if std is None else std
    w = rng.standard_normal((Co, K[0], K[1], K[2], Ci), dtype=np.float32) * np.float32(s)
    return torch.from_numpy(w).to(dtype)


def toy(seed: int = 0) -> Workload:
    """README toy (``README.md:12-39``): diagonal voxels of a 5^3 grid, B=3, C=3, fp32."""
    rng = np.random.default_rng(seed)
    B, W = 3, 5
    c = [(b, i, i, i) for b in range(B) for i in range(W)]
    coords = np.asarray(c, dtype=np.int32)
    feats = _features(rng, coords.shape[0], 3, torch.float32)
    weight = _weights(rng, 3, (3, 3, 3), 3, torch.float32, std=1.0)
    return Workload("toy", coords, feats, weight, (B, 3, W, W, W), (3, 3, 3), (1, 1, 1),
                    torch.float32)


def cube(seed: int = 0, batch: int = 4, res: int = 128, p: float = 0.02, channels: int = 32,
         dtype: torch.dtype = torch.float16) -> Workload:
    """Random-occupancy cube: B=4, 128^3, p=0.02, C=32, fp16."""
    rng = np.random.default_rng(seed)
    coords = _bernoulli_grid(rng, batch, res, res, res, p)
    feats = _features(rng, coords.shape[0], channels, dtype)
    weight = _weights(rng, channels, (3, 3, 3), channels, dtype)
    return Workload("cube", coords, feats, weight, (batch, channels, res, res, res),
                    (3, 3, 3), (1, 1, 1), dtype)


def wide(seed: int = 0, batch: int = 16, res: int = 256, p: float = 0.005, channels: int = 128,
         kernel: int = 3, dtype: torch.dtype = torch.bfloat16) -> Workload:
    """Wide-channel stress: B=16, 256^3, p=0.005, C=128, 3^3 or 5^3, bf16."""
    rng = np.random.default_rng(seed)
    coords = _bernoulli_grid(rng, batch, res, res, res, p)
    feats = _features(rng, coords.shape[0], channels, dtype)
    K = (kernel, kernel, kernel)
    weight = _weights(rng, channels, K, channels, dtype)
    return Workload(f"wide{kernel}", coords, feats, weight, (batch, channels, res, res, res),
                    K, (1, 1, 1), dtype)


def _plane_voxels(rng: np.random.Generator, res: int) -> np.ndarray:
    c = rng.uniform(0, res, size=3)
    n = rng.standard_normal(3)
    n /= np.linalg.norm(n)
    a = np.cross(n, [1.0, 0.0, 0.0] if abs(n[0]) < 0.9 else [0.0, 1.0, 0.0])
    a /= np.linalg.norm(a)
    bvec = np.cross(n, a)
    ha, hb = rng.uniform(16, 112, size=2)
    s = np.arange(-ha, ha, 0.5)
    t = np.arange(-hb, hb, 0.5)
    S, T = np.meshgrid(s, t, indexing="ij")
    pts = c + S.reshape(-1, 1) * a + T.reshape(-1, 1) * bvec
    return np.floor(pts).astype(np.int64)


def _sphere_voxels(rng: np.random.Generator, res: int) -> np.ndarray:
    r = rng.uniform(10, 60)
    c = rng.uniform(0, res, size=3)
    n = int(math.ceil(4 * math.pi * r * r * 4))
    i = np.arange(n) + 0.5
    phi = np.arccos(1 - 2 * i / n)
    theta = math.pi * (1 + 5 ** 0.5) * i
    d = np.stack([np.cos(theta) * np.sin(phi), np.sin(theta) * np.sin(phi), np.cos(phi)], 1)
    return np.floor(c + r * d).astype(np.int64)


def indoor(seed: int = 0, batch: int = 8, res: int = 512, cap: int = 250_000,
           channels: int = 64, dtype: torch.dtype = torch.bfloat16) -> Workload:
    """Indoor-surface-like scene: per sample 20 clipped planes + 30 spheres at unit thickness.

    Objects are added in generation order; the object that crosses the per-sample cap keeps
    an x-ordered prefix of its new voxels, so no surface is thinned at random.
    """
    rng = np.random.default_rng(seed)
    out = []
    for b in range(batch):
        objs = [_plane_voxels(rng, res) for _ in range(20)] + \
               [_sphere_voxels(rng, res) for _ in range(30)]
        order = rng.permutation(len(objs))
        seen = np.empty(0, dtype=np.int64)
        for oi in order:
            p = objs[oi]
            p = p[np.all((p >= 0) & (p < res), axis=1)]
            flat = np.unique((p[:, 0] * res + p[:, 1]) * res + p[:, 2])
            flat = np.setdiff1d(flat, seen, assume_unique=True)
            room = cap - seen.size
            if room <= 0:
                break
            if flat.size > room:
                flat = flat[:room]
            seen = np.concatenate([seen, flat])
        z = seen % res
        y = (seen // res) % res
        x = seen // (res * res)
        out.append(np.stack([np.full(seen.size, b), x, y, z], axis=1))
    coords = _sort_unique(np.concatenate(out), res, res, res)
    feats = _features(rng, coords.shape[0], channels, dtype)
    weight = _weights(rng, channels, (3, 3, 3), channels, dtype)
    return Workload("indoor", coords, feats, weight, (batch, channels, res, res, res),
                    (3, 3, 3), (1, 1, 1), dtype)


def _ray_box_hits(orig: np.ndarray, dirs: np.ndarray, az: np.ndarray, lo: np.ndarray,
                  hi: np.ndarray) -> np.ndarray:
    """Nearest positive hit distance of each ray with a set of axis-aligned boxes (slab test).

    ``dirs`` is [n_az, n_beams, 3] with azimuth ``az`` ascending; each box is tested only
    against the azimuth columns its footprint subtends.
    """
    n_az, n_b, _ = dirs.shape
    best = np.full((n_az, n_b), np.inf, dtype=np.float32)
    inv = 1.0 / np.where(np.abs(dirs) < 1e-9, 1e-9, dirs)
    for k in range(lo.shape[0]):
        cx = np.array([lo[k, 0], hi[k, 0], lo[k, 0], hi[k, 0]]) - orig[0]
        cy = np.array([lo[k, 1], lo[k, 1], hi[k, 1], hi[k, 1]]) - orig[1]
        ang = np.arctan2(cy, cx)
        a0, a1 = np.searchsorted(az, ang.min()), np.searchsorted(az, ang.max()) + 1
        if a1 <= a0:
            continue
        iv = inv[a0:a1]
        t1 = (lo[k] - orig) * iv
        t2 = (hi[k] - orig) * iv
        tmin = np.minimum(t1, t2).max(axis=-1)
        tmax = np.maximum(t1, t2).min(axis=-1)
        hit = (tmax >= np.maximum(tmin, 0)) & (tmin > 0)
        cur = best[a0:a1]
        best[a0:a1] = np.where(hit & (tmin < cur), tmin, cur)
    return best.reshape(-1)


def lidar(seed: int = 0, batch: int = 8, channels: int = 16, azimuth_steps: int = 4096,
          noise: float = 0.06, dtype: torch.dtype = torch.float16) -> Workload:
    """Outdoor-LiDAR-like sweep on a 41(z) x 1600(y) x 1408(x) grid, coords (b, z, y, x).

    A 64-beam sensor 1.7 m above a ground plane at voxel z=2 scans the forward half-space;
    each ray stops at the ground or at the nearest of 200 axis-aligned boxes, and each
    return gets N(0, ``noise``) metres of jitter. Voxels are 0.05 m in x and y and 0.1 m
    in z, so point density falls off with range from the sensor at the grid's x=0 face.
    """
    rng = np.random.default_rng(seed)
    Wz, Hy, Dx = 41, 1600, 1408
    vz, vxy = 0.1, 0.05
    ground_z = 2 * vz + 0.5 * vz
    sensor = np.array([0.0, 0.0, ground_z + 1.7], dtype=np.float32)   # metric (x, y, z)
    elev = np.deg2rad(np.linspace(-24.9, 2.0, 64))
    az = np.deg2rad(np.linspace(-89.9, 89.9, azimuth_steps))
    A, E = np.meshgrid(az, elev, indexing="ij")
    dirs = np.stack([np.cos(E) * np.cos(A), np.cos(E) * np.sin(A), np.sin(E)], -1)
    dirs = dirs.astype(np.float32)
    flat_dirs = dirs.reshape(-1, 3)
    out = []
    for b in range(batch):
        ctr = np.stack([rng.uniform(4, 70, 200), rng.uniform(-40, 40, 200)], 1)
        size = rng.uniform(1.5, 4.5, (200, 2))
        height = rng.uniform(1.4, 3.0, 200)
        lo = np.concatenate([ctr - size / 2, np.full((200, 1), ground_z)], 1).astype(np.float32)
        hi = np.concatenate([ctr + size / 2, (ground_z + height)[:, None]], 1).astype(np.float32)
        t_box = _ray_box_hits(sensor, dirs, az, lo, hi)
        with np.errstate(divide="ignore", invalid="ignore"):
            t_gnd = np.where(flat_dirs[:, 2] < 0, (ground_z - sensor[2]) / flat_dirs[:, 2], np.inf)
        t = np.minimum(t_box, t_gnd)
        ok = np.isfinite(t)
        pts = sensor + flat_dirs[ok] * t[ok, None]
        pts += rng.normal(0.0, noise, pts.shape).astype(np.float32)
        pts[:, 2] = np.maximum(pts[:, 2], ground_z)          # ground returns sit on the plane
        xi = np.floor(pts[:, 0] / vxy).astype(np.int64)
        yi = np.floor((pts[:, 1] + 40.0) / vxy).astype(np.int64)
        zi = np.floor(pts[:, 2] / vz).astype(np.int64)
        keep = (xi >= 0) & (xi < Dx) & (yi >= 0) & (yi < Hy) & (zi >= 0) & (zi < Wz)
        c = np.stack([np.full(int(keep.sum()), b), zi[keep], yi[keep], xi[keep]], 1)
        out.append(c)
    coords = _sort_unique(np.concatenate(out), Wz, Hy, Dx)
    feats = _features(rng, coords.shape[0], channels, dtype)
    weight = _weights(rng, channels, (3, 3, 3), channels, dtype)
    return Workload("lidar", coords, feats, weight, (batch, channels, Wz, Hy, Dx),
                    (3, 3, 3), (1, 1, 1), dtype)


CONFIGS = {
    "toy": toy,
    "cube": cube,
    "indoor": indoor,
    "lidar": lidar,
    "wide3": lambda seed=0, **kw: wide(seed, kernel=3, **kw),
    "wide5": lambda seed=0, **kw: wide(seed, kernel=5, **kw),
}


def make(name: str, seed: int = 0, **kw) -> Workload:
    if name not in CONFIGS:
        raise ValueError(f"unknown workload {name!r}; choose from {sorted(CONFIGS)}")
    return CONFIGS[name](seed=seed, **kw)
