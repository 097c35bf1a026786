"""Splitting one submanifold-conv problem across ranks (one process per GPU).

The path shards without any collective on the data path:

* **by batch index** — every sample is an independent problem (its voxels only see voxels of
  the same sample), so rank r takes the samples ``b`` with ``b % world == r`` and runs the
  ordinary single-GPU op on them; the weights are replicated;
* **by spatial slabs with halo voxels** — one large sample is cut along x into ``world`` slabs.
  Rank r owns the voxels with x in ``[lo_r, hi_r)`` and also receives the voxels within the
  kernel's reach of the slab (``halo = (K // 2) * dilation`` cells on each side), so the
  output rows of its owned voxels are exactly those of the unsharded conv: a submanifold output
  row depends only on input voxels within the kernel's reach.

Both helpers work on host or device tensors and return the global row ids of the local rows, so
results can be scattered back (``merge_rows``) when the caller wants one tensor. The benchmark's
multi-GPU mode is batch sharding with a fixed per-rank batch (weak scaling).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch


@dataclass
class Shard:
    coords: torch.Tensor      # [m, 4] int32, the rows this rank computes on
    feats: torch.Tensor       # [m, C]
    rows: torch.Tensor        # [m] int64: global row of each local row
    owned: torch.Tensor       # [m] bool: the local rows whose outputs this rank is responsible for


def batch_shard(coords: torch.Tensor, feats: torch.Tensor, rank: int, world: int) -> Shard:
    """Samples b with b % world == rank. Every local row is owned (no halo needed)."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world {world}")
    sel = (coords[:, 0].long() % world) == rank
    rows = torch.nonzero(sel, as_tuple=False).flatten()
    return Shard(coords[rows].contiguous(), feats[rows].contiguous(), rows,
                 torch.ones(rows.numel(), dtype=torch.bool, device=coords.device))


def slab_bounds(W: int, world: int) -> list:
    """x ranges [lo, hi) of the slabs, as equal as possible."""
    base, extra = divmod(W, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def slab_shard(coords: torch.Tensor, feats: torch.Tensor, rank: int, world: int, W: int,
               kernel_size: Sequence[int] = (3, 3, 3), dilation: Sequence[int] = (1, 1, 1)) -> Shard:
    """Voxels with x in the rank's slab (owned) plus those within the kernel's reach of it."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world {world}")
    lo, hi = slab_bounds(W, world)[rank]
    kx, dx = int(kernel_size[0]), int(dilation[0])
    halo_lo = (kx // 2) * dx                 # offsets reach x - (K//2)*d .. x + (K-1-K//2)*d
    halo_hi = (kx - 1 - kx // 2) * dx
    x = coords[:, 1].long()
    sel = (x >= lo - halo_lo) & (x < hi + halo_hi)
    rows = torch.nonzero(sel, as_tuple=False).flatten()
    xs = x[rows]
    owned = (xs >= lo) & (xs < hi)
    return Shard(coords[rows].contiguous(), feats[rows].contiguous(), rows, owned)


def merge_rows(total_rows: int, parts: Sequence[tuple]) -> torch.Tensor:
    """Scatter (rows, owned, out) triples from all ranks into one [total_rows, C] tensor."""
    first = parts[0][2]
    merged = torch.zeros((total_rows, first.shape[1]), dtype=first.dtype, device=first.device)
    written = torch.zeros(total_rows, dtype=torch.int32, device=first.device)
    for rows, owned, out in parts:
        r = rows[owned]
        merged[r] = out[owned]
        written[r] += 1
    if not bool((written == 1).all()):
        raise RuntimeError("shards do not cover every row exactly once")
    return merged


def _reduce(value: float, op, group=None) -> float:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op, group=group)
    return float(t.item())


def max_over_ranks(value: float, group=None) -> float:
    """The largest per-rank value (step times are reported as the max over ranks)."""
    import torch.distributed as dist
    return _reduce(value, dist.ReduceOp.MAX, group)


def sum_over_ranks(value: float, group=None) -> float:
    """The sum over ranks (whole-job voxel counts)."""
    import torch.distributed as dist
    return _reduce(value, dist.ReduceOp.SUM, group)
