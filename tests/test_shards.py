"""Sharding across ranks (CPU): batch and spatial-slab shards must reproduce the unsharded
result exactly on the rows each rank owns; the timing reductions run over a two-rank gloo
group. The conv results come from the float64 oracle (the checker), not the product kernels."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from sparseconv import shards


def _scene(seed=0, B=3, R=24, p=0.15, C=4):
    rng = np.random.default_rng(seed)
    occ = rng.random((B, R, R, R)) < p
    b, x, y, z = np.nonzero(occ)
    coords = np.stack([b, x, y, z], 1).astype(np.int32)
    feats = rng.standard_normal((coords.shape[0], C))
    weight = rng.standard_normal((C + 1, 3, 3, 3, C))
    return coords, feats, weight, (B, C, R, R, R)


def _oracle_out(coords, feats, weight, shape, ks=(3, 3, 3), dil=(1, 1, 1)):
    nbr = oracle.neighbor_map(np.ascontiguousarray(coords), shape, ks, dil)
    return oracle.conv_gather_f64(feats, nbr, weight)


def test_batch_shard_partitions_rows():
    coords, feats, _w, _s = _scene()
    c, f = torch.from_numpy(coords), torch.from_numpy(feats)
    seen = torch.zeros(c.shape[0], dtype=torch.int32)
    for r in range(2):
        sh = shards.batch_shard(c, f, r, 2)
        assert bool(((sh.coords[:, 0] % 2) == r).all())
        seen[sh.rows] += 1
    assert bool((seen == 1).all())


@pytest.mark.parametrize("world", [2, 3])
def test_batch_shard_matches_unsharded(world):
    coords, feats, weight, shape = _scene(1)
    full = _oracle_out(coords, feats, weight, shape)
    c, f = torch.from_numpy(coords), torch.from_numpy(feats)
    parts = []
    for r in range(world):
        sh = shards.batch_shard(c, f, r, world)
        out = _oracle_out(sh.coords.numpy(), sh.feats.numpy(), weight, shape)
        parts.append((sh.rows, sh.owned, torch.from_numpy(out)))
    merged = shards.merge_rows(coords.shape[0], parts)
    np.testing.assert_array_equal(merged.numpy(), full)


@pytest.mark.parametrize("world,ks,dil", [(2, (3, 3, 3), (1, 1, 1)), (3, (3, 3, 3), (2, 1, 1)),
                                          (4, (5, 5, 5), (1, 1, 1)), (2, (2, 2, 2), (1, 1, 1))])
def test_slab_shard_matches_unsharded(world, ks, dil):
    coords, feats, _w, shape = _scene(2, B=2, R=20, p=0.2)
    rng = np.random.default_rng(3)
    weight = rng.standard_normal((5, ks[0], ks[1], ks[2], feats.shape[1]))
    full = _oracle_out(coords, feats, weight, shape, ks, dil)
    c, f = torch.from_numpy(coords), torch.from_numpy(feats)
    parts = []
    for r in range(world):
        sh = shards.slab_shard(c, f, r, world, shape[2], ks, dil)
        out = _oracle_out(sh.coords.numpy(), sh.feats.numpy(), weight, shape, ks, dil)
        parts.append((sh.rows, sh.owned, torch.from_numpy(out)))
    merged = shards.merge_rows(coords.shape[0], parts)
    np.testing.assert_array_equal(merged.numpy(), full)


def test_slab_bounds_cover_axis():
    for W in (1, 7, 128, 1600):
        for world in (1, 2, 3, 8):
            b = shards.slab_bounds(W, world)
            assert b[0][0] == 0 and b[-1][1] == W
            assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        coords, feats, weight, shape = _scene(4, B=1, R=24, p=0.2)
        c, f = torch.from_numpy(coords), torch.from_numpy(feats)
        sh = shards.slab_shard(c, f, rank, world, shape[2])
        out = torch.from_numpy(_oracle_out(sh.coords.numpy(), sh.feats.numpy(), weight, shape))
        gathered = [None] * world
        dist.all_gather_object(gathered, (sh.rows, sh.owned, out))
        step_ms = 1.0 + rank                      # a per-rank "time"
        mx = shards.max_over_ranks(step_ms)
        sm = shards.sum_over_ranks(float(sh.owned.sum()))
        if rank == 0:
            merged = shards.merge_rows(coords.shape[0], gathered)
            full = _oracle_out(coords, feats, weight, shape)
            ok = np.array_equal(merged.numpy(), full) and mx == float(world) and sm == coords.shape[0]
            open(os.path.join(result_dir, "ok" if ok else "bad"), "w").write(f"{mx} {sm}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_slab_shards(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert (tmp_path / "ok").exists(), os.listdir(tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("how", ["batch", "slab"])
def test_gpu_shards_reproduce_unsharded_rows(how):
    """The product op on each shard gives, on the rows the shard owns, the same bits as the op
    on the whole problem (the conv's result does not depend on which other voxels share a
    launch, only on each row's own neighbours)."""
    from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d
    dev = torch.device("cuda", 0)
    coords, feats, _w, shape = _scene(5, B=3, R=40, p=0.05, C=32)
    rng = np.random.default_rng(6)
    weight = torch.from_numpy(rng.standard_normal((32, 3, 3, 3, 32)) / 16).half().to(dev)
    c = torch.from_numpy(coords).to(dev)
    f = torch.from_numpy(feats).half().to(dev)
    full, _ = sparse_submanifold_conv3d(f, c, torch.Size(shape), weight, algorithm=Algorithm.IMPLICIT_GEMM)
    parts = []
    for r in range(3):
        sh = shards.batch_shard(c, f, r, 3) if how == "batch" else shards.slab_shard(c, f, r, 3, shape[2])
        out, _ = sparse_submanifold_conv3d(sh.feats, sh.coords, torch.Size(shape), weight,
                                           algorithm=Algorithm.IMPLICIT_GEMM)
        parts.append((sh.rows, sh.owned, out))
    merged = shards.merge_rows(coords.shape[0], parts)
    torch.cuda.synchronize()
    assert torch.equal(merged, full)


@pytest.mark.parametrize("world", [2, 3, 4])
def test_bench_batch_split_renumbers_samples_and_matches_unsharded(world):
    """bench.py's strong-scaling split: rank r takes the samples b % world == r, renumbered
    b // world on a grid of its own samples; every row lands on exactly one rank and each rank's
    float64 oracle conv equals the unsharded one on its rows."""
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    from sparseconv import synthetic
    w = synthetic.cube(seed=3, batch=4, res=16, p=0.1)
    full_nbr = oracle.neighbor_map(w.coords, w.shape, w.kernel_size, w.dilation)
    full = oracle.conv_gather_f64(w.feats.double().numpy(), full_nbr, w.weight.double().numpy())
    seen = np.zeros(w.num_voxels, dtype=np.int64)
    for r in range(world):
        loc = bench._batch_local(w, r, world)
        assert loc.shape[0] == len(range(r, 4, world))
        assert loc.coords[:, 0].max() < loc.shape[0]
        rows = np.nonzero(w.coords[:, 0] % world == r)[0]
        seen[rows] += 1
        np.testing.assert_array_equal(loc.coords[:, 1:], w.coords[rows, 1:])
        nbr = oracle.neighbor_map(loc.coords, loc.shape, loc.kernel_size, loc.dilation)
        out = oracle.conv_gather_f64(loc.feats.double().numpy(), nbr, loc.weight.double().numpy())
        np.testing.assert_array_equal(out, full[rows])
    assert (seen == 1).all()
