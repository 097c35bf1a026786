"""Benchmark of the submanifold-conv path: kernel-map build + implicit-GEMM conv.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cube] [--impl ours|reference]

One step = ``sparse_submanifold_conv3d(feats, coords, shape, weight, IMPLICIT_GEMM)`` on one
batch with no cached map: hash-table build, kernel map, voxel order and conv. The default
workload is the indoor-surface scene (B=8, 512^3, 20 planes + 30 spheres per sample, 2.0 M
voxels, C=64 -> 64, 3^3, bf16), the largest single-GPU workload; others (``cube``, ``lidar``,
``wide3``, ``wide5``, ``toy``) run with ``--workload``.

Metric: voxels/s over all ranks (plus effective TFLOP/s in ``effective``). Under torchrun the
default ``--shard batch`` splits the workload's own batch over the ranks (rank r takes the
samples b with b % N == r, renumbered locally; strong scaling: the total work is fixed), with
no collective on the data path; ``--shard replica`` gives every rank its own full batch of the
same shape (seed = rank; weak scaling). The step time is the max over ranks of the summed
per-step CUDA-event durations. The timed steps are replays of a CUDA graph holding one complete forward (no
cached map), so host-side Python does not sit between kernels; the eager API time per step is
reported beside it. The L2 (126 MB) is flushed by a 256 MB write between timed steps, outside
the step events. Per-kernel times (``stages_ms_per_step``, ``roofline``) come from the
library's CUDA events around each launch, over eager steps that each follow a flush;
``cached_map`` is the same metric for the conv alone, as when a layer reuses the map.

``e2e`` is the same metric through the public API from pinned host buffers: H2D copy of
coords and features, the op, D2H copy of the output, all inside the timed region, with steps
pipelined over two CUDA streams (step i+1's H2D overlaps step i's op and D2H, as a host feeding
batches would run them); ``e2e.serial_value`` is the same with every step on one stream.

``--impl reference`` times the reference's CPU path on this host instead: the oracle's C
restatement of the reference map builder (OpenMP, all cores, every voxel) plus the reference's
EXPLICIT_GEMM forward restated on CPU torch in fp32 (all threads) over a row sample of the map
(at most 2^27 im2col elements), scaled to the whole workload; rank 0 only. That line and, at
N=1, this library's own line carry ``reference_gpu``: the reference's own GPU forward (its CUDA
map builder compiled from its sources + its Triton implicit GEMM, through its public
``sparse_submanifold_conv3d``) timed on cuda:0 by ``oracle/ref_gpu.py`` in a separate process
(``--no-reference-gpu`` leaves it out of this library's line).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sparse-conv_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "subm-conv3d voxels/sec (map build + conv)"
UNIT = "voxels/s"
L2_FLUSH_BYTES = 256 << 20


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def _traffic_per_launch(key: str):
    """DRAM bytes (read + write) per launch of a kernel, from the committed ncu summary
    `profiles/traffic_per_launch.txt` (lines `workload:kernel bytes`), or None."""
    path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == key:
            return int(parts[1])
    return None


def _launches_per_step(M: int, kernel, shape) -> int:
    """Kernels one forward launches: for 3x3x3 kernels on grids of < 2^32 cells and <= 2^23
    (b, x, y) columns the sorted-input prep and the conditional table clear; insert, map, order
    (one bucket scatter, or, for maps of <= 27-offset kernels of >= 2^19 voxels or of > 2^17
    voxels filling at most 0.3 % of the grid, a scan and a scatter per 8-bit radix pass plus a
    count for every pass after the first, whose counts the map kernel makes), conv. Workspace
    clears are driver memsets, not counted."""
    V = int(np.prod(kernel))
    N, W, H, D = int(shape[0]), int(shape[2]), int(shape[3]), int(shape[4])
    cells = N * W * H * D
    prep = 2 if tuple(kernel) == (3, 3, 3) and cells < (1 << 32) and N * W * H <= (1 << 23) else 0
    if V <= 27 and (M >= (1 << 19) or ((1 << 17) < M <= 0.003 * cells)):
        drop = max(V - 21, 0)
        passes = (4 + V - 1 - drop + 7) // 8
        return prep + 2 + 3 * passes - 1 + 1
    return prep + 4


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _alg_figures(w, nnz: int):
    Ci, Co = int(w.weight.shape[-1]), int(w.weight.shape[0])
    V = w.kernel_volume
    M = w.num_voxels
    s = torch.tensor([], dtype=w.dtype).element_size()
    MW = (V + 31) // 32
    flops_alg = 2.0 * Ci * Co * nnz
    flops_dense = 2.0 * Ci * Co * M * V
    # algorithmic bytes per launch (each distinct row counted once)
    conv_bytes = M * (Ci * s + Co * s + 4 * V + 4 * MW + 4) + Co * V * Ci * s
    map_bytes = M * (16 + 4 * V + 4 * MW)              # map_kernel: coords in, map + masks out
    insert_bytes = M * (16 + 8)                          # coords in, one table slot written
    order_bytes = M * (4 * MW + 4)
    return dict(flops_alg=flops_alg, flops_dense=flops_dense, conv_bytes=conv_bytes,
                map_bytes=map_bytes, insert_bytes=insert_bytes, order_bytes=order_bytes)


def _config(w) -> dict:
    """The workload's description; both arms print exactly this dict as ``config``."""
    return dict(w.describe(), l2="GPU arm: flushed between timed steps (256 MB write)")


def _cpu_sampler(w):
    """One CPU step of the reference's path on the host's cores, as a function returning its
    estimated time for the whole workload: the oracle's C map build over every voxel (OpenMP)
    plus the reference's EXPLICIT_GEMM forward (CPU torch, fp32) over the first ``rows`` rows of
    the map, its time scaled by M / rows. The sample bounds im2col at 2^27 elements."""
    sys.path.insert(0, ROOT)
    from oracle import oracle
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    feats32, weight32 = w.feats.float(), w.weight.float()
    M, V, Ci = w.num_voxels, w.kernel_volume, int(w.weight.shape[-1])
    rows = int(min(M, max(4096, (1 << 27) // max(1, V * Ci))))

    def step() -> float:
        t0 = time.perf_counter()
        nbr = oracle.neighbor_map(w.coords, w.shape, w.kernel_size, w.dilation, nthreads=cores)
        t1 = time.perf_counter()
        oracle.explicit_gemm_cpu(feats32, nbr[:rows], weight32)
        t2 = time.perf_counter()
        return (t1 - t0) + (t2 - t1) * (M / rows)

    sample = (f"{w.name} ({M} voxels): oracle C map build of every voxel (OpenMP, {cores} threads) "
              f"+ EXPLICIT_GEMM restated on CPU torch fp32 over the first {rows} map rows, conv time "
              f"scaled x{M / rows:.2f} to the whole workload")
    return step, cores, sample


def _reference_gpu(workload: str, steps: int, warmup: int) -> dict:
    """The reference's own GPU forward (oracle/ref_gpu.py, a separate process) or why not."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    script = os.path.join(ROOT, "oracle", "ref_gpu.py")
    try:
        r = subprocess.run([sys.executable, script, "--workload", workload, "--steps", str(steps),
                            "--warmup", str(warmup)], capture_output=True, text=True, timeout=900)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference GPU run did not finish: {e}"}
    if r.returncode != 0:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"reference GPU run exited {r.returncode}: {tail[0][:300]}"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    return {"unavailable": "reference GPU run printed no result"}


def run_reference(args):
    world, rank, _local = _dist()
    if rank != 0:
        return 0
    from sparseconv import synthetic
    w = synthetic.make(args.workload, seed=0)
    ref_gpu = _reference_gpu(args.workload, max(3, min(args.steps, 10)), args.warmup)
    step, cores, sample = _cpu_sampler(w)
    for _ in range(args.warmup):
        step()
    times = [step() for _ in range(args.steps)]
    total = float(np.sum(times))
    value = w.num_voxels * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong" if args.shard == "batch" else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": _config(w),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu": ref_gpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline(w, budget_s: float = 10.0):
    step, cores, sample = _cpu_sampler(w)
    times = []
    t_start = time.perf_counter()
    while True:
        times.append(step())
        if time.perf_counter() - t_start > budget_s or len(times) >= 20:
            break
    t = float(np.median(times))
    return {"value": w.num_voxels / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": sample + f"; median of {len(times)} runs"}


def _batch_local(w, rank: int, world: int):
    """Rank r's part of the workload's batch: samples b with b % world == r, renumbered
    b // world, so the rank's grid holds only its own samples."""
    import dataclasses
    if world == 1:
        return w
    b = w.coords[:, 0]
    sel = (b % world) == rank
    coords = np.ascontiguousarray(w.coords[sel])
    coords[:, 0] //= world
    B = int(w.shape[0])
    local_b = len(range(rank, B, world))
    if local_b == 0:
        raise ValueError(f"batch {B} has no sample for rank {rank} of {world}")
    feats = w.feats[torch.from_numpy(np.nonzero(sel)[0])].contiguous()
    return dataclasses.replace(w, coords=coords, feats=feats, shape=(local_b,) + tuple(w.shape[1:]))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="indoor")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--shard", default="batch", choices=["batch", "replica"],
                    help="N>1: split the workload's batch over the ranks (strong scaling) or give "
                         "every rank its own full batch (weak scaling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="N=1: skip timing the reference's own GPU forward beside this line")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--e2e-streams", type=int, default=2, help="CUDA streams the end-to-end steps rotate over")
    ap.add_argument("--no-backward", action="store_true", help="skip the training-step (forward + backward) figure")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="run this many eager forwards of the workload and exit (a target for ncu)")
    ap.add_argument("--profile-backward", action="store_true",
                    help="with --profile-steps: each step is a forward + backward through autograd")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
        pg = torch.distributed.group.WORLD

    from sparseconv import _native, shards, synthetic
    from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d

    if args.shard == "batch":
        w_all = synthetic.make(args.workload, seed=0)
        w = _batch_local(w_all, rank, world)
    else:
        w_all = w = synthetic.make(args.workload, seed=rank)
    coords_h = torch.from_numpy(w.coords).pin_memory()
    feats_h = w.feats.pin_memory()
    coords = coords_h.to(dev)
    feats = feats_h.to(dev)
    weight = w.weight.to(dev)
    shape = torch.Size(w.shape)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def step():
        return sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)

    if args.profile_steps > 0:
        if args.profile_backward:
            f_req = feats.detach().clone().requires_grad_(True)
            w_req = weight.detach().clone().requires_grad_(True)
            for _ in range(args.profile_steps):
                o, _c = sparse_submanifold_conv3d(f_req, coords, shape, w_req, algorithm=Algorithm.IMPLICIT_GEMM)
                o.backward(torch.ones_like(o))
        else:
            for _ in range(args.profile_steps):
                step()
        torch.cuda.synchronize()
        _native.check_errors(dev)
        print("profile steps done:", args.workload, w.num_voxels, "voxels x", args.profile_steps)
        return 0

    for _ in range(args.warmup):
        out, cache = step()
    torch.cuda.synchronize()
    _native.check_errors(dev)
    nnz = int((cache.neighbor_map.view(torch.int32) >= 0).sum().item())
    fig = _alg_figures(w, nnz)

    # ---------------- device-resident timed region ----------------
    # One step is captured once into a CUDA graph (the whole forward: workspace memset,
    # insert, map, order, conv; nothing cached) and replayed K times, so host-side Python
    # does not sit between the kernels.
    K = args.steps
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()                                   # allocator warm-up on the capture stream
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        g_out, g_cache = step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if pg is not None:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    for i in range(K):
        flush.fill_(i)
        starts[i].record(stream)
        graph.replay()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if pg is not None:
        torch.distributed.barrier()
    clk = clocks.stop()
    _native.check_errors(dev)
    # the graph's output is the same forward's result: verify it once against the eager one
    ref_out, _ = step()
    torch.cuda.synchronize()
    if not torch.equal(ref_out, g_out):
        raise RuntimeError("graph-replayed forward differs from the eager forward")
    del graph
    step_ms = float(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))

    # Per-kernel device time, live: eager steps with the library's stage events on the launch
    # stream; each step follows a 256 MB flush, so the launches queue ahead of the GPU.
    ks = max(3, min(K, 50))
    _native.stage_timing(ks)
    for i in range(ks):
        flush.fill_(i)
        step()
    torch.cuda.synchronize()
    stage = _native.stage_times_ms()
    _native.stage_timing(0)
    max_ms = shards.max_over_ranks(step_ms)          # step time: the slowest rank
    voxels_all = shards.sum_over_ranks(w.num_voxels)  # whole-job work
    value = voxels_all * K / (max_ms / 1e3)

    # eager API steps (same work, host Python between the kernels), for reference
    ke = max(3, min(K, 50))
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e_s.record(stream)
    for _ in range(ke):
        step()
    e_e.record(stream)
    torch.cuda.synchronize()
    eager_ms = e_s.elapsed_time(e_e) / ke

    # ---------------- end-to-end through the public API from host buffers ----------------
    KE = args.e2e_steps or max(3, min(K, 50))
    out_h = torch.empty((w.num_voxels, int(w.weight.shape[0])), dtype=w.dtype).pin_memory()

    def e2e_step():
        c_d = coords_h.to(dev, non_blocking=True)
        f_d = feats_h.to(dev, non_blocking=True)
        o, _c = sparse_submanifold_conv3d(f_d, c_d, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)
        out_h.copy_(o, non_blocking=True)

    for _ in range(args.warmup):                 # untimed: allocator and pinned-copy warm-up
        e2e_step()
    if pg is not None:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(KE):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_serial_ms = shards.max_over_ranks(e0.elapsed_time(e1))
    e2e_serial = voxels_all * KE / (e2e_serial_ms / 1e3)

    # The same steps pipelined over CUDA streams (two by default: on the cube 548 M voxels/s vs
    # 540 with three and 457 with four, against a 573 M ceiling of the two copy directions
    # running together), as a host feeding batches would run them:
    # step i+1's host-to-device copies overlap step i's op and device-to-host copy (separate
    # copy engines). Every step still copies its own inputs in and its result out in the
    # timed region.
    NS = max(2, args.e2e_streams)
    e2e_streams = [torch.cuda.Stream(dev) for _ in range(NS)]
    outs_h = [out_h] + [torch.empty_like(out_h).pin_memory() for _ in range(NS - 1)]

    def e2e_step_on(j):
        s = e2e_streams[j % NS]
        with torch.cuda.stream(s):
            c_d = coords_h.to(dev, non_blocking=True)
            f_d = feats_h.to(dev, non_blocking=True)
            o, _c = sparse_submanifold_conv3d(f_d, c_d, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)
            outs_h[j % NS].copy_(o, non_blocking=True)

    for j in range(max(args.warmup, 2)):
        e2e_step_on(j)
    torch.cuda.synchronize()
    if pg is not None:
        torch.distributed.barrier()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for s in e2e_streams:
        s.wait_event(p0)
    for j in range(KE):
        e2e_step_on(j)
    for s in e2e_streams:
        done = torch.cuda.Event()
        done.record(s)
        stream.wait_event(done)
    p1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = shards.max_over_ranks(p0.elapsed_time(p1))
    e2e_value = voxels_all * KE / (e2e_ms / 1e3)
    _native.check_errors(dev)

    # ---------------- training step: map build + forward + backward through autograd ----------------
    # Eager (autograd runs between the kernels); every step builds its own map (and so its own
    # transposed map) and computes the input and weight gradients; L2 flushed between steps.
    train = None
    if not args.no_backward:
        f_req = feats.detach().clone().requires_grad_(True)
        w_req = weight.detach().clone().requires_grad_(True)
        g_out_t = torch.randn(out.shape, generator=torch.Generator().manual_seed(3)).to(out.dtype).to(dev)

        def train_step():
            o, _c = sparse_submanifold_conv3d(f_req, coords, shape, w_req, algorithm=Algorithm.IMPLICIT_GEMM)
            o.backward(g_out_t)

        for _ in range(args.warmup):
            train_step()
        KT = max(3, min(K, 20))
        t_s = [torch.cuda.Event(enable_timing=True) for _ in range(KT)]
        t_e = [torch.cuda.Event(enable_timing=True) for _ in range(KT)]
        torch.cuda.synchronize()
        if pg is not None:
            torch.distributed.barrier()
        for i in range(KT):
            flush.fill_(i)
            t_s[i].record(stream)
            train_step()
            t_e[i].record(stream)
        torch.cuda.synchronize()
        _native.check_errors(dev)
        train_ms = shards.max_over_ranks(float(sum(a.elapsed_time(b) for a, b in zip(t_s, t_e))))
        train = {"value": voxels_all * KT / (train_ms / 1e3), "unit": UNIT, "ms_per_step": train_ms / KT,
                 "steps": KT, "step": "eager map build + forward + backward (input and weight gradients) "
                                      "through autograd, fresh map each step"}

    if rank == 0:
        hbm, tc, peak_kind = _peaks()
        # dominant kernel by live stage time
        per_stage = {k: v for k, v in stage.items() if v[1] > 0}
        kern_bytes = {"conv": fig["conv_bytes"], "map": fig["map_bytes"],
                      "insert": fig["insert_bytes"], "order": fig["order_bytes"]}
        dom = max((k for k in per_stage if k in kern_bytes), key=lambda k: per_stage[k][0])
        dom_ms = per_stage[dom][0] / per_stage[dom][1]
        achieved = kern_bytes[dom] / (dom_ms / 1e3) / 1e9
        traffic = _traffic_per_launch(f"{args.workload}:{dom}")
        if traffic is not None and w.num_voxels != w_all.num_voxels:
            # the capture ran the whole workload; a rank of the batch split launches on its share
            # (DRAM bytes grow with the voxels a launch processes)
            traffic = int(round(traffic * w.num_voxels / w_all.num_voxels))
        # Second figure: the conv alone, as when a layer reuses the map (neighbour cache passed
        # back), from the conv kernel's own per-launch events in the eager steps above.
        cached_map = None
        if per_stage.get("conv", (0.0, 0))[0] > 0:
            conv_ms = per_stage["conv"][0] / max(per_stage["conv"][1], 1)
            cached_map = {"value": voxels_all / (conv_ms / 1e3), "unit": UNIT,
                          "conv_ms_per_step": conv_ms,
                          "step": "conv kernel alone on a reused map (per-launch CUDA events, L2 flushed)"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": max_ms / K, "higher_is_better": True,
            "scaling": "strong" if args.shard == "batch" else "weak", "vs_baseline": None,
            "dtype": str(w.dtype).replace("torch.", "").replace("float16", "f16").replace("bfloat16", "bf16").replace("float32", "f32"),
            "data": "synthetic",
            "config": _config(w_all),
            "details": {"parallelism": (f"batch split over {world} ranks (samples b % {world} == rank)"
                                        if args.shard == "batch" else f"{world} replicas, own batch each"),
                        "rank0_voxels": w.num_voxels, "nnz_per_voxel_rank0": nnz / w.num_voxels},
            "effective": {"tflops_alg": fig["flops_alg"] * world * K / (max_ms / 1e3) / 1e12,
                          "tflops_dense_equivalent": fig["flops_dense"] * world * K / (max_ms / 1e3) / 1e12},
            "stages_ms_per_step": {k: v[0] / max(v[1], 1) for k, v in per_stage.items()},
            "cached_map": cached_map,
            "step": "CUDA-graph replay of one full forward (map build + conv, no cached map)",
            "eager_api_ms_per_step": eager_ms,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind,
                         "algorithmic_bytes": kern_bytes[dom], "traffic": traffic},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": int(coords_h.numel() * 4 + feats_h.numel() * feats_h.element_size()),
                    "d2h_bytes_per_step": int(out_h.numel() * out_h.element_size()), "steps": KE,
                    "pipelined": f"{NS} CUDA streams: step i+1's H2D overlaps step i's op and D2H",
                    "serial_value": e2e_serial},
            "gpu_launches": _launches_per_step(w.num_voxels, w.kernel_size, w.shape) * K,
            "clocks": clk,
        }
        if train is not None:
            line["training_step"] = train
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        if world == 1 and not args.no_reference_gpu:
            # the reference's own GPU forward on the same workload and device (separate process)
            line["reference_gpu"] = _reference_gpu(args.workload, 5, 3)
        print(json.dumps(line), flush=True)
    if pg is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
