#!/usr/bin/env python
"""Benchmark of the B200 point-op hot path (one JSON line on rank 0).

Workload (the metric's single-GPU configuration):
squared-L2 Chamfer distance forward + backward on B = 32 pairs of clouds of
N = M = 8192 fp32 points per GPU, x ~ N(0,1)^3 and y = x + N(0,0.05)^3 in a
per-cloud random permutation, mean/mean reduction, gradients for both clouds.
A step is one `chamfer_distance(x, y)` + `loss.backward()` through the public
API.  Metric: Chamfer pairs/s = B * N * M per step / step time (whole job).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs one process per GPU under torchrun (NCCL over NVLink): each rank
owns 32 clouds (weak scaling) and the only collective is the all-reduce of the
Chamfer loss partials, which runs on NCCL's stream during the backward.  `--impl reference` times the reference's CPU algorithm
(the C restatement in oracle/, all host threads) on the same workload; under
torchrun only rank 0 runs it.

Also reported: `e2e` (the same step with the inputs copied from pinned host
memory and the loss read back every step), the live CUDA-event time of the
dominant kernel against its roofline, the CPU baseline, SM clocks sampled
during the timed region, the native kernel launch count, and secondary lines:
BASELINE config 1 (FPS + ball query + kNN, clouds/s; 8 clouds per GPU), config 4
(feature kNN, queries/s; 16 clouds per GPU), config 1 with its 8 clouds split
over the GPUs (strong scaling) and config 5 with its 2^20 queries split over
the GPUs (strong scaling), their all-gathers timed apart, and the latency of
the loss all-reduce.
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "mps-pointops_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B_PER_GPU, NPTS, D = 32, 8192, 3
FLOPS_PER_PAIR = 8  # 3 sub + 3 mul + 2 add, each rounded (no FMA)
METRIC = "Chamfer pairs/sec"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="chamfer_config2",
                    choices=["chamfer_config2", "ssg_config1_ops", "fps_config3", "fps_large",
                             "feature_knn_config4", "knn_config5", "ball_query_config5",
                             "flat_ops", "sa_grouping_config1", "chamfer_variants_config2",
                             "config5_grid"],
                    help="single-GPU measurement of one BASELINE config (the default is the "
                         "headline line; the others print their own JSON line and are used "
                         "for the per-kernel profiles)")
    ap.add_argument("--queries", type=int, default=131072,
                    help="config 5: queries per GPU (1M queries / 8 GPUs)")
    ap.add_argument("--loss-reducer", choices=["peer", "nccl"], default="peer",
                    help="N > 1: all-reduce of the Chamfer loss partials through the library's "
                         "peer-memory kernel (default) or NCCL")
    return ap.parse_args()


def chamfer_inputs(batch: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, NPTS, D, generator=g)
    y = x + 0.05 * torch.randn(batch, NPTS, D, generator=g)
    y = torch.stack([y[b, torch.randperm(NPTS, generator=g)] for b in range(batch)])
    return x.contiguous(), y.contiguous()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    QUERY = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self, begin: bool):
        if begin:
            self.t0 = time.monotonic()
        else:
            self.t1 = time.monotonic()

    def stop(self, bus_ids: set[str]) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 10]
        mine = [r for r in rows if r[1].strip().lower()[-12:] in bus_ids] or rows
        sm = [float(r[2]) for r in mine if r[2].strip().replace(".", "").isdigit()]
        mx = [float(r[3]) for r in mine if r[3].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in mine for i in range(4)
                          if r[6 + i].strip().lower() == "active"})
        if not sm:
            return None
        busy = [s for s in sm if s > 0.5 * max(sm)]
        return {"sm_mhz": statistics.median(busy or sm), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm),
                "gpus": len({r[1].strip().lower() for r in mine})}


# ------------------------------------------------------------------ distributed
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ B200 arm
def chamfer_step(x, y, world, group_batch, reducer=None):
    from mps_pointops.chamfer import chamfer_distance
    from mps_pointops.dist import chamfer_distance_sharded
    xr = x.detach().requires_grad_()
    yr = y.detach().requires_grad_()
    if world > 1:
        # The loss all-reduce (peer-memory kernel, or NCCL without a reducer)
        # runs on a side stream during the backward; the step ends once its
        # global loss is in (the compute stream waits on it).
        local, pending = chamfer_distance_sharded(xr, yr, group_batch, overlap=True,
                                                  reducer=reducer)
        local.backward()
        return pending.value()
    loss, _ = chamfer_distance(xr, yr)
    loss.backward()
    return loss


def timed_steps(fn, steps: int, flush: torch.Tensor | None) -> list[float]:
    """Per-step CUDA-event times (ms); the L2 flush between steps is untimed."""
    times = []
    s = torch.cuda.current_stream()
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        times.append((a, b))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def ssg_secondary(steps: int, warmup: int, world: int, rank: int) -> dict:
    """compat FPS 1024 -> gather -> ball query (0.2, 32) ->
    kNN k=16 on 8 uniform clouds of 4096 points per GPU; clouds/s."""
    from mps_pointops import compat, knn
    g = torch.Generator().manual_seed(1000 * rank)
    xyz = torch.rand(8, 4096, 3, generator=g).cuda()

    def step():
        idx = compat.furthest_point_sample(xyz, 1024)
        centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx)
        centres = centres.transpose(1, 2).contiguous()
        compat.ball_query(0.2, 32, xyz, centres)
        knn(centres, xyz, 16)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ms = statistics.mean(timed_steps(step, steps, None))
    ms = max_over_ranks(ms, world)
    return {"metric": "clouds/sec for FPS+ball_query+kNN (B=8,N=4096)",
            "value": 8 * world / (ms / 1e3), "unit": "clouds/s", "ms_per_step": ms,
            "config": {"workload": "ssg_config1", "global_batch": 8 * world, "points": 4096}}


def _split_ms(step_fn, steps: int, warmup: int, world: int) -> tuple[float, float]:
    """Per-step time and the part after the compute (the collective), both
    from CUDA events on the current stream, means over `steps`, max over
    ranks.  step_fn(mark) must call mark() between its compute and its
    collective."""
    for _ in range(warmup):
        step_fn(lambda: None)
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.current_stream()
    rec = []
    for _ in range(steps):
        a, m, b = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(s)
        step_fn(lambda: m.record(s))
        b.record(s)
        rec.append((a, m, b))
    torch.cuda.synchronize()
    total = statistics.mean(a.elapsed_time(b) for a, _, b in rec)
    coll = statistics.mean(m.elapsed_time(b) for _, m, b in rec)
    return max_over_ranks(total, world), max_over_ranks(coll, world)


def ssg_strong_secondary(steps: int, warmup: int, world: int, rank: int) -> dict:
    """BASELINE config 1 with its 8 clouds split over the ranks (strong
    scaling: 8 / world clouds per GPU): compat FPS 1024 -> gather -> ball
    query (0.2, 32) -> kNN k=16, then (world > 1) the FPS, ball-query and kNN
    outputs all-gathered so every rank holds the batch's results."""
    from mps_pointops import compat, knn
    from mps_pointops.dist import all_gather_shards, shard_range
    g = torch.Generator().manual_seed(0)
    xyz_all = torch.rand(8, 4096, 3, generator=g)
    lo, hi = shard_range(8, rank, world)
    xyz = xyz_all[lo:hi].contiguous().cuda()

    def step(mark):
        idx = compat.furthest_point_sample(xyz, 1024)
        centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx)
        centres = centres.transpose(1, 2).contiguous()
        bq = compat.ball_query(0.2, 32, xyz, centres)
        d, i = knn(centres, xyz, 16)
        mark()
        if world > 1:
            for t in (idx, bq, d, i):
                all_gather_shards(t, 8)

    ms, coll = _split_ms(step, steps, warmup, world)
    return {"metric": "clouds/sec for FPS+ball_query+kNN (B=8,N=4096)",
            "value": 8 / (ms / 1e3), "unit": "clouds/s", "ms_per_step": ms,
            "all_gather_ms_per_step": coll, "scaling": "strong",
            "config": {"workload": "ssg_config1_strong", "global_batch": 8,
                       "clouds_per_gpu": hi - lo, "points": 4096,
                       "collective": "all_gather_into_tensor of FPS idx, ball-query idx, kNN "
                                     "dist and idx (NCCL)" if world > 1 else "none"}}


def config5_secondary(steps: int, warmup: int, world: int, rank: int) -> dict:
    """BASELINE config 5 sharded as specified: 2^20 queries split contiguously
    over the ranks against the replicated 2^20-point reference cloud (built
    identically on every rank), brute-force kNN k=16 and ball query r=0.3,
    K=32 through the public API, then (world > 1) the four outputs
    all-gathered along the query axis.  Queries/s of the whole job."""
    from mps_pointops import ball_query, knn
    from mps_pointops.dist import all_gather_shards, shard_range
    nq = 1 << 20
    ref = _config5_cloud(6, 1 << 20).cuda()
    lo, hi = shard_range(nq, rank, world)
    q = _config5_cloud(7, nq)[:, lo:hi].contiguous().cuda()

    def step(mark):
        kd, ki = knn(q, ref, 16)
        bd, bi = ball_query(q, ref, 0.3, 32)
        mark()
        if world > 1:
            for t in (kd, ki, bd, bi):
                all_gather_shards(t, nq, dim=1)

    ms, coll = _split_ms(step, steps, warmup, world)
    return {"metric": "config 5 queries/sec (kNN k=16 + ball query r=0.3 K=32, 2^20 x 2^20)",
            "value": nq / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
            "all_gather_ms_per_step": coll, "scaling": "strong",
            "config": {"workload": "config5_sharded", "queries": nq, "refs": 1 << 20,
                       "queries_per_gpu": hi - lo, "search": "brute force (public API)",
                       "collective": "all_gather_into_tensor of kNN dist/idx and ball-query "
                                     "dist/idx along the query axis (NCCL)"
                                     if world > 1 else "none"}}


def loss_all_reduce_us(world: int, reducer=None, reps: int = 50) -> float | None:
    """Latency of the Chamfer step's collective alone: a 4-byte all-reduce
    through NCCL, or through ``reducer`` (the peer-memory kernel), ``reps``
    times back to back.  A ~2.5 ms spin kernel goes first so that the host
    has enqueued every reduction before the first runs: the time is the
    device's, not the Python launch rate's.  CUDA events, mean, max over
    ranks."""
    if world == 1:
        return None
    import torch.distributed as dist
    t = torch.ones(1, device="cuda")

    def one():
        if reducer is None:
            dist.all_reduce(t)
            return None
        return reducer.reduce(t)

    for _ in range(5):
        p = one()
        if p is not None:
            p.value()
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(5_000_000)
    a.record(s)
    last = None
    for _ in range(reps):
        last = one()
    if last is not None:
        last.value()
    b.record(s)
    torch.cuda.synchronize()
    return max_over_ranks(a.elapsed_time(b) * 1e3 / reps, world)


def feature_knn_secondary(steps: int, warmup: int, world: int, rank: int,
                          flush: torch.Tensor) -> dict:
    """knn(f, f, 20) on 16 clouds of 4096 unit-norm D=64
    features per GPU (tensor-core candidates + exact fp32 re-rank); queries/s.
    L2 flushed between timed steps (the inputs are 16 MB)."""
    from mps_pointops import knn
    g = torch.Generator().manual_seed(5 + 1000 * rank)
    f = torch.nn.functional.normalize(torch.randn(16, 4096, 64, generator=g), dim=-1).cuda()

    def step():
        knn(f, f, 20)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(statistics.mean(timed_steps(step, steps, flush)), world)
    return {"metric": "feature kNN queries/sec (B=16,N=4096,D=64,k=20)",
            "value": 16 * 4096 * world / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
            "config": {"workload": "feature_knn_config4", "global_batch": 16 * world,
                       "points": 4096, "dims": 64, "k": 20,
                       "l2": "flushed between timed steps"}}


def _event_ms(fn, steps: int, warmup: int, flush: torch.Tensor | None) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    return statistics.median(timed_steps(fn, steps, flush))


def ssg_config1_ops(steps: int, warmup: int) -> dict:
    """BASELINE config 1, op by op (B=8 uniform clouds of 4096 points): compat
    FPS 1024, compat ball query (0.2, 32), kNN k=16 centres -> points, three_nn
    points -> centres, three_interpolate of 64 N(0,1) features (forward and
    backward); per-op median ms with the L2 flushed between steps."""
    from mps_pointops import compat, knn, three_interpolate, three_nn
    g = torch.Generator().manual_seed(0)
    xyz = torch.rand(8, 4096, 3, generator=g).cuda()
    feats = torch.randn(8, 64, 1024, generator=torch.Generator().manual_seed(1)).cuda()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    idx = compat.furthest_point_sample(xyz, 1024)
    centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx)
    centres = centres.transpose(1, 2).contiguous()
    dist, nidx = three_nn(xyz, centres)
    w = 1.0 / (dist + 1e-8)
    w = w / w.sum(dim=2, keepdim=True)
    fg = feats.clone().requires_grad_()
    out = three_interpolate(fg, nidx, w)
    gout = torch.randn_like(out)
    ops = {
        "fps": lambda: compat.furthest_point_sample(xyz, 1024),
        "ball_query": lambda: compat.ball_query(0.2, 32, xyz, centres),
        "knn": lambda: knn(centres, xyz, 16),
        "three_nn": lambda: three_nn(xyz, centres),
        "three_interpolate_fwd": lambda: three_interpolate(feats, nidx, w),
        "three_interpolate_fwd_bwd": lambda: torch.autograd.grad(
            three_interpolate(fg, nidx, w), fg, gout),
    }
    res = {name: _event_ms(fn, steps, warmup, flush) for name, fn in ops.items()}
    return {"workload": "ssg_config1_ops", "unit": "ms (median, public API, L2 flushed)",
            "per_op_ms": res, "clouds": 8, "points": 4096, "centres": 1024}


def fps_config3(steps: int, warmup: int) -> dict:
    """FPS of 65,536 centres from one cloud of 2^20 points
    on the unit sphere with N(0, 0.01) radial jitter, start 0."""
    from mps_pointops import furthest_point_sample
    g = torch.Generator().manual_seed(4)
    p = torch.randn(1, 1 << 20, 3, generator=g)
    p = p / p.norm(dim=-1, keepdim=True)
    p = p * (1 + 0.01 * torch.randn(1, 1 << 20, 1, generator=g))
    p = p.cuda()
    ms = _event_ms(lambda: furthest_point_sample(p, 65536), max(steps, 1), max(warmup, 1), None)
    stream_bytes = 65536 * (1 << 20) * 20
    return {"workload": "fps_config3", "ms": ms, "ns_per_step": ms * 1e6 / 65536,
            "samples_per_s": 65536 / (ms / 1e3),
            "streaming_model_GBps": stream_bytes / (ms / 1e3) / 1e9,
            "note": "streaming model: 20 B per point-step (12 B xyz + 4 B read + 4 B write of "
                    "min_d2); the kernel keeps the cloud in registers, so this is the rate an "
                    "HBM-streaming design would need, not DRAM traffic"}


def fps_large(steps: int, warmup: int) -> dict:
    """FPS beyond 8192 points per SM: 4096 samples from jittered-sphere clouds
    of 1.5 M points (registers + shared-memory tier) and 4 M points
    (registers + shared memory + workspace tier), start 0; ns per step."""
    from mps_pointops import furthest_point_sample
    res = {"workload": "fps_large", "unit": "ns per FPS step (median of CUDA-event runs)"}
    for n, seed in ((1_500_000, 41), (4_000_000, 42)):
        g = torch.Generator().manual_seed(seed)
        p = torch.randn(1, n, 3, generator=g)
        p = p / p.norm(dim=-1, keepdim=True)
        p = (p * (1 + 0.01 * torch.randn(1, n, 1, generator=g))).cuda()
        ms = _event_ms(lambda: furthest_point_sample(p, 4096), max(steps, 1), max(warmup, 1),
                       None)
        res[f"n{n}"] = {"ms": ms, "ns_per_step": ms * 1e6 / 4096, "samples": 4096}
    return res


def _config5_cloud(seed: int, n: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    centres = torch.rand(64, 3, generator=torch.Generator().manual_seed(6)) * 20 - 10
    labels = torch.randint(64, (n,), generator=g)
    return (centres[labels] + 0.5 * torch.randn(n, 3, generator=g)).unsqueeze(0)


def config5(kind: str, queries: int, steps: int, warmup: int) -> dict:
    """BASELINE config 5 on one GPU: reference cloud of 2^20 points from 64
    Gaussian clusters (centres U[-10,10]^3, sigma 0.5), `queries` query points
    from the same distribution (the per-GPU shard of the 2^20 queries):
    knn k=16 or ball_query r=0.3, K=32."""
    from mps_pointops import ball_query, knn
    ref = _config5_cloud(6, 1 << 20).cuda()
    q = _config5_cloud(7, 1 << 20)[:, :queries].contiguous().cuda()
    if kind == "knn":
        fn = lambda: knn(q, ref, 16)  # noqa: E731
    else:
        fn = lambda: ball_query(q, ref, 0.3, 32)  # noqa: E731
    ms = _event_ms(fn, max(steps, 1), max(warmup, 1), None)
    return {"workload": f"{kind}_config5", "queries": queries, "refs": 1 << 20, "ms": ms,
            "queries_per_s": queries / (ms / 1e3),
            "pairs_per_s_brute_force": queries * (1 << 20) / (ms / 1e3)}


def _flat_public_fixture(n: int):
    """The fixture of the reference's public flat benchmark
    (bench/bench_flat_public.py:43-61): two randomly ordered clouds with batch
    ids 0 and 2 (batch_size 3) of 3n/4 and n/4 points whose coordinates are
    integers in [-128, 128] / 16, and n/32 queries taken from the clouds at a
    regular stride."""
    g = torch.Generator().manual_seed(7102 + n)
    xs, ys, bx, by = [], [], [], []
    for bid, length, nq in ((0, 3 * n // 4, 3 * n // 128), (2, n // 4, n // 128)):
        cloud = torch.randint(-128, 129, (length, 3), generator=g).float() / 16
        xs.append(cloud)
        ys.append(cloud[torch.arange(nq) * length // nq])
        bx.append(torch.full((length,), bid, dtype=torch.long))
        by.append(torch.full((nq,), bid, dtype=torch.long))
    return tuple(torch.cat(t) for t in (xs, ys, bx, by))


def _flat_scale_fixture(clouds: int, seed: int):
    """A PyG-scale ragged batch: `clouds` clouds of U[4096, 28672) points in
    the unit cube (about 2^20 points for 64 clouds), queries = every 16th
    point of each cloud."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(4096, 28672, (clouds,), generator=g).tolist()
    x = torch.rand(sum(lengths), 3, generator=g)
    bx = torch.repeat_interleave(torch.arange(clouds), torch.tensor(lengths))
    ptr = [0]
    for n in lengths:
        ptr.append(ptr[-1] + n)
    rows = torch.cat([torch.arange(ptr[b], ptr[b + 1], 16) for b in range(clouds)])
    return x, x[rows].contiguous(), bx, bx[rows].contiguous(), lengths


def flat_ops(steps: int, warmup: int) -> dict:
    """The flat torch_cluster API (mps_pointops/flat.py) on two workloads.
    (1) The reference's public flat benchmark (bench/bench_flat_public.py):
    N = 1024 and 4096, fps(ratio 1/64), knn(k 16), radius(2.0, 16), timed as
    there -- public call, inputs resident, synchronized host wall time, median.
    (2) A PyG-scale ragged batch (64 clouds, ~2^20 points, ~65k queries):
    fps(ratio 1/16), knn(k 16), radius(0.05, 32) through the public calls
    (host wall) and the search kernels alone (CUDA events), with the FP32
    roofline of the kNN pair work; the oracle times the same searches on a
    bounded query sample for the CPU baseline."""
    from mps_pointops import flat
    from mps_pointops import _native as N
    res = {"workload": "flat_ops"}

    def wall_ms(fn, reps):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        t = []
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter_ns()
            fn()
            torch.cuda.synchronize()
            t.append((time.perf_counter_ns() - t0) / 1e6)
        return statistics.median(t)

    public = {}
    for n in (1024, 4096):
        x, y, bx, by = (t.cuda() for t in _flat_public_fixture(n))
        public[str(n)] = {
            "fps": wall_ms(lambda: flat.fps(x, bx, ratio=1 / 64, random_start=False,
                                            batch_size=3), steps),
            "knn": wall_ms(lambda: flat.knn(x, y, 16, bx, by, batch_size=3), steps),
            "radius": wall_ms(lambda: flat.radius(x, y, 2.0, bx, by, max_num_neighbors=16,
                                                  batch_size=3), steps),
        }
    res["public_median_ms"] = public

    x, y, bx, by, lengths = _flat_scale_fixture(64, 11)
    xc, yc, bxc, byc = x.cuda(), y.cuda(), bx.cuda(), by.cuda()
    ptr_x, ptr_y = flat._pair_ptrs(xc, yc, bxc, byc, None)
    pairs = sum(n * len(range(0, n, 16)) for n in lengths)
    scale = {"clouds": 64, "points": len(x), "queries": len(y),
             "pairs_per_search": pairs}
    scale["public_ms"] = {
        "fps": wall_ms(lambda: flat.fps(xc, bxc, ratio=1 / 16, random_start=False), 3),
        "knn": wall_ms(lambda: flat.knn(xc, yc, 16, bxc, byc), steps),
        "radius": wall_ms(lambda: flat.radius(xc, yc, 0.05, bxc, byc, max_num_neighbors=32),
                          steps),
    }
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    knn_ms = _event_ms(lambda: flat.knn_indices(xc, yc, ptr_x, ptr_y, 16), steps, warmup, flush)
    rad_ms = _event_ms(lambda: flat.radius_indices(xc, yc, ptr_x, ptr_y, 0.05, 32), steps,
                       warmup, flush)
    mhz = _sm_max_mhz()
    peak = 128 * torch.cuda.get_device_properties(0).multi_processor_count * mhz * 1e6 / 1e12
    achieved = pairs * FLOPS_PER_PAIR / (knn_ms / 1e3) / 1e12
    scale["search_ms"] = {"knn": knn_ms, "radius": rad_ms}
    scale["knn_roofline"] = {"bound": "fp32", "achieved": achieved, "peak": peak,
                             "unit": "TFLOP/s", "frac": achieved / peak,
                             "note": "8 rounded FP32 ops per pair; peak = 128 lane-ops/SM/clk "
                                     "at the max SM clock"}
    res["scale"] = scale

    # CPU baseline: the oracle's flat search on the first 2048 queries.
    from oracle import oracle as O
    xn, yn = x.numpy(), y.numpy()
    pxn, pyn = ptr_x.cpu().numpy(), ptr_y.cpu().numpy()
    sub = 2048
    pys = np.minimum(pyn, sub)
    t0 = time.perf_counter()
    O.flat_knn_indices(xn, yn[:sub], pxn, pys, 16)
    sec = time.perf_counter() - t0
    sub_pairs = sum(int(pxn[b + 1] - pxn[b]) * int(pys[b + 1] - pys[b])
                    for b in range(len(pxn) - 1))
    res["cpu_baseline"] = {"value": sub / sec, "unit": "kNN queries/s", "cores": O.threads(),
                           "kind": "port", "pairs_per_s": sub_pairs / sec,
                           "sample": f"{sub} of {len(y)} queries of the scale batch, k=16"}
    res["gpu_knn_queries_per_s"] = len(y) / (knn_ms / 1e3)
    res["launches"] = N.launch_count()
    return res


def sa_grouping_config1(steps: int, warmup: int) -> dict:
    """SA grouping at BASELINE config 1 sizes (8 clouds of 4096 points, 1024
    centres, r 0.2, 32 samples, 64 feature channels), forward + backward:
    (1) the reference's composition (tests/test_pointnet2_e2e.py:40-44) with
    its torch gather grouping (compat.py:68-73), (2) the same composition on
    the native grouping kernel, (3) the fused query_and_group.  CUDA events,
    L2 flushed between steps; HBM roofline of the fused forward kernel."""
    from mps_pointops import compat, grouping
    from mps_pointops import _native as N
    from mps_pointops._ball_query_cuda import _checked_radius_and_k
    g = torch.Generator().manual_seed(0)
    xyz = torch.rand(8, 4096, 3, generator=g).cuda()
    feats = torch.randn(8, 64, 4096, generator=g).cuda()
    idx0 = compat.furthest_point_sample(xyz, 1024)
    centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx0)
    centres = centres.transpose(1, 2).contiguous()
    B, P, S, C = 8, 1024, 32, 64
    gout = torch.randn(B, 3 + C, P, S, generator=g).cuda()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def torch_group(f, i):
        flat_i = i.long().reshape(B, 1, P * S).expand(B, f.shape[1], -1)
        return f.gather(2, flat_i).reshape(B, f.shape[1], P, S)

    def composed(group):
        def run(backward):
            x = xyz.clone().requires_grad_(backward)
            q = centres.clone().requires_grad_(backward)
            f = feats.clone().requires_grad_(backward)
            nb = compat.ball_query(0.2, S, x, q)
            gx = group(x.transpose(1, 2).contiguous(), nb) - q.transpose(1, 2).unsqueeze(-1)
            out = torch.cat((gx, group(f, nb)), dim=1)
            if backward:
                out.backward(gout)
            return out
        return run

    def fused(backward):
        x = xyz.clone().requires_grad_(backward)
        q = centres.clone().requires_grad_(backward)
        f = feats.clone().requires_grad_(backward)
        out, _ = grouping.query_and_group(x, q, f, 0.2, S)
        if backward:
            out.backward(gout)
        return out

    arms = {"reference_torch_gather": composed(torch_group),
            "native_unfused": composed(compat.grouping_operation), "fused": fused}
    res = {"workload": "sa_grouping_config1", "unit": "ms (median, CUDA events, L2 flushed)",
           "shape": {"clouds": B, "points": 4096, "centres": P, "nsample": S, "channels": C}}
    for name, fn in arms.items():
        res[name] = {"fwd": _event_ms(lambda: fn(False), steps, warmup, flush),
                     "fwd_bwd": _event_ms(lambda: fn(True), steps, warmup, flush)}
    # The sampling step: compat FPS then gather_operation, vs the fused FPS.
    res["sampling"] = {
        "fps_then_gather": _event_ms(lambda: compat.gather_operation(
            xyz.transpose(1, 2).contiguous(), compat.furthest_point_sample(xyz, P)),
            steps, warmup, flush),
        "fused_sample_and_gather": _event_ms(lambda: grouping.sample_and_gather(xyz, P), steps,
                                             warmup, flush)}
    # The fused forward kernel alone (events on the launching stream).
    idx = torch.empty((B, P, S), dtype=torch.int32, device="cuda")
    out = torch.empty((B, 3 + C, P, S), device="cuda")
    lib = N.lib()
    _, r2 = _checked_radius_and_k(0.2, S)

    ws_bytes = int(lib.mpo_query_and_group_workspace_bytes(B, 4096, P, S, C))
    ws = N.workspace(ws_bytes, xyz.device)

    def kernel_call():
        N.check(lib.mpo_query_and_group(N.ptr(xyz), N.ptr(centres), N.ptr(feats), B, 4096, P, S, C,
                                        r2, 1, N.ptr(idx), N.ptr(out), N.ptr(ws), ws_bytes,
                                        N.stream(xyz.device)), "query_and_group")
    q_ms = _event_ms(kernel_call, steps, warmup, flush)
    algo = out.numel() * 4 + idx.numel() * 4 + feats.numel() * 4 + xyz.numel() * 4 \
        + centres.numel() * 4
    peak = _measured_hbm_gbs()
    res["fused_forward_call"] = {"ms": q_ms, "algorithmic_bytes": algo,
                                 "achieved_GBps": algo / (q_ms / 1e3) / 1e9, "peak_GBps": peak,
                                 "frac": algo / (q_ms / 1e3) / 1e9 / peak,
                                 "note": "ball query + grouping launches; bytes = output + "
                                         "indices written, features + xyz + centres read once "
                                         "(the transposed copy of the features adds 2 x 8.4 MB "
                                         "not counted)"}
    return res


def chamfer_variants_config2(steps: int, warmup: int) -> dict:
    """Chamfer forward + backward at BASELINE config 2 (32 x 8192^2, D = 3) for
    the calls outside the headline's fused path: L1 (norm=1), per-cloud
    weights (squared L2, the general path), and normals; pairs/s, CUDA
    events, L2 flushed between steps."""
    from mps_pointops.chamfer import chamfer_distance
    x, y = (t.cuda() for t in chamfer_inputs(B_PER_GPU, seed=2))
    g = torch.Generator().manual_seed(3)
    xn = torch.nn.functional.normalize(torch.randn(x.shape, generator=g), dim=-1).cuda()
    yn = torch.nn.functional.normalize(torch.randn(y.shape, generator=g), dim=-1).cuda()
    w = torch.rand(B_PER_GPU, generator=g).cuda() + 0.5
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def step(**kw):
        xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
        loss, nl = chamfer_distance(xr, yr, **kw)
        (loss + (nl if nl is not None else 0)).backward()

    arms = {"l2_fused": {}, "l1": {"norm": 1}, "l2_weights": {"weights": w},
            "l2_normals": {"x_normals": xn, "y_normals": yn}}
    pairs = B_PER_GPU * NPTS * NPTS
    res = {"workload": "chamfer_variants_config2", "unit": "ms (median fwd+bwd)",
           "pairs_per_step": pairs}
    for name, kw in arms.items():
        ms = _event_ms(lambda: step(**kw), steps, warmup, flush)
        res[name] = {"ms": ms, "pairs_per_s": pairs / (ms / 1e3)}
    return res


def _measured_hbm_gbs() -> float:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"])
    except Exception:  # noqa: BLE001
        return 6650.0


def _sm_max_mhz() -> float:
    try:
        outp = subprocess.run(["nvidia-smi", "--query-gpu=clocks.max.sm", "--format=csv,noheader,nounits",
                               "-i", "0"], capture_output=True, text=True, timeout=20).stdout
        return float(outp.strip().splitlines()[0])
    except Exception:  # noqa: BLE001
        return 1965.0


def config5_grid(queries: int, steps: int, warmup: int) -> dict:
    """BASELINE config 5 through the grid-accelerated SpatialIndex (exact,
    same results as the scan; a different amount of work, reported on its
    own): build time, kNN k=16 and ball query r=0.3 K=32 for `queries`
    queries against the 2^20-point clustered cloud."""
    from mps_pointops.spatial import SpatialIndex
    ref = _config5_cloud(6, 1 << 20)[0].contiguous().cuda()
    q = _config5_cloud(7, 1 << 20)[0, :queries].contiguous().cuda()
    build = []
    for _ in range(max(steps, 1) + 1):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        index = SpatialIndex(ref, backend="grid")
        index._get_grid()
        torch.cuda.synchronize()
        build.append((time.perf_counter() - t0) * 1e3)
    grid = index._get_grid()
    knn_ms = _event_ms(lambda: index.knn(q, 16), max(steps, 1), max(warmup, 1), None)
    bq_ms = _event_ms(lambda: index.ball_query(q, 0.3, 32), max(steps, 1), max(warmup, 1), None)
    return {"workload": "config5_grid", "queries": queries, "refs": 1 << 20,
            "grid": {"dims": list(grid.dims), "cell_size": grid.h, "n_extra": grid.n_extra},
            "build_ms_host_wall": statistics.median(build[1:]),
            "knn_k16_ms": knn_ms, "knn_queries_per_s": queries / (knn_ms / 1e3),
            "ball_query_r0.3_K32_ms": bq_ms, "ball_query_queries_per_s": queries / (bq_ms / 1e3),
            "note": "exact: equal to the brute-force results; build includes the sampled "
                    "8-NN cell-size estimate and one host read of the box"}


def cpu_baseline_sample(max_seconds: float = 15.0) -> dict:
    """The oracle (C restatement of the reference's CPU Chamfer search,
    mps_pointops/chamfer.py:161-251) on the bench inputs, forward + backward,
    all host threads, over as many clouds as fit in ~max_seconds."""
    from oracle import oracle as O
    x, y = chamfer_inputs(B_PER_GPU, seed=2)
    xn, yn = x.numpy(), y.numpy()
    t0 = time.perf_counter()
    done = 0
    while done < B_PER_GPU:
        O.chamfer_mean_loss_and_grad(xn[done:done + 1], yn[done:done + 1])
        done += 1
        if time.perf_counter() - t0 > max_seconds:
            break
    sec = time.perf_counter() - t0
    return {"value": done * NPTS * NPTS / sec, "unit": "pairs/s", "cores": O.threads(),
            "kind": "port",
            "sample": f"{done} of {B_PER_GPU} cloud pairs (8192 x 8192), forward+backward, "
                      f"{sec:.1f} s"}


def e2e_chamfer(xh, yh, dev, world, group_batch, steps, reducer=None):
    """End-to-end Chamfer steps through the public API from pinned host inputs.

    Pipelined (the first number): step i+1's inputs are copied host->device
    on a copy stream while step i computes (two device buffers, events
    guard reuse); every step's loss is copied device->host into pinned
    memory on the compute stream, and the host reads step i-1's loss after
    enqueueing step i.  The timed region runs from before the first input
    copy to the completion of the last loss copy (CUDA events).  Sequential
    (the second number): copy, step and loss.item() one after another.
    Returns (pipelined ms per step, sequential ms per step), max over ranks."""
    comp = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    bufs = [(torch.empty(xh.shape, device=dev), torch.empty(yh.shape, device=dev))
            for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    host_loss = torch.empty(steps + 4, dtype=torch.float32).pin_memory()
    ready = [torch.cuda.Event() for _ in range(steps + 4)]

    def issue_copy(i):
        k = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[k])      # step i - 2 is done with buffer k
            bufs[k][0].copy_(xh, non_blocking=True)
            bufs[k][1].copy_(yh, non_blocking=True)
            copied[k].record(copy_stream)

    def run_step(i):
        k = i % 2
        comp.wait_event(copied[k])
        loss = chamfer_step(bufs[k][0], bufs[k][1], world, group_batch, reducer)
        host_loss[i].copy_(loss.detach(), non_blocking=True)
        # Buffer k is released after the loss read-back is queued: the next
        # input upload into it then starts behind the 4-byte copy instead of
        # holding it back on the copy engines for the length of its 6.3 MB.
        consumed[k].record(comp)
        ready[i].record(comp)

    def pipelined(n):
        total = 0.0
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            run_step(i)
            if i >= 1:
                ready[i - 1].synchronize()
                total += float(host_loss[i - 1])
        ready[n - 1].synchronize()
        total += float(host_loss[n - 1])
        if not math.isfinite(total):
            raise RuntimeError("non-finite Chamfer loss in the end-to-end loop")

    pipelined(2)
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    copy_stream.wait_event(a)
    pipelined(steps)
    b.record(comp)
    torch.cuda.synchronize()
    pipe_ms = max_over_ranks(a.elapsed_time(b) / steps, world)

    def sequential_step():
        xd = xh.to(dev, non_blocking=True)
        yd = yh.to(dev, non_blocking=True)
        return float(chamfer_step(xd, yd, world, group_batch, reducer).item())

    sequential_step()
    barrier(world)
    torch.cuda.synchronize()
    a.record(comp)
    for _ in range(steps):
        sequential_step()
    b.record(comp)
    torch.cuda.synchronize()
    seq_ms = max_over_ranks(a.elapsed_time(b) / steps, world)
    return pipe_ms, seq_ms


def run_b200(args, world, rank, local):
    from mps_pointops import _native as N
    from mps_pointops.chamfer import chamfer_distance  # noqa: F401  (import before timing)
    dev = torch.device("cuda", local)
    N.lib()
    group_batch = B_PER_GPU * world
    x_cpu, y_cpu = chamfer_inputs(B_PER_GPU, seed=2 + 1000 * rank)
    x, y = x_cpu.to(dev), y_cpu.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    props = torch.cuda.get_device_properties(dev)
    bus = {str(getattr(props, "pci_bus_id", "")).lower()[-12:]}
    reducer = None
    if world > 1 and args.loss_reducer == "peer":
        from mps_pointops.dist import PeerLossReducer
        reducer = PeerLossReducer()
    out = _run_b200_steps(args, world, rank, dev, props, bus, x, y, x_cpu, y_cpu, flush,
                          group_batch, reducer)
    if reducer is not None:
        reducer.close()      # collective: every rank got here without an error
    return out


def _run_b200_steps(args, world, rank, dev, props, bus, x, y, x_cpu, y_cpu, flush, group_batch,
                    reducer):
    from mps_pointops import _native as N
    for _ in range(max(args.warmup, 3)):
        chamfer_step(x, y, world, group_batch, reducer)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        buses: list = [None] * world
        dist.all_gather_object(buses, sorted(bus))
        bus = set().union(*(set(b) for b in buses))
    barrier(world)
    # One sampler (rank 0, single node) records the clocks of every rank's GPU.
    clocks = ClockSampler() if rank == 0 else None
    if clocks:
        clocks.start()
    time.sleep(0.3)
    launches0 = N.launch_count()
    if clocks:
        clocks.mark(True)
    with N.KernelTimer("chamfer_nearest") as ktimer:
        step_ms = timed_steps(lambda: chamfer_step(x, y, world, group_batch, reducer), args.steps,
                              flush)
    if clocks:
        clocks.mark(False)
    launches = N.launch_count() - launches0
    barrier(world)
    clock_info = clocks.stop(bus) if clocks else None
    ms = max_over_ranks(statistics.mean(step_ms), world)
    kernel_ms = max_over_ranks(ktimer.mean_ms(), world)
    pairs_per_step = group_batch * NPTS * NPTS
    value = pairs_per_step / (ms / 1e3)

    # e2e: public API with pinned host inputs, H2D every step, loss read back.
    xh, yh = x_cpu.pin_memory(), y_cpu.pin_memory()
    e2e_ms, e2e_seq_ms = e2e_chamfer(xh, yh, dev, world, group_batch, args.steps, reducer)

    secondary = None if args.no_secondary else ssg_secondary(args.steps, args.warmup, world, rank)
    fknn = None if args.no_secondary else feature_knn_secondary(args.steps, max(args.warmup, 3),
                                                                world, rank, flush)
    strong = None if args.no_secondary else ssg_strong_secondary(min(args.steps, 20),
                                                                 max(args.warmup, 3), world, rank)
    c5 = None if args.no_secondary else config5_secondary(min(args.steps, 3), 1, world, rank)
    ar_us = loss_all_reduce_us(world, reducer)
    nccl_us = loss_all_reduce_us(world) if reducer is not None else ar_us
    if reducer is not None:
        reducer.check()

    # Roofline of the dominant kernel: the nearest search (8 separately rounded
    # flops per unique pair) against the FP32 pipe: 128 rounded fp32 ops per
    # SM per clock (a packed f32x2 op holds the pipe for two cycles, so
    # packing saves issue slots but does not raise this bound).
    local_pairs = B_PER_GPU * NPTS * NPTS
    achieved = local_pairs * FLOPS_PER_PAIR / (kernel_ms / 1e3) / 1e12
    sm_max = (clock_info or {}).get("sm_max_mhz") or 1965.0
    peak = 128 * props.multi_processor_count * sm_max * 1e6 / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "chamfer_sym3_config2.md"
    if tfile.exists():
        for line in tfile.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = float(line.split(":", 1)[1])
    out = {
        "metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic, seeded: x ~ N(0,1)^3, y = x + N(0,0.05)^3, per-cloud permutation",
        "config": {"workload": "chamfer_config2_fwd_bwd", "global_batch": group_batch,
                   "points_per_cloud": NPTS, "dims": D, "reduction": "mean/mean",
                   "parallelism": f"dp{world}",
                   "l2": "flushed between timed steps (256 MiB write, untimed)"},
        "e2e": {"value": pairs_per_step / (e2e_ms / 1e3), "unit": "pairs/s",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(x_cpu.numel() * 4 + y_cpu.numel() * 4),
                "d2h_bytes_per_step": 4,
                "sequential_ms_per_step": e2e_seq_ms,
                "note": "public chamfer_distance + backward; each step copies its inputs from "
                        "pinned host memory (a second stream, overlapping the previous step) "
                        "and its loss back to pinned host memory, read by the host one step "
                        "later; sequential_ms_per_step: copy, step, loss.item() in series"},
        "gpu_launches": int(max_over_ranks(float(launches), world)),
        "roofline": {"kernel": "chamfer_sym3_kernel + finalize (mpo_chamfer_nearest, both "
                               "directions in one pass)",
                     "bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       "launch of this kernel in the ncu capture summarised in "
                                       "profiles/chamfer_sym3_config2.md (same workload), not "
                                       "measured in this run",
                     "kernel_ms": kernel_ms,
                     "work": f"{FLOPS_PER_PAIR} flop x {local_pairs} unique pairs per launch",
                     "peak_source": "nominal FP32 pipe rate for separately rounded add/sub/mul: "
                                    f"128 lanes x {props.multi_processor_count} SMs x "
                                    f"{sm_max:.0f} MHz (MEASURED_PEAKS.json has no FP32 figure; "
                                    "a packed fma.rn.f32x2 probe on this pool sustained one "
                                    "instruction per 2 cycles per SM sub-partition, i.e. the "
                                    "same 128 lane-ops per SM per clock)"},
        "clocks": clock_info,
    }
    if secondary:
        out["secondary"] = secondary
    if fknn:
        out["secondary_feature_knn"] = fknn
    if strong:
        out["secondary_config1_strong"] = strong
    if c5:
        out["secondary_config5"] = c5
    if ar_us is not None:
        out["collectives"] = {
            "chamfer_loss_all_reduce_us": ar_us,
            "loss_reducer": "peer-memory kernel (mpo_allreduce_sum_f32_p2p)" if reducer
                            is not None else "NCCL all_reduce",
            "nccl_all_reduce_us": nccl_us,
            "note": "the Chamfer step's only collective (4-byte all-reduce of the loss "
                    "partials) runs on a side stream during the backward; these are latencies "
                    "alone (mean of 50 back to back, enqueued behind a spin kernel so that the "
                    "host launch rate does not bound them; max over ranks)"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_sample()
    return out


# ------------------------------------------------------------------ reference arm
def run_reference(args) -> dict:
    """The reference's CPU algorithm (oracle/ C restatement of
    mps_pointops/chamfer.py:161-251 + the mean reductions) on the bench
    workload, every host thread; each step is one cloud pair of the batch."""
    from oracle import oracle as O
    O.build()
    x, y = chamfer_inputs(B_PER_GPU, seed=2)
    xn, yn = x.numpy(), y.numpy()
    for i in range(min(args.warmup, 1)):
        O.chamfer_mean_loss_and_grad(xn[i:i + 1], yn[i:i + 1])
    steps = max(1, min(args.steps, 8))
    t0 = time.perf_counter()
    for i in range(steps):
        O.chamfer_mean_loss_and_grad(xn[i % B_PER_GPU:i % B_PER_GPU + 1],
                                     yn[i % B_PER_GPU:i % B_PER_GPU + 1])
    sec = (time.perf_counter() - t0) / steps
    value = NPTS * NPTS / sec
    return {"metric": METRIC, "value": value, "unit": "pairs/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic, seeded (same inputs as the b200 arm)", "impl": "reference",
            "config": {"workload": "chamfer_config2_fwd_bwd",
                       "global_batch": B_PER_GPU * max(1, args.gpus),
                       "points_per_cloud": NPTS, "dims": D, "reduction": "mean/mean",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": O.threads(),
                             "kind": "port",
                             "sample": f"{steps} steps of 1 cloud pair (8192 x 8192), "
                                       "forward+backward, C restatement of the reference's "
                                       "CPU path"},
            "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    args = parse_args()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return
    if args.workload != "chamfer_config2":
        torch.cuda.set_device(0)
        steps, warmup = min(args.steps, 20), max(args.warmup, 1)
        if args.workload == "ssg_config1_ops":
            out = ssg_config1_ops(steps, max(warmup, 3))
        elif args.workload == "fps_config3":
            out = fps_config3(min(steps, 3), 1)
        elif args.workload == "fps_large":
            out = fps_large(min(steps, 5), 1)
        elif args.workload == "config5_grid":
            out = config5_grid(args.queries, min(steps, 5), 1)
        elif args.workload == "chamfer_variants_config2":
            out = chamfer_variants_config2(min(steps, 10), max(warmup, 3))
        elif args.workload == "sa_grouping_config1":
            out = sa_grouping_config1(steps, max(warmup, 3))
        elif args.workload == "flat_ops":
            out = flat_ops(steps, max(warmup, 3))
        elif args.workload == "feature_knn_config4":
            flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
            out = feature_knn_secondary(steps, max(warmup, 3), 1, 0, flush)
        else:
            out = config5(args.workload.split("_config")[0], args.queries, min(steps, 5), 1)
        print(json.dumps(out), flush=True)
        return
    world, rank, local = init_dist()
    try:
        out = run_b200(args, world, rank, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
