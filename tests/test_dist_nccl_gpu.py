"""Multi-GPU path over NCCL (runs only when 2+ GPUs are visible).

Two ranks, one per GPU: the Chamfer loss of a batch split across the ranks
(one all-reduce of the loss partials) and its gradients must equal the
single-GPU result, and the sharded kNN / ball query with a replicated
reference cloud (all-gather of the outputs) must equal the single-GPU call.
The same loss through the peer-memory all-reduce kernel (PeerLossReducer,
CUDA IPC mappings of each rank's exchange array) must carry the same bits on
both ranks, step after step.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(8)
    x = torch.randn(6, 2000, 3, generator=g)
    y = x + 0.05 * torch.randn(6, 2000, 3, generator=g)
    q = torch.randn(1, 3001, 3, generator=g)
    r = torch.randn(1, 5000, 3, generator=g)
    return x, y, q, r


def _worker(rank, world, port, results):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "mps-pointops_b200"))
    import torch.distributed as dist
    from mps_pointops.dist import (PeerLossReducer, all_gather_shards, ball_query_sharded,
                                   chamfer_distance_sharded, knn_query_sharded, shard_range)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        x, y, q, r = _inputs()
        lo, hi = shard_range(x.shape[0], rank, world)
        xl = x[lo:hi].to(dev).requires_grad_()
        yl = y[lo:hi].to(dev).requires_grad_()
        loss = chamfer_distance_sharded(xl, yl, x.shape[0])
        loss.backward()
        gx = all_gather_shards(xl.grad, x.shape[0])
        gy = all_gather_shards(yl.grad, x.shape[0])
        d, i = knn_query_sharded(q.to(dev), r.to(dev), 16)
        bd, bi = ball_query_sharded(q.to(dev), r.to(dev), 0.3, 32)
        torch.cuda.synchronize()
        red = PeerLossReducer(timeout_s=20.0)
        peer = []
        for step in range(4):
            xo = x[lo:hi].to(dev).requires_grad_()
            yo = (y[lo:hi] * (1.0 + 0.01 * step)).to(dev).requires_grad_()
            local, pending = chamfer_distance_sharded(xo, yo, x.shape[0], overlap=True,
                                                      reducer=red)
            local.backward()
            peer.append(pending.value().item())
        pgx = all_gather_shards(xo.grad, x.shape[0])
        red.check()
        red.close()
        results[rank] = {"loss": loss.item(), "gx": gx.cpu(), "gy": gy.cpu(), "knn": (d.cpu(), i.cpu()),
                         "ball": (bd.cpu(), bi.cpu()), "peer": peer, "peer_gx": pgx.cpu()}
    finally:
        dist.destroy_process_group()


def test_two_rank_nccl_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import mps_pointops
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    x, y, q, r = _inputs()
    xc = x.cuda().requires_grad_()
    yc = y.cuda().requires_grad_()
    loss, _ = mps_pointops.chamfer_distance(xc, yc)
    loss.backward()
    d, i = mps_pointops.knn(q.cuda(), r.cuda(), 16)
    bd, bi = mps_pointops.ball_query(q.cuda(), r.cuda(), 0.3, 32)
    assert results[0]["peer"] == results[1]["peer"]          # same bits on both ranks
    for step, got in enumerate(results[0]["peer"]):
        xs = x.cuda().requires_grad_()
        ys = (y * (1.0 + 0.01 * step)).cuda().requires_grad_()
        want, _ = mps_pointops.chamfer_distance(xs, ys)
        want.backward()
        assert abs(got - want.item()) <= 1e-5 * abs(want.item())
    for rank in (0, 1):
        torch.testing.assert_close(results[rank]["peer_gx"], xs.grad.cpu(), rtol=1e-5, atol=1e-8)
    for rank in (0, 1):
        res = results[rank]
        assert abs(res["loss"] - loss.item()) <= 1e-5 * abs(loss.item())
        torch.testing.assert_close(res["gx"], xc.grad.cpu(), rtol=1e-5, atol=1e-8)
        torch.testing.assert_close(res["gy"], yc.grad.cpu(), rtol=1e-5, atol=1e-8)
        assert torch.equal(res["knn"][1], i.cpu()) and torch.equal(res["knn"][0], d.cpu())
        assert torch.equal(res["ball"][1], bi.cpu()) and torch.equal(res["ball"][0], bd.cpu())
