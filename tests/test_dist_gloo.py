"""Multi-GPU partitioning logic on CPU: world size 2 over gloo (127.0.0.1).

The native kernels need a GPU, so the local op is a CPU stand-in built on the
oracle (the reference's CPU algorithm); what is tested is the sharding, the
gather order and the loss all-reduce of mps_pointops.dist.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mps_pointops.dist import (all_gather_shards, ball_query_sharded, batch_sharded,
                               chamfer_distance_sharded, knn_query_sharded, shard_range)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_chamfer(x, y, batch_reduction="sum"):
    """Differentiable CPU stand-in: oracle indices, distances recomputed in torch."""
    from oracle import oracle as O
    _, ix = O.chamfer_nearest(x.detach().numpy(), y.detach().numpy())
    _, iy = O.chamfer_nearest(y.detach().numpy(), x.detach().numpy())
    ix, iy = torch.from_numpy(ix), torch.from_numpy(iy)
    dx = ((x - y.gather(1, ix[..., None].expand(-1, -1, 3))) ** 2).sum(-1)
    dy = ((y - x.gather(1, iy[..., None].expand(-1, -1, 3))) ** 2).sum(-1)
    per_cloud = dx.mean(1) + dy.mean(1)
    assert batch_reduction == "sum"
    return per_cloud.sum(), None


def oracle_knn(q, r, k):
    from oracle import oracle as O
    d, i = O.knn(q.numpy(), r.numpy(), k)
    return torch.from_numpy(d), torch.from_numpy(i)


def oracle_ball(q, r, radius, K):
    from oracle import oracle as O
    d, i = O.ball_query(q.numpy(), r.numpy(), radius, K)
    return torch.from_numpy(d), torch.from_numpy(i)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        g = torch.Generator().manual_seed(0)
        B = 5
        x, y = torch.randn(B, 40, 3, generator=g), torch.randn(B, 33, 3, generator=g)
        lo, hi = shard_range(B, rank, world)
        xl = x[lo:hi].clone().requires_grad_()
        yl = y[lo:hi].clone().requires_grad_()
        loss = chamfer_distance_sharded(xl, yl, B, local_fn=oracle_chamfer)
        loss.backward()
        out["loss"] = loss.item()
        out["gx"] = all_gather_shards(xl.grad, B).numpy()
        out["gy"] = all_gather_shards(yl.grad, B).numpy()
        # overlapped mode: backward on this rank's term, global value later
        xo = x[lo:hi].clone().requires_grad_()
        yo = y[lo:hi].clone().requires_grad_()
        local, pending = chamfer_distance_sharded(xo, yo, B, local_fn=oracle_chamfer,
                                                  overlap=True)
        local.backward()
        out["loss_overlap"] = pending.value().item()
        out["gx_overlap"] = all_gather_shards(xo.grad, B).numpy()
        out["gy_overlap"] = all_gather_shards(yo.grad, B).numpy()
        q, r = torch.randn(1, 37, 3, generator=g), torch.randn(1, 200, 3, generator=g)
        d, i = knn_query_sharded(q, r, 5, local_fn=oracle_knn)
        out["knn"] = (d.numpy(), i.numpy())
        d2, i2 = ball_query_sharded(q, r, 0.8, 6, local_fn=oracle_ball)
        out["ball"] = (d2.numpy(), i2.numpy())
        a = torch.arange(7 * 3, dtype=torch.float32).reshape(7, 3)
        out["batch"] = batch_sharded(lambda t: t * 2, a, batch_total=7).numpy()
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions():
    for total in (0, 1, 5, 8, 33):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.timeout(300)
def test_world2_gloo_matches_single_process():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
        assert p.exitcode == 0
    r0, r1 = results[0], results[1]

    g = torch.Generator().manual_seed(0)
    x, y = torch.randn(5, 40, 3, generator=g), torch.randn(5, 33, 3, generator=g)
    xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
    loss, _ = oracle_chamfer(xr, yr)
    (loss / 5).backward()
    for r in (r0, r1):
        for tag in ("", "_overlap"):
            np.testing.assert_allclose(r["loss" + tag], loss.item() / 5, rtol=1e-6)
            np.testing.assert_allclose(r["gx" + tag], xr.grad.numpy(), rtol=1e-6, atol=1e-7)
            np.testing.assert_allclose(r["gy" + tag], yr.grad.numpy(), rtol=1e-6, atol=1e-7)
    q, ref = torch.randn(1, 37, 3, generator=g), torch.randn(1, 200, 3, generator=g)
    wd, wi = oracle_knn(q, ref, 5)
    bd, bi = oracle_ball(q, ref, 0.8, 6)
    for r in (r0, r1):
        np.testing.assert_array_equal(r["knn"][1], wi.numpy())
        np.testing.assert_array_equal(r["knn"][0], wd.numpy())
        np.testing.assert_array_equal(r["ball"][1], bi.numpy())
        np.testing.assert_array_equal(r["ball"][0], bd.numpy())
        np.testing.assert_array_equal(r["batch"], np.arange(21, dtype=np.float32).reshape(7, 3) * 2)
