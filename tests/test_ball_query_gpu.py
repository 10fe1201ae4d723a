"""Ball query on B200 vs the reference's CPU path (golden fixtures,
mps_pointops/reference.py:83-121) and the oracle: indices and squared
distances bit-exact.  Cases follow gamzerA/mps-pointops
tests/test_ball_query_mps.py and tests/test_ball_query_api.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mps_pointops
from conftest import golden
from mps_pointops import _native as N
from mps_pointops import compat
from mps_pointops._ball_query_cuda import _checked_radius_and_k, ball_query as core_ball_query
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_golden_cases(cuda_device):
    for name, c in golden("ball_query").items():
        d2, idx = mps_pointops.ball_query(torch.from_numpy(c["query"]).to(cuda_device),
                                          torch.from_numpy(c["ref"]).to(cuda_device),
                                          float(c["radius"]), int(c["K"]))
        np.testing.assert_array_equal(idx.cpu().numpy(), c["idx"], err_msg=name)
        np.testing.assert_array_equal(d2.cpu().numpy().view(np.int32),
                                      c["dist2"].view(np.int32), err_msg=name)


@pytest.mark.parametrize("K", [1, 7, 31, 32, 33, 64, 65])
def test_random_matches_oracle(cuda_device, K):
    g = torch.Generator().manual_seed(K)
    q, r = torch.rand(3, 257, 3, generator=g), torch.rand(3, 3001, 3, generator=g)
    want_d, want_i = O.ball_query(q.numpy(), r.numpy(), 0.12, K)
    d, i = mps_pointops.ball_query(q.to(cuda_device), r.to(cuda_device), 0.12, K)
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy().view(np.int32), want_d.view(np.int32))


def test_lengths_match_oracle(cuda_device):  # tests/test_ball_query_mps.py:58-73
    torch.manual_seed(9)
    q, p = torch.randn(2, 7, 3), torch.randn(2, 19, 3)
    ql, pl = torch.tensor([7, 4]), torch.tensor([19, 11])
    want_d, want_i = O.ball_query(q.numpy(), p.numpy(), 2.0, 5, ql.numpy(), pl.numpy())
    res = core_ball_query(q.to(cuda_device), p.to(cuda_device), radius=2.0, k=5,
                          query_lengths=ql.to(cuda_device), point_lengths=pl.to(cuda_device))
    np.testing.assert_array_equal(res.indices.cpu().numpy(), want_i)
    np.testing.assert_array_equal(res.distances.cpu().numpy(), want_d)
    with pytest.raises(ValueError, match="query_lengths"):
        core_ball_query(q.to(cuda_device), p.to(cuda_device), radius=1.0, k=1,
                        query_lengths=torch.tensor([8, 1], device=cuda_device))


@pytest.mark.parametrize("k", [1, 31, 32, 33, 65])
def test_every_output_slot_written(cuda_device, k):
    """Sentinel-prefilled buffers through the C ABI (tests/test_ball_query_mps.py:115-180)."""
    batch, qn, pn = 2, 9, 65
    q = torch.zeros((batch, qn, 3))
    p = torch.zeros((batch, pn, 3))
    for j in range(pn):
        p[:, j, 0] = 2.0 if j % 5 == 1 else (0.25 if j % 3 == 0 else 0.5)
    p[:, 31, 0], p[:, 32, 0] = float("nan"), float("inf")
    q[:, 2, 0], q[:, 4, 0] = 0.5, 20.0
    ql, pl = torch.tensor([9, 7]), torch.tensor([65, 49])
    want_d, want_i = O.ball_query(q.numpy(), p.numpy(), 1.0, k, ql.numpy(), pl.numpy())
    idx = torch.full((batch, qn, k), -777, dtype=torch.long, device=cuda_device)
    dist = torch.full((batch, qn, k), float("nan"), device=cuda_device)
    qc, pc, qlc, plc = (t.to(cuda_device) for t in (q, p, ql, pl))
    _, r2 = _checked_radius_and_k(1.0, k)
    N.check(N.lib().mpo_ball_query(N.ptr(qc), N.ptr(pc), N.ptr(qlc), N.ptr(plc), batch, qn, pn, k,
                                   r2, N.ptr(dist), N.ptr(idx), N.stream(cuda_device)), "bq")
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dist.cpu().numpy().view(np.int32), want_d.view(np.int32))


def test_pointnet2_padding_matches_oracle(cuda_device):
    c = golden("config1")
    xyz = torch.from_numpy(c["xyz"]).to(cuda_device)
    centres = torch.from_numpy(c["centres"]).to(cuda_device)
    got = compat.ball_query(0.2, 32, xyz, centres)
    assert got.dtype == torch.int32
    np.testing.assert_array_equal(got.cpu().numpy(), c["ball_query_idx"])
    xyz = torch.tensor([[[5.0, 0, 0], [0.1, 0, 0], [9, 9, 9], [0.2, 0, 0]]], device=cuda_device)
    new = torch.tensor([[[0.0, 0, 0], [50.0, 50, 50]]], device=cuda_device)
    assert compat.ball_query(0.5, 4, xyz, new).tolist() == [[[1, 3, 1, 1], [0, 0, 0, 0]]]


def test_empty_and_public_padding(cuda_device):  # tests/test_ball_query_api.py:20-34
    queries = torch.zeros((1, 2, 3), device=cuda_device)
    points = torch.tensor([[[0.25, 0.0, 0.0], [2.0, 0.0, 0.0]]], device=cuda_device)
    d, i = mps_pointops.ball_query(queries, points, 1.0, 3)
    assert i.cpu().tolist() == [[[0, -1, -1], [0, -1, -1]]]
    assert d.cpu().tolist() == [[[0.0625, 0.0, 0.0]] * 2]
    assert compat.ball_query(1.0, 3, points, queries).cpu().tolist() == [[[0, 0, 0], [0, 0, 0]]]
    base = torch.tensor([[[0.0, 0.0, 0.0], [2.0, 0.0, 0.0]]], device=cuda_device)
    res = core_ball_query(base, points[:, :0], radius=1.0, k=2)
    assert res.indices.cpu().tolist() == [[[-1, -1], [-1, -1]]]
    assert core_ball_query(base, points, radius=1.0, k=0).indices.shape == (1, 2, 0)
    assert core_ball_query(base[:, :0], points, radius=1.0, k=2).indices.shape == (1, 0, 2)
    d, i = mps_pointops.ball_query(base, points, 0.0, 3)
    assert (i == -1).all() and (d == 0).all()


def test_gradients(cuda_device):  # tests/test_ball_query_mps.py:493-562
    q = torch.tensor([[[0.0, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    p = torch.tensor([[[0.2, 0.0, 0.0], [0.5, 0.0, 0.0], [4.0, 0.0, 0.0]]], device=cuda_device,
                     requires_grad=True)
    res = core_ball_query(q, p, radius=1.0, k=3)
    assert res.indices.cpu().tolist() == [[[0, 1, -1]]]
    res.distances.backward(torch.tensor([[[2.0, 3.0, 99.0]]], device=cuda_device))
    torch.testing.assert_close(q.grad.cpu(), torch.tensor([[[-3.8, 0.0, 0.0]]]))
    torch.testing.assert_close(p.grad.cpu(), torch.tensor([[[0.8, 0, 0], [3.0, 0, 0], [0, 0, 0]]]))

    qs = torch.tensor([[[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    ps = torch.tensor([[[0.25, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    r = core_ball_query(qs, ps, radius=2.0, k=1)
    r.distances.backward(torch.tensor([[[2.0], [3.0]]], device=cuda_device))
    torch.testing.assert_close(qs.grad.cpu(), torch.tensor([[[-1.0, 0, 0], [4.5, 0, 0]]]))
    torch.testing.assert_close(ps.grad.cpu(), torch.tensor([[[-3.5, 0.0, 0.0]]]))

    q = torch.zeros((1, 1, 3), device=cuda_device, requires_grad=True)
    p = torch.tensor([[[0.25, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    loss = core_ball_query(q, p, radius=1.0, k=1).distances.sum()
    grad_q, grad_p = torch.autograd.grad(loss, (q, p), create_graph=True)
    torch.testing.assert_close(torch.autograd.grad(grad_q.sum(), q, retain_graph=True)[0],
                               torch.full_like(q, 2.0))
    torch.testing.assert_close(torch.autograd.grad(grad_p.sum(), p)[0], torch.full_like(p, 2.0))


def test_random_backward_matches_formula(cuda_device):
    g = torch.Generator().manual_seed(3)
    q = torch.rand(2, 100, 3, generator=g)
    p = torch.rand(2, 500, 3, generator=g)
    up = torch.randn(2, 100, 16, generator=g)
    qc = q.to(cuda_device).requires_grad_()
    pc = p.to(cuda_device).requires_grad_()
    res = core_ball_query(qc, pc, radius=0.2, k=16)
    res.distances.backward(up.to(cuda_device))
    idx = res.indices.cpu()
    valid = idx >= 0
    sel = p.gather(1, idx.clamp_min(0).reshape(2, -1, 1).expand(-1, -1, 3)).reshape(2, 100, 16, 3)
    contrib = torch.where(valid[..., None], 2 * up[..., None] * (q[:, :, None] - sel), 0.0)
    gq = contrib.sum(2)
    gp = torch.zeros_like(p).scatter_add_(1, idx.clamp_min(0).reshape(2, -1, 1).expand(-1, -1, 3),
                                          -contrib.reshape(2, -1, 3))
    torch.testing.assert_close(qc.grad.cpu(), gq, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(pc.grad.cpu(), gp, rtol=1e-5, atol=1e-6)


def test_float16_inputs(cuda_device):  # tests/test_ball_query_mps.py:565-583
    q = torch.tensor([[[0.0, 0.0, 0.0]]], device=cuda_device, dtype=torch.float16,
                     requires_grad=True)
    p = torch.tensor([[[0.25, 0.0, 0.0], [0.5, 0.0, 0.0]]], device=cuda_device,
                     dtype=torch.float16, requires_grad=True)
    res = core_ball_query(q, p, radius=1.0, k=2)
    assert res.distances.dtype == torch.float32
    assert res.indices.cpu().tolist() == [[[0, 1]]]
    res.distances.backward(torch.tensor([[[1.0, 2.0]]], device=cuda_device))
    torch.testing.assert_close(q.grad.cpu(), torch.tensor([[[-2.5, 0.0, 0.0]]], dtype=torch.float16))


def test_large_search_in_morton_order_matches_oracle(cuda_device):
    """Searches of >= 16384 queries over >= 65536 points run their queries in
    Morton order and scatter the results back: identical to the oracle, to
    the input-order run (a ragged query count keeps the input order) and
    with gradients in the callers' order.  Clustered clouds as BASELINE
    config 5, with far and non-finite queries."""
    g = torch.Generator().manual_seed(55)
    centres = torch.rand(16, 3, generator=g) * 10 - 5
    ref = (centres[torch.randint(16, (70000,), generator=g)] +
           0.5 * torch.randn(70000, 3, generator=g)).unsqueeze(0)
    q = (centres[torch.randint(16, (20000,), generator=g)] +
         0.5 * torch.randn(20000, 3, generator=g)).unsqueeze(0)
    q[0, 5] = torch.tensor([100.0, 100.0, 100.0])
    q[0, 77, 1] = float("nan")
    want_d, want_i = O.ball_query(q.numpy(), ref.numpy(), 0.3, 32)
    qc, rc = q.to(cuda_device), ref.to(cuda_device)
    d, i = mps_pointops.ball_query(qc, rc, 0.3, 32)
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)
    lengths = torch.tensor([20000], device=cuda_device)
    res = core_ball_query(qc, rc, query_lengths=lengths, radius=0.3, k=32)
    assert torch.equal(res.indices, i) and torch.equal(res.distances, d)
    qg = qc.clone().requires_grad_()
    rg = rc.clone().requires_grad_()
    dd, _ = mps_pointops.ball_query(qg, rg, 0.3, 32)
    dd.sum().backward()
    qh = qc.clone().requires_grad_()
    rh = rc.clone().requires_grad_()
    res = core_ball_query(qh, rh, query_lengths=lengths, radius=0.3, k=32)
    res.distances.sum().backward()
    torch.testing.assert_close(qg.grad, qh.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(rg.grad, rh.grad, rtol=1e-5, atol=1e-6)
