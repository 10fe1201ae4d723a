"""Grid-accelerated SpatialIndex (mpo_grid_build / mpo_grid_knn /
mpo_grid_ball_query) vs the full scan (the brute-force kernels that
tests/test_knn_gpu.py and tests/test_ball_query_gpu.py pin to the oracle) and
the oracle itself: indices and distances bit-exact.  Counterpart of the
reference's SpatialIndex (mps_pointops/spatial.py:76-264,
tests/test_spatial_public.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mps_pointops import ball_query, knn
from mps_pointops.spatial import SpatialIndex
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def clustered(n, seed, clusters=64, spread=10.0, sigma=0.5):
    g = torch.Generator().manual_seed(seed)
    centres = torch.rand(clusters, 3, generator=g) * 2 * spread - spread
    labels = torch.randint(clusters, (n,), generator=g)
    return centres[labels] + sigma * torch.randn(n, 3, generator=g)


def scan_knn(points, query, k):
    d, i = knn(query.unsqueeze(0), points.unsqueeze(0), k)
    return d[0], i[0]


def scan_bq(points, query, r, K):
    d, i = ball_query(query.unsqueeze(0), points.unsqueeze(0), r, K)
    return d[0], i[0]


@pytest.mark.parametrize("k", [1, 8, 16, 32])
def test_grid_knn_matches_scan_clustered(cuda_device, k):
    pts = clustered(200_000, 1).to(cuda_device)
    q = clustered(6000, 2).to(cuda_device)
    q[:100] = q[:100] * 3.0          # some queries far outside the cloud's box
    index = SpatialIndex(pts, backend="grid")
    d, i = index.knn(q, k)
    wd, wi = scan_knn(pts, q, k)
    assert torch.equal(i, wi)
    assert torch.equal(d, wd)


def test_grid_knn_uniform_ties_duplicates_and_nonfinite(cuda_device):
    g = torch.Generator().manual_seed(3)
    pts = torch.randint(0, 40, (100_000, 3), generator=g).float() * 0.25   # heavy ties
    pts[5] = torch.tensor([float("nan"), 0.0, 0.0])
    pts[6] = torch.tensor([float("inf"), 1.0, 1.0])
    pts[7] = torch.tensor([0.0, -float("inf"), 1.0])
    q = torch.randint(0, 40, (3000, 3), generator=g).float() * 0.25 + 0.1
    q[0] = torch.tensor([float("nan"), 0.0, 0.0])
    q[1] = torch.tensor([float("inf"), 0.0, 0.0])
    q[2] = pts[100]
    pts_c, q_c = pts.to(cuda_device), q.to(cuda_device)
    index = SpatialIndex(pts_c, backend="grid")
    for k in (4, 16, 32):
        d, i = index.knn(q_c, k)
        wd, wi = scan_knn(pts_c, q_c, k)
        assert torch.equal(i, wi), k
        assert torch.equal(d, wd), k
    # and against the oracle on a slice
    d, i = index.knn(q_c[:300], 16)
    od, oi = O.knn(q[:300].unsqueeze(0).numpy(), pts.unsqueeze(0).numpy(), 16)
    np.testing.assert_array_equal(i.cpu().numpy(), oi[0])
    np.testing.assert_array_equal(d.cpu().numpy(), od[0])


def test_grid_knn_small_cloud_and_user_grid(cuda_device):
    g = torch.Generator().manual_seed(4)
    pts = torch.rand(40, 3, generator=g).to(cuda_device)
    q = torch.rand(50, 3, generator=g).to(cuda_device) * 2 - 0.5
    for kw in ({}, {"cell_size": 0.01}, {"cell_size": 5.0},
               {"origin": torch.full((3,), 0.5, device=cuda_device), "cell_size": 0.1}):
        index = SpatialIndex(pts, backend="grid", **kw)
        d, i = index.knn(q, 32)
        wd, wi = scan_knn(pts, q, 32)
        assert torch.equal(i, wi), kw
        assert torch.equal(d, wd), kw


@pytest.mark.parametrize("r,K", [(0.05, 8), (0.3, 32), (0.3, 1), (2.0, 32), (100.0, 16)])
def test_grid_ball_query_matches_scan(cuda_device, r, K):
    pts = clustered(150_000, 5).to(cuda_device)
    q = clustered(4000, 6).to(cuda_device)
    q[:50] += 30.0
    index = SpatialIndex(pts, backend="grid")
    d, i = index.ball_query(q, r, K)
    wd, wi = scan_bq(pts, q, r, K)
    assert torch.equal(i, wi)
    assert torch.equal(d, wd)
    # and against the oracle on a slice (including the far queries)
    od, oi = O.ball_query(q[:300].unsqueeze(0).cpu().numpy(), pts.unsqueeze(0).cpu().numpy(), r, K)
    np.testing.assert_array_equal(i[:300].cpu().numpy(), oi[0])
    np.testing.assert_array_equal(d[:300].cpu().numpy().view(np.int32), od[0].view(np.int32))


def test_grid_ball_query_gradients_and_auto(cuda_device):
    pts = clustered(70_000, 7).to(cuda_device).requires_grad_()
    q = clustered(500, 8).to(cuda_device).requires_grad_()
    index = SpatialIndex(pts)                      # auto: 70K points -> grid
    assert index._selected_backend(16, None) == "grid"
    d, i = index.ball_query(q, 0.4, 16)
    g = torch.randn(d.shape, device=cuda_device)
    (d * g).sum().backward()
    gq, gp = q.grad.clone(), pts.grad.clone()
    q.grad = None
    pts.grad = None
    wd, wi = scan_bq(pts, q, 0.4, 16)
    assert torch.equal(i, wi)
    (wd * g).sum().backward()
    torch.testing.assert_close(gq, q.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gp, pts.grad, rtol=1e-5, atol=1e-6)
    assert SpatialIndex(pts[:1000].detach())._selected_backend(16, None) == "scan"


def test_mutation_and_argument_checks(cuda_device):
    pts = torch.rand(100, 3, device=cuda_device)
    index = SpatialIndex(pts, backend="bvh")
    index.knn(pts[:3], 4)
    pts.add_(1.0)
    with pytest.raises(ValueError, match="points changed"):
        index.knn(pts[:3], 4)
    with pytest.raises(ValueError, match="k <= 32"):
        SpatialIndex(pts, backend="grid").knn(pts[:3], 33)


def test_config5_scale_grid_equals_scan(cuda_device):
    """BASELINE config 5 cloud (2^20 points, 64 Gaussian clusters): 16K
    queries, kNN k=16 and ball query r=0.3 K=32, grid == scan."""
    g = torch.Generator().manual_seed(6)
    centres = torch.rand(64, 3, generator=torch.Generator().manual_seed(6)) * 20 - 10
    labels = torch.randint(64, (1 << 20,), generator=g)
    pts = (centres[labels] + 0.5 * torch.randn(1 << 20, 3, generator=g)).to(cuda_device)
    q = clustered(16384, 9).to(cuda_device)
    index = SpatialIndex(pts, backend="grid")
    d, i = index.knn(q, 16)
    wd, wi = scan_knn(pts, q, 16)
    assert torch.equal(i, wi) and torch.equal(d, wd)
    d, i = index.ball_query(q, 0.3, 32)
    wd, wi = scan_bq(pts, q, 0.3, 32)
    assert torch.equal(i, wi) and torch.equal(d, wd)
