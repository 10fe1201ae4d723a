"""The fused Chamfer loss (mpo_chamfer_loss / mpo_chamfer_loss_backward) that
serves chamfer_distance without weights or normals, against the oracle's
loss and gradients (mps_pointops/chamfer.py:342-488 reduction rules) and
against the generic search + torch reduction path (forced with unit
weights)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mps_pointops.chamfer import chamfer_distance
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def clouds(b, p, q, seed, d=3):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, p, d, generator=g), torch.randn(b, q, d, generator=g)


def run(x, y, dev, **kw):
    xr = x.to(dev).requires_grad_()
    yr = y.to(dev).requires_grad_()
    loss, normals = chamfer_distance(xr, yr, **kw)
    assert normals is None
    (loss.sum() if loss.ndim else loss).backward()
    return loss.detach().cpu(), xr.grad.cpu(), yr.grad.cpu()


@pytest.mark.parametrize("p,q,d", [(600, 700, 3), (100, 90, 3), (530, 515, 7)])
@pytest.mark.parametrize("point", ["mean", "sum"])
@pytest.mark.parametrize("batch", [None, "sum", "mean"])
@pytest.mark.parametrize("single", [False, True])
def test_matches_generic_path(cuda_device, p, q, d, point, batch, single):
    x, y = clouds(3, p, q, seed=p + q + d, d=d)
    kw = dict(point_reduction=point, batch_reduction=batch, single_directional=single)
    fused = run(x, y, cuda_device, **kw)
    generic = run(x, y, cuda_device, weights=torch.ones(3, device=cuda_device), **kw)
    # The loss sums run in different orders; gradients add float atomics in
    # different orders: the Chamfer bar (rtol 1e-5).
    for a, b in zip(fused, generic):
        assert a.shape == b.shape
        np.testing.assert_allclose(a.numpy(), b.numpy(), rtol=1e-5, atol=1e-6)


def test_lengths_and_empty_clouds(cuda_device):
    x, y = clouds(4, 700, 650, seed=3)
    xl = torch.tensor([700, 0, 333, 1])
    yl = torch.tensor([650, 10, 0, 649])
    fused = run(x, y, cuda_device, x_lengths=xl.to(cuda_device), y_lengths=yl.to(cuda_device),
                batch_reduction=None)
    generic = run(x, y, cuda_device, x_lengths=xl.to(cuda_device), y_lengths=yl.to(cuda_device),
                  batch_reduction=None, weights=torch.ones(4, device=cuda_device))
    for a, b in zip(fused, generic):
        np.testing.assert_allclose(a.numpy(), b.numpy(), rtol=1e-5, atol=1e-6)


def test_config2_slice_against_oracle(cuda_device):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 8192, 3, generator=g)
    y = (x + 0.05 * torch.randn(2, 8192, 3, generator=g))[:, torch.randperm(8192, generator=g)]
    loss, gx, gy = run(x, y, cuda_device)
    want_loss, want_gx, want_gy, _, _ = O.chamfer_mean_loss_and_grad(x.numpy(), y.numpy())
    np.testing.assert_allclose(loss.item(), want_loss, rtol=1e-5)
    np.testing.assert_allclose(gx.numpy(), want_gx, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(gy.numpy(), want_gy, rtol=1e-5, atol=1e-9)


def test_reproducible(cuda_device):
    x, y = clouds(8, 2048, 2048, seed=9)
    a = run(x, y, cuda_device)[0]
    b = run(x, y, cuda_device)[0]
    assert torch.equal(a, b)
