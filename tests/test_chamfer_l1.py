"""L1 Chamfer (norm=1) vs the reference's CPU path (tests/golden/chamfer_l1.npz,
made by mps_pointops/chamfer.py with norm=1): the oracle is pinned on the CPU;
the CUDA path (mpo_chamfer_nearest_l1 / mpo_chamfer_l1_backward) is checked
on the GPU.  Nearest indices bit-exact; losses and gradients rtol 1e-5 (the
reference reduces in torch's order)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops.chamfer import chamfer_distance
from oracle import oracle as O

CASES = {
    "plain": lambda i: dict(),
    "lengths": lambda i: dict(x_lengths=i["x_lengths"], y_lengths=i["y_lengths"]),
    "weights_sum": lambda i: dict(x_lengths=i["x_lengths"], y_lengths=i["y_lengths"],
                                  weights=i["weights"], batch_reduction="sum"),
    "normals": lambda i: dict(x_lengths=i["x_lengths"], y_lengths=i["y_lengths"],
                              x_normals=i["x_normals"], y_normals=i["y_normals"]),
    "single_max": lambda i: dict(single_directional=True, point_reduction="max",
                                 batch_reduction=None),
    "d5": lambda i: dict(),
}


def test_oracle_l1_nearest_matches_reference():
    z = golden("chamfer_l1")
    inp = z["inputs"]
    for name in ("plain", "lengths", "normals"):
        c = z[name]
        kw = CASES[name](inp)
        B, P, _ = c["x"].shape
        lx = kw.get("x_lengths", np.full(B, P))
        ly = kw.get("y_lengths", np.full(B, c["y"].shape[1]))
        _, idx = O.chamfer_nearest(c["x"], c["y"], lx, ly, norm=1)
        valid = np.arange(P)[None] < np.asarray(lx)[:, None]
        np.testing.assert_array_equal(np.where(valid, idx, -1), np.where(valid, c["idx_x"], -1),
                                      err_msg=name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_l1_chamfer_matches_reference(cuda_device, name):
    z = golden("chamfer_l1")
    c = z[name]
    kw = {k: torch.from_numpy(v).to(cuda_device) for k, v in CASES[name](z["inputs"]).items()
          if isinstance(v, np.ndarray)}
    kw.update({k: v for k, v in CASES[name](z["inputs"]).items() if not isinstance(v, np.ndarray)})
    x = torch.from_numpy(c["x"]).to(cuda_device).requires_grad_()
    y = torch.from_numpy(c["y"]).to(cuda_device).requires_grad_()
    loss, nl = chamfer_distance(x, y, norm=1, **kw)
    np.testing.assert_allclose(loss.detach().cpu().numpy(), c["loss"], rtol=1e-5, atol=1e-6)
    if "normal_loss" in c:
        np.testing.assert_allclose(nl.cpu().numpy(), c["normal_loss"], rtol=1e-5, atol=1e-6)
    loss.sum().backward()
    np.testing.assert_allclose(x.grad.cpu().numpy(), c["grad_x"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(y.grad.cpu().numpy(), c["grad_y"], rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_l1_nearest_against_oracle_at_scale(cuda_device):
    from mps_pointops import _native as N
    g = torch.Generator().manual_seed(9)
    x, y = torch.randn(4, 3000, 3, generator=g), torch.randn(4, 2500, 3, generator=g)
    lx, ly = torch.tensor([3000, 10, 2999, 0]), torch.tensor([2500, 2500, 1, 7])
    B, P, D = x.shape
    Q = y.shape[1]
    xc, yc, lxc, lyc = (t.to(cuda_device) for t in (x, y, lx, ly))
    dx = torch.empty(B, P, device=cuda_device)
    ix = torch.empty(B, P, dtype=torch.long, device=cuda_device)
    dy = torch.empty(B, Q, device=cuda_device)
    iy = torch.empty(B, Q, dtype=torch.long, device=cuda_device)
    N.check(N.lib().mpo_chamfer_nearest_l1(N.ptr(xc), N.ptr(yc), N.ptr(lxc), N.ptr(lyc), B, P, Q, D,
                                           1, N.ptr(dx), N.ptr(ix), N.ptr(dy), N.ptr(iy),
                                           N.stream(cuda_device)), "l1")
    want_d, want_i = O.chamfer_nearest(x.numpy(), y.numpy(), lx.numpy(), ly.numpy(), norm=1)
    np.testing.assert_array_equal(ix.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dx.cpu().numpy(), want_d)
    want_d, want_i = O.chamfer_nearest(y.numpy(), x.numpy(), ly.numpy(), lx.numpy(), norm=1)
    np.testing.assert_array_equal(iy.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dy.cpu().numpy(), want_d)
    gdx = torch.randn(B, P, generator=g)
    gdy = torch.randn(B, Q, generator=g)
    gx = torch.empty_like(xc)
    gy = torch.empty_like(yc)
    gdx_c, gdy_c = gdx.to(cuda_device), gdy.to(cuda_device)  # kept alive for the launch
    N.check(N.lib().mpo_chamfer_l1_backward(N.ptr(xc), N.ptr(yc), B, P, Q, D, N.ptr(ix),
                                            N.ptr(gdx_c), N.ptr(iy), N.ptr(gdy_c), N.ptr(gx),
                                            N.ptr(gy), N.stream(cuda_device)), "l1 bwd")
    wx, wy = O.chamfer_l1_grads(x.numpy(), y.numpy(), ix.cpu().numpy(), iy.cpu().numpy(),
                                gdx.numpy(), gdy.numpy())
    np.testing.assert_allclose(gx.cpu().numpy(), wx, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gy.cpu().numpy(), wy, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_l1_symmetric_path_ties_and_single_direction(cuda_device):
    """Both directions at once (P, Q >= 512, D = 3: the symmetric tile kernel
    with the L1 metric, keys held in the idx outputs) on an integer lattice,
    where equal L1 distances are everywhere and the lowest index must win;
    the one-direction call takes the per-direction kernel."""
    from mps_pointops import _native as N
    g = torch.Generator().manual_seed(10)
    x = torch.randint(0, 5, (2, 1500, 3), generator=g).float()
    y = torch.randint(0, 5, (2, 1300, 3), generator=g).float()
    B, P, D = x.shape
    Q = y.shape[1]
    xc, yc = x.to(cuda_device), y.to(cuda_device)
    for bidirectional in (1, 0):
        dx = torch.full((B, P), 7.0, device=cuda_device)
        ix = torch.full((B, P), 7, dtype=torch.long, device=cuda_device)
        dy = torch.full((B, Q), 7.0, device=cuda_device)
        iy = torch.full((B, Q), 7, dtype=torch.long, device=cuda_device)
        N.check(N.lib().mpo_chamfer_nearest_l1(N.ptr(xc), N.ptr(yc), None, None, B, P, Q, D,
                                               bidirectional, N.ptr(dx), N.ptr(ix), N.ptr(dy),
                                               N.ptr(iy), N.stream(cuda_device)), "l1")
        want_d, want_i = O.chamfer_nearest(x.numpy(), y.numpy(), norm=1)
        np.testing.assert_array_equal(ix.cpu().numpy(), want_i)
        np.testing.assert_array_equal(dx.cpu().numpy(), want_d)
        if bidirectional:
            want_d, want_i = O.chamfer_nearest(y.numpy(), x.numpy(), norm=1)
            np.testing.assert_array_equal(iy.cpu().numpy(), want_i)
            np.testing.assert_array_equal(dy.cpu().numpy(), want_d)
