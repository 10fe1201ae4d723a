"""Squared-L2 Chamfer on B200 vs the reference (golden fixtures made by
mps_pointops.chamfer on CPU, closed-form cases of gamzerA/mps-pointops
tests/test_chamfer.py) and the oracle.  Nearest indices and per-point squared
distances are bit-exact; loss and gradients within rtol 1e-5."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import _native as N
from mps_pointops.chamfer import chamfer_distance
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def nearest(x, y, lx=None, ly=None):
    B, P, D = x.shape
    Q = y.shape[1]
    dev = x.device
    dx = torch.empty(B, P, device=dev)
    ix = torch.empty(B, P, dtype=torch.long, device=dev)
    dy = torch.empty(B, Q, device=dev)
    iy = torch.empty(B, Q, dtype=torch.long, device=dev)
    lib = N.lib()
    nbytes = lib.mpo_chamfer_workspace_bytes(B, P, Q, D, 1)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    N.check(lib.mpo_chamfer_nearest(N.ptr(x), N.ptr(y), N.ptr(lx), N.ptr(ly), B, P, Q, D, 1,
                                    N.ptr(dx), N.ptr(ix), N.ptr(dy), N.ptr(iy), N.ptr(ws),
                                    ws.numel(), N.stream(dev)), "nearest")
    return dx, ix, dy, iy


def test_golden_cases(cuda_device):
    for name, c in golden("chamfer").items():
        x = torch.from_numpy(c["x"]).to(cuda_device)
        y = torch.from_numpy(c["y"]).to(cuda_device)
        lx = torch.from_numpy(c["x_lengths"]).to(cuda_device) if "x_lengths" in c else None
        ly = torch.from_numpy(c["y_lengths"]).to(cuda_device) if "y_lengths" in c else None
        dx, ix, dy, iy = nearest(x, y, lx, ly)
        P, Q = x.shape[1], y.shape[1]
        vx = np.arange(P)[None] < (c["x_lengths"][:, None] if lx is not None else P)
        vy = np.arange(Q)[None] < (c["y_lengths"][:, None] if ly is not None else Q)
        np.testing.assert_array_equal(np.where(vx, ix.cpu().numpy(), -1),
                                      np.where(vx, c["idx_x"], -1), err_msg=name)
        np.testing.assert_array_equal(np.where(vy, iy.cpu().numpy(), -1),
                                      np.where(vy, c["idx_y"], -1), err_msg=name)
        np.testing.assert_array_equal(dx.cpu().numpy(), c["dist_x"], err_msg=name)
        np.testing.assert_array_equal(dy.cpu().numpy(), c["dist_y"], err_msg=name)
        xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
        loss, normals = chamfer_distance(xr, yr, lx, ly)
        assert normals is None
        loss.backward()
        np.testing.assert_allclose(loss.item(), c["loss"], rtol=1e-5, atol=1e-7, err_msg=name)
        np.testing.assert_allclose(xr.grad.cpu().numpy(), c["grad_x"], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(yr.grad.cpu().numpy(), c["grad_y"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("shape", [(1, 1, 1, 3), (2, 33, 1025, 3), (3, 4097, 2000, 3),
                                   (2, 100, 300, 1), (2, 100, 300, 5), (1, 64, 64, 128)])
def test_nearest_matches_oracle(cuda_device, shape):
    B, P, Q, D = shape
    g = torch.Generator().manual_seed(P + Q)
    x, y = torch.randn(B, P, D, generator=g), torch.randn(B, Q, D, generator=g)
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device))
    wdx, wix = O.chamfer_nearest(x.numpy(), y.numpy())
    wdy, wiy = O.chamfer_nearest(y.numpy(), x.numpy())
    np.testing.assert_array_equal(ix.cpu().numpy(), wix)
    np.testing.assert_array_equal(iy.cpu().numpy(), wiy)
    np.testing.assert_array_equal(dx.cpu().numpy(), wdx)
    np.testing.assert_array_equal(dy.cpu().numpy(), wdy)


def test_config2_slice_loss_and_grads(cuda_device):
    """BASELINE config 2 distribution (x ~ N(0,1), y = x + 0.05 N(0,1), permuted), B = 4."""
    g = torch.Generator().manual_seed(2)
    x = torch.randn(4, 8192, 3, generator=g)
    g3 = torch.Generator().manual_seed(3)
    y = x + 0.05 * torch.randn(4, 8192, 3, generator=g3)
    y = torch.stack([y[b, torch.randperm(8192, generator=g3)] for b in range(4)])
    loss_w, gx_w, gy_w, (dxw, ixw), (dyw, iyw) = O.chamfer_mean_loss_and_grad(x.numpy(), y.numpy())
    xc = x.to(cuda_device).requires_grad_()
    yc = y.to(cuda_device).requires_grad_()
    loss, _ = chamfer_distance(xc, yc)
    loss.backward()
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device))
    np.testing.assert_array_equal(ix.cpu().numpy(), ixw)
    np.testing.assert_array_equal(iy.cpu().numpy(), iyw)
    np.testing.assert_allclose(loss.item(), loss_w, rtol=1e-5)
    np.testing.assert_allclose(xc.grad.cpu().numpy(), gx_w, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(yc.grad.cpu().numpy(), gy_w, rtol=1e-5, atol=1e-9)


def test_closed_forms(cuda_device):  # tests/test_chamfer.py:8-150
    d = cuda_device
    x = torch.tensor([[[0.0, 0.0, 0.0], [2.0, 0.0, 0.0]]], device=d, requires_grad=True)
    y = torch.tensor([[[1.0, 0.0, 0.0]]], device=d, requires_grad=True)
    loss, normals = chamfer_distance(x, y, batch_reduction="sum")
    assert normals is None and loss.item() == 2.0
    loss.backward()
    torch.testing.assert_close(x.grad.cpu(), torch.tensor([[[-3.0, 0.0, 0.0], [1.0, 0.0, 0.0]]]))
    torch.testing.assert_close(y.grad.cpu(), torch.tensor([[[2.0, 0.0, 0.0]]]))

    x = torch.tensor([[[0.0, 0, 0], [float("nan"), 0, 0]]], device=d, requires_grad=True)
    y = torch.tensor([[[1.0, 0, 0], [float("inf"), 0, 0]]], device=d, requires_grad=True)
    lengths = torch.tensor([1], device=d)
    loss, _ = chamfer_distance(x, y, lengths, lengths)
    assert loss.item() == 2.0
    loss.backward()
    torch.testing.assert_close(x.grad[0, 0].cpu(), torch.tensor([-4.0, 0.0, 0.0]))
    torch.testing.assert_close(y.grad[0, 0].cpu(), torch.tensor([4.0, 0.0, 0.0]))
    assert torch.equal(x.grad[0, 1].cpu(), torch.zeros(3))

    x = torch.zeros((2, 1, 3), device=d)
    y = torch.tensor([[[1.0, 0.0, 0.0]], [[2.0, 0.0, 0.0]]], device=d)
    w = torch.tensor([0.1, 0.2], device=d)
    torch.testing.assert_close(chamfer_distance(x, y, weights=w)[0].cpu(), torch.tensor(6.0))
    torch.testing.assert_close(chamfer_distance(x, y, weights=w, point_reduction="sum",
                                                batch_reduction="sum")[0].cpu(), torch.tensor(1.8))
    torch.testing.assert_close(chamfer_distance(x, y, point_reduction="max",
                                                batch_reduction=None)[0].cpu(),
                               torch.tensor([1.0, 4.0]))
    torch.testing.assert_close(chamfer_distance(x, y, single_directional=True,
                                                batch_reduction=None)[0].cpu(),
                               torch.tensor([1.0, 4.0]))
    assert chamfer_distance(x, y, weights=torch.zeros(2, device=d))[0].item() == 0.0

    x = torch.zeros((2, 1, 3), device=d, requires_grad=True)
    y = torch.tensor([[[1.0, 0, 0]], [[2.0, 0, 0]]], device=d, requires_grad=True)
    loss, _ = chamfer_distance(x, y, weights=torch.tensor([1.0, 3.0], device=d))
    loss.backward()
    assert loss.item() == 6.5
    assert x.grad[:, 0, 0].cpu().tolist() == [-1.0, -6.0]
    assert y.grad[:, 0, 0].cpu().tolist() == [1.0, 6.0]

    for reduction, want_loss, want_xg, want_yg in (("sum", 6.0, [-4.0, 4.0], 0.0),
                                                   ("max", 4.0, [0.0, 4.0], -4.0)):
        x = torch.tensor([[[0.0, 0, 0], [3.0, 0, 0]]], device=d, requires_grad=True)
        y = torch.tensor([[[1.0, 0, 0]]], device=d, requires_grad=True)
        loss, _ = chamfer_distance(x, y, point_reduction=reduction)
        loss.backward()
        assert loss.item() == want_loss
        assert x.grad[0, :, 0].cpu().tolist() == want_xg
        assert y.grad[0, 0, 0].item() == want_yg


def test_overflow_selects_first_reference(cuda_device):  # tests/test_chamfer.py:178-197
    x = torch.tensor([[[1e20, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    y = torch.tensor([[[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    dx, ix, _, _ = nearest(x.detach(), y.detach())
    assert torch.isinf(dx).all() and ix.cpu().tolist() == [[0]]
    loss, _ = chamfer_distance(x, y, single_directional=True)
    assert torch.isinf(loss).item()
    loss.backward()
    torch.testing.assert_close(x.grad.cpu(), torch.tensor([[[2e20, 0.0, 0.0]]]))
    torch.testing.assert_close(y.grad.cpu(), torch.tensor([[[-2e20, 0, 0], [0.0, 0, 0]]]))


def test_first_tie_across_tiles_and_padding(cuda_device):  # tests/test_chamfer.py:452-477
    q = torch.zeros((2, 9, 3))
    r = torch.full((2, 3000, 3), 9.0)
    for j in (0, 31, 36, 1024, 2047, 2999):
        r[:, j] = torch.tensor([1.0, 0.0, 0.0]) if j % 2 else torch.tensor([0.0, -1.0, 0.0])
    q[0, 8, 0] = float("nan")
    ql, rl = torch.tensor([8, 7]), torch.tensor([3000, 2048])
    dx, ix, _, _ = nearest(q.to(cuda_device), r.to(cuda_device), ql.to(cuda_device),
                           rl.to(cuda_device))
    want_i = torch.zeros((2, 9), dtype=torch.long)
    want_i[0, 8] = -1
    want_i[1, 7:] = -1
    want_d = torch.ones((2, 9))
    want_d[0, 8] = 0
    want_d[1, 7:] = 0
    assert torch.equal(ix.cpu(), want_i) and torch.equal(dx.cpu(), want_d)


def test_normals_and_empty(cuda_device):  # tests/test_chamfer.py:307-420
    d = cuda_device
    for abs_cosine, want in ((True, 0.5), (False, 3.5)):
        x = torch.tensor([[[0., 0., 0.], [2., 0., 0.]]], device=d, requires_grad=True)
        y = torch.tensor([[[1., 0., 0.]]], device=d, requires_grad=True)
        xn = torch.tensor([[[1., 0., 0.], [0., 1., 0.]]], device=d, requires_grad=True)
        yn = torch.tensor([[[-1., 0., 0.]]], device=d, requires_grad=True)
        loss, normals = chamfer_distance(x, y, x_normals=xn, y_normals=yn, abs_cosine=abs_cosine)
        assert normals.item() == want
        grads = torch.autograd.grad(loss + normals, (x, y, xn, yn))
        assert grads[0].cpu().tolist() == [[[-3., 0., 0.], [1., 0., 0.]]]
        assert grads[1].cpu().tolist() == [[[2., 0., 0.]]]
    for x_empty in (True, False):
        x = torch.zeros((1, 0 if x_empty else 2, 3), device=d, requires_grad=True)
        y = torch.ones((1, 2 if x_empty else 0, 3), device=d, requires_grad=True)
        loss, normals = chamfer_distance(x, y)
        assert normals is None and loss.item() == 0.0
        gx, gy = torch.autograd.grad(loss, (x, y))
        assert not gx.any() and not gy.any()
    x = torch.zeros((1, 2, 3), device=d)
    with pytest.raises(ValueError, match="finite"):
        chamfer_distance(x.clone().fill_(float("nan")), x)
    with pytest.raises(ValueError, match=r"\[0, 2\]"):
        chamfer_distance(x, x, torch.tensor([3], device=d), torch.tensor([2], device=d))
    with pytest.raises(ValueError, match="nonnegative"):
        chamfer_distance(x, x, weights=torch.tensor([-1.0], device=d))


@pytest.mark.parametrize("where", ["x_last", "x_first", "y_mid", "both"])
def test_nonfinite_check_float4_arrays(cuda_device, where):
    # Both arrays a multiple of four floats and 16-byte aligned: the check's
    # combined x/y scan (mps_pointops/chamfer.py:79-110 messages).
    d = cuda_device
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 40, 3, generator=g)
    y = torch.randn(2, 28, 3, generator=g)
    if where in ("x_last", "both"):
        x[1, 39, 2] = float("nan")
    if where == "x_first":
        x[0, 0, 0] = float("inf")
    if where in ("y_mid", "both"):
        y[1, 5, 1] = -float("inf")
    msg = "valid y coordinates" if where == "y_mid" else "valid x coordinates"
    with pytest.raises(ValueError, match=msg):
        chamfer_distance(x.to(d), y.to(d))
    # the clean pair passes
    chamfer_distance(torch.randn(2, 40, 3, generator=g).to(d), torch.randn(2, 28, 3, generator=g).to(d))


@pytest.mark.parametrize("pos", [0, 12345, 4 * 8192 * 3 - 1])
def test_nonfinite_check_large_arrays(cuda_device, pos):
    # Config-2-sized clouds: the check's grid (one CTA per SM) takes several
    # strided rounds of four loads per thread; the first, a middle and the
    # last element are each found in either cloud.
    g = torch.Generator().manual_seed(12)
    x = torch.randn(4, 8192, 3, generator=g)
    y = torch.randn(4, 8192, 3, generator=g)
    xb = x.clone()
    xb.view(-1)[pos] = float("nan")
    with pytest.raises(ValueError, match="valid x coordinates"):
        chamfer_distance(xb.to(cuda_device), y.to(cuda_device))
    yb = y.clone()
    yb.view(-1)[pos] = float("inf")
    with pytest.raises(ValueError, match="valid y coordinates"):
        chamfer_distance(x.to(cuda_device), yb.to(cuda_device))
    chamfer_distance(x.to(cuda_device), y.to(cuda_device))


def test_length_check_more_clouds_than_threads(cuda_device):
    # 50,000 clouds: more lengths than the check's threads (one 256-thread CTA
    # per SM), so the lengths are checked in a strided loop; the bad one is
    # the last.
    B = 50000
    x = torch.zeros(B, 2, 3, device=cuda_device)
    ok = torch.full((B,), 2, dtype=torch.long, device=cuda_device)
    bad = ok.clone()
    bad[-1] = 3
    with pytest.raises(ValueError, match=r"y_lengths must lie in \[0, 2\]"):
        chamfer_distance(x, x, ok, bad)
    chamfer_distance(x, x, ok, ok)


@pytest.mark.parametrize("dimension", [1, 2, 4, 64, 128])
def test_first_index_tie_any_dimension(cuda_device, dimension):  # tests/test_chamfer_nd.py:50-73
    x = torch.zeros((1, 1, dimension), device=cuda_device, requires_grad=True)
    y = torch.zeros((1, 2, dimension), device=cuda_device)
    y[0, 0, 0], y[0, 1, 0] = 1, -1
    y.requires_grad_()
    loss, _ = chamfer_distance(x, y, single_directional=True, point_reduction="sum",
                               batch_reduction="sum")
    loss.backward()
    assert loss.item() == 1
    want = torch.zeros(dimension)
    want[0] = -2.0
    assert torch.equal(x.grad[0, 0].cpu(), want)
    assert torch.equal(y.grad[0, 0].cpu(), -want)
    assert not y.grad[0, 1].any()


# ---------------------------------------------------------------- symmetric D == 3 path
# Clouds of >= 512 points on both sides take the one-pass symmetric kernel
# (1024 x 1024 work items, 64-bit key atomics); these cases cross item edges.

@pytest.mark.parametrize("shape", [(1, 512, 512), (2, 1500, 2100), (3, 3000, 700),
                                   (1, 1025, 4097)])
def test_symmetric_matches_oracle(cuda_device, shape):
    B, P, Q = shape
    g = torch.Generator().manual_seed(P * 7 + Q)
    x, y = torch.randn(B, P, 3, generator=g), torch.randn(B, Q, 3, generator=g)
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device))
    wdx, wix = O.chamfer_nearest(x.numpy(), y.numpy())
    wdy, wiy = O.chamfer_nearest(y.numpy(), x.numpy())
    np.testing.assert_array_equal(ix.cpu().numpy(), wix)
    np.testing.assert_array_equal(iy.cpu().numpy(), wiy)
    np.testing.assert_array_equal(dx.cpu().numpy(), wdx)
    np.testing.assert_array_equal(dy.cpu().numpy(), wdy)


def test_symmetric_lengths_and_padding(cuda_device):
    g = torch.Generator().manual_seed(11)
    x, y = torch.randn(3, 2100, 3, generator=g), torch.randn(3, 1900, 3, generator=g)
    x[:, 1500:] = float("nan")  # padding may hold anything
    y[:, 1800:] = float("inf")
    lx, ly = torch.tensor([1500, 0, 1025]), torch.tensor([1800, 700, 0])
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device), lx.to(cuda_device),
                             ly.to(cuda_device))
    wdx, wix = O.chamfer_nearest(x.numpy(), y.numpy(), lx.numpy(), ly.numpy())
    wdy, wiy = O.chamfer_nearest(y.numpy(), x.numpy(), ly.numpy(), lx.numpy())
    np.testing.assert_array_equal(ix.cpu().numpy(), wix)
    np.testing.assert_array_equal(iy.cpu().numpy(), wiy)
    np.testing.assert_array_equal(dx.cpu().numpy(), wdx)
    np.testing.assert_array_equal(dy.cpu().numpy(), wdy)


def test_symmetric_ties_across_items(cuda_device):
    """Exact ties spread over warps, lanes, blocks and 1024-point items: the
    lowest index must win in both directions."""
    x = torch.full((1, 3000, 3), 50.0)
    y = torch.full((1, 2500, 3), -50.0)
    for i in (7, 8, 255, 256, 1023, 1024, 2047, 2999):
        x[0, i] = torch.tensor([1.0, 0.0, 0.0]) if i % 2 else torch.tensor([0.0, 0.0, -1.0])
    for j in (3, 511, 512, 1023, 1024, 1031, 2499):
        y[0, j] = torch.tensor([0.0, 1.0, 0.0]) if j % 2 else torch.tensor([-1.0, 0.0, 0.0])
    x[0, 2000] = torch.tensor([0.0, 0.0, 0.0])
    y[0, 2400] = torch.tensor([0.0, 0.0, 0.0])
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device))
    wdx, wix = O.chamfer_nearest(x.numpy(), y.numpy())
    wdy, wiy = O.chamfer_nearest(y.numpy(), x.numpy())
    np.testing.assert_array_equal(ix.cpu().numpy(), wix)
    np.testing.assert_array_equal(iy.cpu().numpy(), wiy)
    np.testing.assert_array_equal(dx.cpu().numpy(), wdx)
    np.testing.assert_array_equal(dy.cpu().numpy(), wdy)


def test_symmetric_overflow_rows(cuda_device):
    g = torch.Generator().manual_seed(5)
    x, y = torch.randn(1, 600, 3, generator=g), torch.randn(1, 1100, 3, generator=g)
    x[0, 17] = torch.tensor([3e19, 0.0, 0.0])   # every SD of this row overflows
    y[0, 1099] = torch.tensor([-3e19, 0.0, 0.0])
    dx, ix, dy, iy = nearest(x.to(cuda_device), y.to(cuda_device))
    wdx, wix = O.chamfer_nearest(x.numpy(), y.numpy())
    wdy, wiy = O.chamfer_nearest(y.numpy(), x.numpy())
    np.testing.assert_array_equal(ix.cpu().numpy(), wix)
    np.testing.assert_array_equal(iy.cpu().numpy(), wiy)
    assert ix[0, 17].item() == 0 and torch.isinf(dx[0, 17])
