"""Feature-space (D != 3) Chamfer on the symmetric tile kernel, float64
Chamfer, and BASELINE config 2 at its full size, on B200.

Fixtures: tests/golden/chamfer_nd.npz, made by the reference's CPU path
(mps_pointops/chamfer.py:161-212 search, :342-488 loss, autograd gradients)
for norm 2 and norm 1 in float32 and float64.  Nearest indices are bit-exact
on valid rows; float32 losses within rtol 1e-5, float64 within rtol 1e-10.
Gradients: the kernels' float atomics sum each point's terms in another order
than torch, and a point matched by hundreds of others (a cloud of two points)
sums terms of both signs that cancel, so gradients are compared with
rtol 1e-5 (1e-10) plus atol 1e-5 (1e-10) times the largest gradient
magnitude of the array.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from cases import ND_CASES, nd_cloud_pair
from conftest import golden
from mps_pointops import _native as N
from mps_pointops.chamfer import chamfer_distance
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(rtol=1e-5, atol=1e-7), torch.float64: dict(rtol=1e-10, atol=1e-12)}


def _case(name):
    c = golden("chamfer_nd")[name]
    B, P, Q, D, seed, lens = ND_CASES[name]
    x, y = nd_cloud_pair(B, P, Q, D, seed, lattice=name.endswith("lattice"))
    digest = hashlib.sha256(x.numpy().tobytes() + y.numpy().tobytes()).digest()
    assert np.frombuffer(digest, dtype=np.uint8).tolist() == c["sha256"].tolist()
    lx = None if lens is None else torch.tensor(lens[0])
    ly = None if lens is None else torch.tensor(lens[1])
    return c, x, y, lx, ly


def _valid(n, lengths, B):
    lens = np.full(B, n) if lengths is None else lengths.numpy()
    return np.arange(n)[None, :] < lens[:, None]


def _nearest(x, y, lx, ly, norm):
    """Both directions through the C ABI: mpo_chamfer_nearest (float32, norm 2),
    mpo_chamfer_nearest_l1 (float32, norm 1), mpo_chamfer_nearest_f64."""
    B, P, D = x.shape
    Q = y.shape[1]
    dev = x.device
    dx = torch.empty(B, P, dtype=x.dtype, device=dev)
    dy = torch.empty(B, Q, dtype=x.dtype, device=dev)
    ix = torch.empty(B, P, dtype=torch.long, device=dev)
    iy = torch.empty(B, Q, dtype=torch.long, device=dev)
    lib = N.lib()
    args = (N.ptr(x), N.ptr(y), N.ptr(lx), N.ptr(ly), B, P, Q, D)
    outs = (N.ptr(dx), N.ptr(ix), N.ptr(dy), N.ptr(iy))
    if x.dtype == torch.float64:
        rc = lib.mpo_chamfer_nearest_f64(*args, norm, 1, *outs, N.stream(dev))
    elif norm == 1:
        rc = lib.mpo_chamfer_nearest_l1(*args, 1, *outs, N.stream(dev))
    else:
        ws = torch.empty(max(1, lib.mpo_chamfer_workspace_bytes(B, P, Q, D, 1)),
                         dtype=torch.uint8, device=dev)
        rc = lib.mpo_chamfer_nearest(*args, 1, *outs, N.ptr(ws), ws.numel(), N.stream(dev))
    N.check(rc, "nearest")
    return dx, ix, dy, iy


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("norm", [1, 2])
@pytest.mark.parametrize("name", list(ND_CASES))
def test_feature_space_and_float64_match_reference(cuda_device, name, norm, dtype):
    c, x, y, lx, ly = _case(name)
    tag = "f64" if dtype == torch.float64 else "f32"
    B, P = x.shape[:2]
    Q = y.shape[1]
    xd, yd = x.to(cuda_device, dtype), y.to(cuda_device, dtype)
    lxd = None if lx is None else lx.to(cuda_device)
    lyd = None if ly is None else ly.to(cuda_device)
    _, ix, _, iy = _nearest(xd, yd, lxd, lyd, norm)
    vx, vy = _valid(P, lx, B), _valid(Q, ly, B)
    ix, iy = ix.cpu().numpy(), iy.cpu().numpy()
    np.testing.assert_array_equal(ix[vx], c[f"{tag}_n{norm}_idx_x"][vx])
    np.testing.assert_array_equal(iy[vy], c[f"{tag}_n{norm}_idx_y"][vy])
    assert (ix[~vx] == -1).all() and (iy[~vy] == -1).all()
    if dtype == torch.float32:   # the oracle too (its float32 search)
        _, wix = O.chamfer_nearest(x.numpy(), y.numpy(), None if lx is None else lx.numpy(),
                                   None if ly is None else ly.numpy(), norm=norm)
        np.testing.assert_array_equal(ix, wix)
    xr, yr = xd.clone().requires_grad_(), yd.clone().requires_grad_()
    loss, _ = chamfer_distance(xr, yr, lxd, lyd, norm=norm)
    loss.backward()
    assert loss.dtype == dtype and xr.grad.dtype == dtype
    np.testing.assert_allclose(loss.item(), c[f"{tag}_n{norm}_loss"], **TOL[dtype])
    if f"{tag}_n{norm}_grad_x" in c:
        for got, want in ((xr.grad, c[f"{tag}_n{norm}_grad_x"]),
                          (yr.grad, c[f"{tag}_n{norm}_grad_y"])):
            rtol = TOL[dtype]["rtol"]
            np.testing.assert_allclose(got.cpu().numpy(), want, rtol=rtol,
                                       atol=rtol * float(np.abs(want).max()))


def test_symmetric_kernel_matches_one_direction_passes(cuda_device):
    """The D != 3 symmetric kernel (both directions from one evaluation per
    pair) against two single-direction searches, on tile-edge sizes."""
    g = torch.Generator().manual_seed(77)
    for B, P, Q, D in ((1, 1, 1, 2), (2, 511, 513, 4), (1, 1025, 129, 16), (2, 257, 65, 96),
                       (1, 300, 1000, 144), (1, 64, 64, 145)):
        x = torch.randn(B, P, D, generator=g).to(cuda_device)
        y = torch.randn(B, Q, D, generator=g).to(cuda_device)
        for norm in (1, 2):
            both = chamfer_distance(x, y, norm=norm, point_reduction=None, batch_reduction=None)[0]
            fx = chamfer_distance(x, y, norm=norm, point_reduction=None, batch_reduction=None,
                                  single_directional=True)[0]
            fy = chamfer_distance(y, x, norm=norm, point_reduction=None, batch_reduction=None,
                                  single_directional=True)[0]
            assert torch.equal(both[0], fx) and torch.equal(both[1], fy), (B, P, Q, D, norm)


def test_float64_weighted_single_directional(cuda_device):
    c = golden("chamfer_nd")["f64_weighted"]
    x = torch.from_numpy(c["x"]).to(cuda_device).requires_grad_()
    y = torch.from_numpy(c["y"]).to(cuda_device).requires_grad_()
    w = torch.from_numpy(c["weights"]).to(cuda_device)
    loss, _ = chamfer_distance(x, y, weights=w, batch_reduction="sum", single_directional=True)
    loss.backward()
    np.testing.assert_allclose(loss.item(), c["loss"], **TOL[torch.float64])
    np.testing.assert_allclose(x.grad.cpu().numpy(), c["grad_x"], **TOL[torch.float64])
    np.testing.assert_allclose(y.grad.cpu().numpy(), c["grad_y"], **TOL[torch.float64])


def test_float64_gradcheck(cuda_device):
    """tests/test_chamfer.py:200 of the reference: a float64 gradcheck."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 9, 3, generator=g, dtype=torch.float64).to(cuda_device)
    y = torch.randn(2, 7, 3, generator=g, dtype=torch.float64).to(cuda_device)
    for norm in (2, 1):
        assert torch.autograd.gradcheck(
            lambda a, b: chamfer_distance(a, b, norm=norm)[0],
            (x.clone().requires_grad_(), y.clone().requires_grad_()), eps=1e-6, atol=1e-5)


def test_bench_config2_full_batch_matches_oracle(cuda_device):
    """BASELINE config 2 exactly as bench.py's timed step runs it (its own
    inputs: B = 32 pairs of 8192 points, x ~ N(0,1), y = x + 0.05 N(0,1) in a
    per-cloud permutation, rank 0's seed): indices bit-exact, loss and
    gradients within rtol 1e-5 of the oracle."""
    import bench
    x, y = bench.chamfer_inputs(bench.B_PER_GPU, seed=2)
    assert x.shape == (32, 8192, 3)
    loss_w, gx_w, gy_w, (_, ixw), (_, iyw) = O.chamfer_mean_loss_and_grad(x.numpy(), y.numpy())
    xc = x.to(cuda_device).requires_grad_()
    yc = y.to(cuda_device).requires_grad_()
    loss, _ = chamfer_distance(xc, yc)
    loss.backward()
    _, ix, _, iy = _nearest(x.to(cuda_device), y.to(cuda_device), None, None, 2)
    np.testing.assert_array_equal(ix.cpu().numpy(), ixw)
    np.testing.assert_array_equal(iy.cpu().numpy(), iyw)
    np.testing.assert_allclose(loss.item(), loss_w, rtol=1e-5)
    np.testing.assert_allclose(xc.grad.cpu().numpy(), gx_w, rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(yc.grad.cpu().numpy(), gy_w, rtol=1e-5, atol=1e-9)
