"""SA grouping on the B200 kernels (mpo_group_points, mpo_query_and_group and
their backward passes) vs the oracle and the reference's own outputs
(tests/golden/grouping.npz).  Forward results are exact copies and one
subtraction, compared bit-exactly; gradients are float scatter-adds, compared
with rtol 1e-5 (atol 1e-5)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import _native as N
from mps_pointops import compat, grouping
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64, torch.int16])
def test_grouping_operation_matches_oracle(cuda_device, idx_dtype):
    g = torch.Generator().manual_seed(1)
    B, C, Np, P, S = 3, 37, 500, 61, 9
    f = torch.randn(B, C, Np, generator=g)
    idx = torch.randint(0, Np, (B, P, S), generator=g)
    fc = f.to(cuda_device).requires_grad_()
    launches = N.launch_count()
    out = compat.grouping_operation(fc, idx.to(idx_dtype).to(cuda_device))
    assert N.launch_count() > launches, "native kernel not used"
    np.testing.assert_array_equal(out.detach().cpu().numpy(), O.group_points(f.numpy(), idx.numpy()))
    gout = torch.randn(out.shape, generator=g)
    out.backward(gout.to(cuda_device))
    np.testing.assert_allclose(fc.grad.cpu().numpy(),
                               O.group_points_backward(gout.numpy(), idx.numpy(), Np), **TOL)


def test_gather_operation_matches_reference_golden(cuda_device):
    c = golden("grouping")["gather"]
    f = torch.from_numpy(c["features"]).to(cuda_device).requires_grad_()
    out = compat.gather_operation(f, torch.from_numpy(c["idx"]).to(cuda_device))
    np.testing.assert_array_equal(out.detach().cpu().numpy(), c["out"])
    out.sum().backward()
    want = O.group_points_backward(np.ones(out.shape + (1,)), c["idx"][..., None], f.shape[2])
    np.testing.assert_allclose(f.grad.cpu().numpy(), want, **TOL)


def test_out_of_range_index_raises(cuda_device):
    # Reported without a host wait: by the call itself once the device is
    # done, else by the next grouping call or check_indices().
    f = torch.randn(1, 4, 10, device=cuda_device)
    bad = torch.tensor([[[0, 3, 10]]], device=cuda_device)
    with pytest.raises(RuntimeError, match="out of bounds"):
        compat.grouping_operation(f, bad)
        grouping.check_indices()
    with pytest.raises(RuntimeError, match="out of bounds"):
        compat.gather_operation(f, torch.tensor([[-1, 2]], device=cuda_device))
        grouping.check_indices()
    grouping.check_indices()  # nothing left pending
    out = compat.gather_operation(f, torch.tensor([[9, 2]], device=cuda_device))
    grouping.check_indices()
    assert torch.equal(out, f[:, :, [9, 2]])


@pytest.mark.parametrize("case", ["qg_r0.15", "qg_r0.4"])
def test_query_and_group_matches_reference_composition(cuda_device, case):
    """tests/test_pointnet2_e2e.py:40-44 in one call: values bit-exact,
    gradients of xyz, new_xyz and features against the reference's autograd."""
    c = golden("grouping")[case]
    radius, nsample = float(c["meta"][0]), int(c["meta"][1])
    x = torch.from_numpy(c["xyz"]).to(cuda_device).requires_grad_()
    q = torch.from_numpy(c["new_xyz"]).to(cuda_device).requires_grad_()
    f = torch.from_numpy(c["features"]).to(cuda_device).requires_grad_()
    out, idx = grouping.query_and_group(x, q, f, radius, nsample)
    np.testing.assert_array_equal(idx.cpu().numpy(), c["idx"])
    np.testing.assert_array_equal(out.detach().cpu().numpy(), c["out"])
    out.backward(torch.from_numpy(c["grad_out"]).to(cuda_device))
    np.testing.assert_allclose(x.grad.cpu().numpy(), c["grad_xyz"], **TOL)
    np.testing.assert_allclose(q.grad.cpu().numpy(), c["grad_new_xyz"], **TOL)
    np.testing.assert_allclose(f.grad.cpu().numpy(), c["grad_features"], **TOL)


def test_query_and_group_config1_against_oracle_and_unfused(cuda_device):
    """BASELINE config 1 sizes: 8 clouds of 4096 points, 1024 centres, r 0.2,
    32 samples, 64 feature channels."""
    g = torch.Generator().manual_seed(2)
    xyz = torch.rand(8, 4096, 3, generator=g)
    feats = torch.randn(8, 64, 4096, generator=g)
    xc, fc = xyz.to(cuda_device), feats.to(cuda_device)
    idx0 = compat.furthest_point_sample(xc, 1024)
    new_xyz = compat.gather_operation(xc.transpose(1, 2).contiguous(), idx0)
    new_xyz = new_xyz.transpose(1, 2).contiguous()
    out, idx = grouping.query_and_group(xc, new_xyz, fc, 0.2, 32)
    want, want_idx = O.query_and_group(xyz.numpy(), new_xyz.cpu().numpy(), feats.numpy(), 0.2, 32)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_idx)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    # The unfused composition on the native pieces gives the same bits.
    nb = compat.ball_query(0.2, 32, xc, new_xyz)
    gx = compat.grouping_operation(xc.transpose(1, 2).contiguous(), nb)
    gx = gx - new_xyz.transpose(1, 2).unsqueeze(-1)
    unfused = torch.cat((gx, compat.grouping_operation(fc, nb)), dim=1)
    assert torch.equal(unfused, out)


def test_query_and_group_variants(cuda_device):
    g = torch.Generator().manual_seed(3)
    xyz = torch.rand(2, 700, 3, generator=g)
    q = xyz[:, :50].clone()
    f = torch.randn(2, 6, 700, generator=g)
    xc, qc, fc = xyz.to(cuda_device), q.to(cuda_device), f.to(cuda_device)
    out, idx = grouping.query_and_group(xc, qc, None, 0.3, 16)          # coordinates only
    want, _ = O.query_and_group(xyz.numpy(), q.numpy(), None, 0.3, 16)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    out, _ = grouping.query_and_group(xc, qc, fc, 0.3, 16, use_xyz=False)  # features only
    want, _ = O.query_and_group(xyz.numpy(), q.numpy(), f.numpy(), 0.3, 16, use_xyz=False)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    module = compat.QueryAndGroup(0.3, 16)
    np.testing.assert_array_equal(module(xc, qc, fc).cpu().numpy(),
                                  O.query_and_group(xyz.numpy(), q.numpy(), f.numpy(), 0.3, 16)[0])
    # Far-away centres: no hit, all-zero indices (pointnet2_ops padding).
    out, idx = grouping.query_and_group(xc, qc + 100.0, fc, 0.3, 4)
    assert torch.equal(idx, torch.zeros_like(idx))
    # Gradient only for some inputs.
    fr = fc.clone().requires_grad_()
    out, _ = grouping.query_and_group(xc, qc, fr, 0.3, 16)
    gout = torch.randn(out.shape, generator=g)
    out.backward(gout.to(cuda_device))
    _, want_idx = O.query_and_group(xyz.numpy(), q.numpy(), None, 0.3, 16)
    _, _, gf = O.query_and_group_backward(gout.numpy(), want_idx, 700)
    np.testing.assert_allclose(fr.grad.cpu().numpy(), gf, **TOL)


def test_sample_and_gather_matches_fps_then_gather(cuda_device):
    """tests/test_pointnet2_e2e.py:37-39 (compat FPS, then gather_operation) in
    one launch: identical indices and coordinates, and the gradient of the
    gathered points scatters back to xyz."""
    g = torch.Generator().manual_seed(4)
    for B, Np, P in ((8, 4096, 1024), (2, 9000, 300), (3, 50, 64)):
        xyz = torch.rand(B, Np, 3, generator=g).to(cuda_device)
        idx, new_xyz = grouping.sample_and_gather(xyz, P)
        want_idx = compat.furthest_point_sample(xyz, P)
        want = compat.gather_operation(xyz.transpose(1, 2).contiguous(), want_idx)
        assert torch.equal(idx, want_idx)
        assert torch.equal(new_xyz, want.transpose(1, 2))
    xr = xyz.clone().requires_grad_()
    idx, new_xyz = grouping.sample_and_gather(xr, 64)
    gout = torch.randn(new_xyz.shape, generator=g).to(cuda_device)
    new_xyz.backward(gout)
    want = O.group_points_backward(gout.cpu().numpy().transpose(0, 2, 1)[..., None],
                                   idx.cpu().numpy()[..., None], 50).transpose(0, 2, 1)
    np.testing.assert_allclose(xr.grad.cpu().numpy(), want, **TOL)


@pytest.mark.parametrize("B,Np,P,S,C,use_xyz", [
    (2, 700, 10, 16, 8, True),      # P*S < N: gathers straight from (B, C, N)
    (2, 700, 60, 16, 8, False),     # transposed features, 16-byte loads, no coordinates
    (3, 257, 33, 9, 12, True),      # transposed, 12 channels (partial second chunk)
    (1, 300, 40, 8, 3, True)])      # C < 4: direct path
def test_query_and_group_paths(cuda_device, B, Np, P, S, C, use_xyz):
    g = torch.Generator().manual_seed(5 + C)
    xyz = torch.rand(B, Np, 3, generator=g)
    q = xyz[:, :P].clone()
    f = torch.randn(B, C, Np, generator=g)
    xr = xyz.to(cuda_device).requires_grad_()
    qr = q.to(cuda_device).requires_grad_()
    fr = f.to(cuda_device).requires_grad_()
    out, idx = grouping.query_and_group(xr, qr, fr, 0.25, S, use_xyz=use_xyz)
    want, want_idx = O.query_and_group(xyz.numpy(), q.numpy(), f.numpy(), 0.25, S, use_xyz=use_xyz)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_idx)
    np.testing.assert_array_equal(out.detach().cpu().numpy(), want)
    gout = torch.randn(out.shape, generator=g)
    out.backward(gout.to(cuda_device))
    gx, gq, gf = O.query_and_group_backward(gout.numpy(), want_idx, Np, use_xyz=use_xyz)
    np.testing.assert_allclose(fr.grad.cpu().numpy(), gf, **TOL)
    if use_xyz:
        np.testing.assert_allclose(xr.grad.cpu().numpy(), gx, **TOL)
        np.testing.assert_allclose(qr.grad.cpu().numpy(), gq, **TOL)
    fg = f.to(cuda_device).requires_grad_()
    got = compat.grouping_operation(fg, idx)
    np.testing.assert_array_equal(got.detach().cpu().numpy(), O.group_points(f.numpy(), want_idx))
    gg = torch.randn(got.shape, generator=g)
    got.backward(gg.to(cuda_device))
    np.testing.assert_allclose(fg.grad.cpu().numpy(),
                               O.group_points_backward(gg.numpy(), want_idx, Np), **TOL)
