"""three_nn / three_interpolate on B200 vs the reference's CPU path, the
original PointNet++ CUDA extension's outputs (docs/parity/pointnet2-cuda.json
of gamzerA/mps-pointops) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops.pointnet2 import three_interpolate, three_nn
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_three_nn_golden(cuda_device):
    g = golden("pointnet2")
    for name in ("nn_random", "nn_ties"):
        c = g[name]
        d, i = three_nn(torch.from_numpy(c["unknown"]).to(cuda_device),
                        torch.from_numpy(c["known"]).to(cuda_device))
        assert i.dtype == torch.int32
        np.testing.assert_array_equal(i.cpu().numpy(), c["idx"], err_msg=name)
        np.testing.assert_allclose(d.cpu().numpy(), c["dist"], rtol=1e-6, atol=0, err_msg=name)
    d, i = three_nn(torch.tensor([[[0., 0., 0.], [2., 0., 0.]]], device=cuda_device),
                    torch.tensor([[[1., 0., 0.], [-1., 0., 0.], [0., 2., 0.], [1., 0., 0.]]],
                                 device=cuda_device))
    assert i.cpu().tolist() == [[[0, 1, 3], [0, 3, 2]]]


@pytest.mark.parametrize("case", ["ties_and_duplicates", "seeded_stride"])
def test_original_pointnet2_cuda_fixture(cuda_device, case):
    c = golden("pointnet2_upstream_cuda")[case]
    d, i = three_nn(torch.from_numpy(c["unknown"]).to(cuda_device),
                    torch.from_numpy(c["known"]).to(cuda_device))
    np.testing.assert_array_equal(i.cpu().numpy(), c["nearest_indices"])
    np.testing.assert_allclose(d.cpu().numpy(), c["distances"], rtol=2e-6, atol=1e-5)
    f = torch.from_numpy(c["features"]).to(cuda_device).requires_grad_()
    w = torch.from_numpy(c["weights"]).to(cuda_device).requires_grad_()
    out = three_interpolate(f, torch.from_numpy(c["interpolate_indices"]).to(cuda_device), w)
    np.testing.assert_allclose(out.detach().cpu().numpy(), c["interpolated"], rtol=2e-6, atol=1e-5)
    out.backward(torch.from_numpy(c["gradient"]).to(cuda_device))
    np.testing.assert_allclose(f.grad.cpu().numpy(), c["feature_gradient"], rtol=2e-6, atol=1e-5)
    np.testing.assert_array_equal(w.grad.cpu().numpy(), c["weight_gradient"])


@pytest.mark.parametrize("shape", [(1, 5, 3), (2, 1000, 7), (8, 4096, 1024)])
def test_three_nn_matches_oracle(cuda_device, shape):
    B, Nq, M = shape
    g = torch.Generator().manual_seed(Nq)
    u, k = torch.rand(B, Nq, 3, generator=g), torch.rand(B, M, 3, generator=g)
    want_d, want_i = O.three_nn(u.numpy(), k.numpy())
    d, i = three_nn(u.to(cuda_device), k.to(cuda_device))
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)


def test_three_nn_nan_last(cuda_device):
    k = torch.rand(1, 6, 3)
    k[0, 1, 0] = float("nan")
    k[0, 4, 2] = float("nan")
    u = torch.rand(1, 9, 3)
    want_d, want_i = O.three_nn(u.numpy(), k[:, :5].numpy())
    d, i = three_nn(u.to(cuda_device), k[:, :5].to(cuda_device))
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)


def test_interpolate_golden_and_known_answer(cuda_device):
    c = golden("pointnet2")["interp_random"]
    f = torch.from_numpy(c["features"]).to(cuda_device).requires_grad_()
    out = three_interpolate(f, torch.from_numpy(c["indices"]).to(cuda_device),
                            torch.from_numpy(c["weights"]).to(cuda_device))
    np.testing.assert_array_equal(out.detach().cpu().numpy(), c["out"])
    out.backward(torch.from_numpy(c["grad_out"]).to(cuda_device))
    np.testing.assert_allclose(f.grad.cpu().numpy(), c["grad_features"], rtol=2e-6, atol=2e-6)
    features = torch.tensor([[[2., 3., 5., 7.], [11., 13., 17., 19.]]], device=cuda_device,
                            requires_grad=True)
    indices = torch.tensor([[[0, 1, 1], [3, 1, 0]]], dtype=torch.int32, device=cuda_device)
    weights = torch.tensor([[[0.5, 0.25, 0.25], [1., 0.5, -0.5]]], device=cuda_device,
                           requires_grad=True)
    output = three_interpolate(features, indices, weights)
    assert output.cpu().tolist() == [[[2.5, 7.5], [12., 20.]]]
    output.sum().backward()
    assert features.grad.cpu().tolist() == [[[0., 1., 0., 1.], [0., 1., 0., 1.]]]
    assert not weights.grad.any()


@pytest.mark.parametrize("shape", [(8, 64, 1024, 4096), (2, 3, 70000, 500), (1, 1, 1, 1)])
def test_interpolate_matches_oracle(cuda_device, shape):
    B, C, M, Nn = shape
    g = torch.Generator().manual_seed(M)
    f = torch.randn(B, C, M, generator=g)
    i = torch.randint(M, (B, Nn, 3), generator=g, dtype=torch.int32)
    w = torch.rand(B, Nn, 3, generator=g)
    up = torch.randn(B, C, Nn, generator=g)
    fc = f.to(cuda_device).requires_grad_()
    out = three_interpolate(fc, i.to(cuda_device), w.to(cuda_device))
    np.testing.assert_array_equal(out.detach().cpu().numpy(),
                                  O.three_interpolate(f.numpy(), i.numpy(), w.numpy()))
    out.backward(up.to(cuda_device))
    want = O.three_interpolate_backward(up.numpy(), i.numpy(), w.numpy(), M)
    np.testing.assert_allclose(fc.grad.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


def test_empty_and_bad_indices(cuda_device):  # tests/test_pointnet2.py:129-148
    features = torch.randn(1, 2, 4, device=cuda_device, requires_grad=True)
    empty = three_interpolate(features, torch.empty((1, 0, 3), dtype=torch.int32, device=cuda_device),
                              torch.empty((1, 0, 3), device=cuda_device))
    assert empty.shape == (1, 2, 0)
    empty.sum().backward()
    assert features.grad is not None and torch.count_nonzero(features.grad).item() == 0
    with pytest.raises(IndexError):
        three_interpolate(features, torch.tensor([[[0, 4, 1]]], device=cuda_device),
                          torch.ones((1, 1, 3), device=cuda_device))
    # The check runs on the caller's indices (device-side, read after the
    # launch): negative int32, and int64 values that would wrap into range.
    for bad in (torch.tensor([[[0, -1, 1]]], dtype=torch.int32),
                torch.tensor([[[0, 2**32 + 1, 1]]], dtype=torch.int64)):
        with pytest.raises(IndexError, match=r"\[0, 4\)"):
            three_interpolate(features, bad.to(cuda_device), torch.ones((1, 1, 3), device=cuda_device))
    ok = three_interpolate(features, torch.tensor([[[0, 3, 1]]], device=cuda_device),
                           torch.ones((1, 1, 3), device=cuda_device))
    assert ok.shape == (1, 2, 1)
    for shape in [(0, 7, 0), (2, 0, 0), (2, 0, 5)]:
        b, q, p = shape
        d, i = three_nn(torch.empty((b, q, 3), device=cuda_device),
                        torch.empty((b, p, 3), device=cuda_device))
        assert d.shape == i.shape == (b, q, 3)
