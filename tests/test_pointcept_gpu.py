"""Pointcept ``pointops`` subset on CUDA vs the reference.

Known answers of gamzerA/mps-pointops tests/test_pointcept.py:20-178 run on
the CUDA tensors; the golden cases of tests/golden/pointcept.npz (the
reference's CPU path on ragged batches with empty clouds, non-finite and far
points) pin indices bit for bit and distances to the oracle's IEEE values
(the golden distances come from torch's CPU sqrt, within one ulp of them);
grouping and interpolation match the reference's outputs and gradients."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import pointcept
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    return torch.as_tensor(np.asarray(a), device=dev, dtype=dtype)


def test_fps_uses_cumulative_offsets_and_global_int32_indices(cuda_device):
    xyz = torch.tensor([[0., 0, 0], [1., 0, 0], [4., 0, 0], [9., 0, 0],
                        [10., 0, 0], [11., 0, 0], [15., 0, 0]], device=cuda_device)
    offset = torch.tensor([4, 7], dtype=torch.int32, device=cuda_device)
    new_offset = torch.tensor([2, 4], dtype=torch.int32, device=cuda_device)
    result = pointcept.farthest_point_sampling(xyz, offset, new_offset)
    assert result.dtype == torch.int32 and result.device == xyz.device
    assert result.cpu().tolist() == [0, 3, 4, 6]


def test_knn_euclidean_distances_and_minus_one_padding(cuda_device):
    xyz = torch.tensor([[0., 0, 0], [2., 0, 0], [10., 0, 0], [12., 0, 0], [14., 0, 0]],
                       device=cuda_device, requires_grad=True)
    query = torch.tensor([[0.5, 0, 0], [11., 0, 0]], device=cuda_device, requires_grad=True)
    offset = torch.tensor([2, 5], dtype=torch.int64, device=cuda_device)
    new_offset = torch.tensor([1, 2], dtype=torch.int32, device=cuda_device)
    idx, dist = pointcept.knn_query(4, xyz, offset, query, new_offset)
    assert idx.dtype == torch.int32 and idx.cpu().tolist() == [[0, 1, -1, -1], [2, 3, 4, -1]]
    torch.testing.assert_close(dist.cpu(), torch.tensor([[0.5, 1.5, 1e5, 1e5], [1., 1., 3., 1e5]]),
                               rtol=1e-5, atol=1e-5)
    assert not dist.requires_grad


def test_knn_equal_distances_use_smaller_reference_index(cuda_device):
    x = torch.arange(16, dtype=torch.float32, device=cuda_device) * 0.25
    xyz = torch.stack((x, torch.zeros_like(x), torch.zeros_like(x)), dim=1)
    idx, dist = pointcept.knn_query(8, xyz, torch.tensor([16], dtype=torch.int32,
                                                          device=cuda_device))
    assert idx[2].cpu().tolist() == [2, 1, 3, 0, 4, 5, 6, 7]
    torch.testing.assert_close(dist[2].cpu(),
                               torch.tensor([0., 0.25, 0.25, 0.5, 0.5, 0.75, 1., 1.25]))


def test_knn_strict_upstream_distance_ceiling(cuda_device):
    xyz = torch.tensor([[99_999., 0, 0], [100_000., 0, 0], [100_001., 0, 0]], device=cuda_device)
    query = torch.zeros((1, 3), device=cuda_device)
    offset = torch.tensor([3], dtype=torch.int32, device=cuda_device)
    new_offset = torch.tensor([1], dtype=torch.int32, device=cuda_device)
    idx, dist = pointcept.knn_query(3, xyz, offset, query, new_offset)
    assert idx.cpu().tolist() == [[0, -1, -1]]
    assert dist.cpu().tolist() == [[99_999., 100_000., 100_000.]]


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_knn_nonfinite_reference_keeps_missing_slot_outside_other_batches(cuda_device, bad):
    dev = cuda_device
    query = torch.tensor([[0., 0, 0]], device=dev)
    new_offset = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    xyz = torch.tensor([[0., 0, 0], [bad, 0, 0]], device=dev)
    idx, dist = pointcept.knn_query(1, xyz, torch.tensor([1, 2], dtype=torch.int32, device=dev),
                                    query, new_offset)
    assert idx.cpu().tolist() == [[-1]] and dist.cpu().tolist() == [[100_000.]]
    xyz = torch.tensor([[0., 0, 0], [bad, 0, 0], [1., 0, 0]], device=dev)
    idx, dist = pointcept.knn_query(2, xyz, torch.tensor([1, 3], dtype=torch.int32, device=dev),
                                    query, new_offset)
    assert idx.cpu().tolist() == [[2, -1]] and dist.cpu().tolist() == [[1., 100_000.]]


def test_grouping_zero_padding_relative_xyz_and_gradients(cuda_device):
    dev = cuda_device
    xyz = torch.tensor([[0., 0, 0], [1., 0, 0], [2., 0, 0]], device=dev, requires_grad=True)
    feat = torch.tensor([[1., 2.], [3., 4.], [5., 6.]], device=dev, requires_grad=True)
    query = torch.tensor([[1., 0, 0]], device=dev, requires_grad=True)
    idx = torch.tensor([[2, -1, 2]], dtype=torch.int32, device=dev)
    result = pointcept.grouping(idx, feat, xyz, query, with_xyz=True)
    assert result.shape == (1, 3, 5)
    torch.testing.assert_close(result[0, 1], torch.zeros(5, device=dev))
    torch.testing.assert_close(result[0, 0], torch.tensor([1., 0, 0, 5, 6], device=dev))
    result.sum().backward()
    torch.testing.assert_close(feat.grad.cpu(), torch.tensor([[0., 0], [0, 0], [2, 2.]]))
    torch.testing.assert_close(xyz.grad.cpu(), torch.tensor([[0., 0, 0], [0, 0, 0], [2, 2, 2.]]))
    torch.testing.assert_close(query.grad.cpu(), torch.tensor([[-2., -2, -2.]]))


def test_query_and_group_reuses_indices_and_interpolation_gradient(cuda_device):
    dev = cuda_device
    xyz = torch.tensor([[0., 0, 0], [2., 0, 0]], device=dev, requires_grad=True)
    feat = torch.tensor([[2.], [10.]], device=dev, requires_grad=True)
    query = torch.tensor([[0.5, 0, 0]], device=dev, requires_grad=True)
    offset = torch.tensor([2], dtype=torch.int32, device=dev)
    new_offset = torch.tensor([1], dtype=torch.int32, device=dev)
    grouped, idx = pointcept.knn_query_and_group(feat, xyz, offset, query, new_offset,
                                                 nsample=3, with_xyz=True)
    assert idx.cpu().tolist() == [[0, 1, -1]]
    reused, same = pointcept.knn_query_and_group(feat, xyz, idx=idx, new_xyz=query)
    assert same is idx
    torch.testing.assert_close(reused, grouped[..., 3:])
    result = pointcept.interpolation(xyz, query, feat, offset, new_offset, k=3)
    torch.testing.assert_close(result.cpu(), torch.tensor([[4.]]), atol=1e-5, rtol=1e-5)
    result.sum().backward()
    torch.testing.assert_close(feat.grad.cpu(), torch.tensor([[0.75], [0.25]]), atol=1e-5,
                               rtol=1e-5)
    assert xyz.grad is None and query.grad is None


def test_empty_reference_batch_interpolates_zero(cuda_device):
    dev = cuda_device
    xyz = torch.tensor([[10., 0, 0]], device=dev)
    feat = torch.tensor([[3.]], device=dev, requires_grad=True)
    query = torch.tensor([[0., 0, 0], [10., 0, 0]], device=dev)
    offset = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    new_offset = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    output = pointcept.interpolation(xyz, query, feat, offset, new_offset)
    torch.testing.assert_close(output.cpu(), torch.tensor([[0.], [3.]]))
    output.sum().backward()
    torch.testing.assert_close(feat.grad.cpu(), torch.tensor([[1.]]))


@pytest.mark.parametrize("k", [1, 3, 16, 50])
def test_knn_query_golden(cuda_device, k):
    c = golden("pointcept")
    dev = cuda_device
    idx, dist = pointcept.knn_query(k, _t(c["x"], dev), _t(c["offset"], dev), _t(c["y"], dev),
                                    _t(c["new_offset"], dev))
    np.testing.assert_array_equal(idx.cpu().numpy(), c[f"knn_k{k}"]["idx"])
    want_i, want_d = O.pointcept_knn(k, c["x"], c["offset"], c["y"], c["new_offset"])
    np.testing.assert_array_equal(idx.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dist.cpu().numpy(), want_d)
    np.testing.assert_allclose(dist.cpu().numpy(), c[f"knn_k{k}"]["dist"], rtol=2.4e-7, atol=0)


def test_knn_query_ties_self_query(cuda_device):
    c = golden("pointcept")
    idx, dist = pointcept.knn_query(12, _t(c["ties"]["x"], cuda_device),
                                    _t(c["offset"], cuda_device))
    np.testing.assert_array_equal(idx.cpu().numpy(), c["ties"]["idx"])
    _, want_d = O.pointcept_knn(12, c["ties"]["x"], c["offset"])
    np.testing.assert_array_equal(dist.cpu().numpy(), want_d)
    np.testing.assert_allclose(dist.cpu().numpy(), c["ties"]["dist"], rtol=2.4e-7, atol=0)


def test_fps_golden(cuda_device):
    c = golden("pointcept")
    got = pointcept.farthest_point_sampling(_t(c["fps"]["x"], cuda_device),
                                            _t(c["offset"], cuda_device),
                                            _t(c["fps"]["new_offset"], cuda_device))
    assert got.dtype == torch.int32
    np.testing.assert_array_equal(got.cpu().numpy(), c["fps"]["idx"])


def test_grouping_and_interpolation_golden(cuda_device):
    c = golden("pointcept")
    dev = cuda_device
    xf = _t(c["fps"]["x"], dev)
    y = _t(c["y"], dev)
    feat = _t(c["interp"]["feat"], dev).requires_grad_()
    out = pointcept.interpolation(xf, y, feat, _t(c["offset"], dev), _t(c["new_offset"], dev), k=3)
    out.backward(_t(c["interp"]["grad_out"], dev))
    np.testing.assert_allclose(out.detach().cpu().numpy(), c["interp"]["out"], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(feat.grad.cpu().numpy(), c["interp"]["grad_feat"], rtol=1e-5,
                               atol=1e-6)
    g = c["group"]
    xr = xf.clone().requires_grad_()
    qr = y.clone().requires_grad_()
    f2 = _t(c["interp"]["feat"], dev).requires_grad_()
    grouped = pointcept.grouping(_t(g["idx"], dev), f2, xr, qr, with_xyz=True)
    grouped.backward(_t(g["grad_out"], dev))
    np.testing.assert_array_equal(grouped.detach().cpu().numpy(), g["out"])
    np.testing.assert_allclose(xr.grad.cpu().numpy(), g["grad_xyz"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(qr.grad.cpu().numpy(), g["grad_new_xyz"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(f2.grad.cpu().numpy(), g["grad_feat"], rtol=1e-5, atol=1e-6)
    # The indices the reference grouped with are this build's kNN result too.
    idx, _ = pointcept.knn_query(8, xf, _t(c["offset"], dev), y, _t(c["new_offset"], dev))
    np.testing.assert_array_equal(idx.cpu().numpy(), g["idx"])


def test_large_ragged_batch_matches_oracle(cuda_device):
    """A Point Transformer-sized flat batch: 6 clouds, 2k-9k points each,
    FPS to a quarter of each cloud, then kNN of the samples (k = 16)."""
    g = torch.Generator().manual_seed(123)
    lens = [2048, 5000, 9000, 3001, 7777, 4096]
    xyz = torch.rand(sum(lens), 3, generator=g) * 4.0
    offset = torch.tensor(np.cumsum(lens), dtype=torch.int32)
    new_offset = torch.tensor(np.cumsum([n // 4 for n in lens]), dtype=torch.int32)
    dev = cuda_device
    samples = pointcept.farthest_point_sampling(xyz.to(dev), offset.to(dev), new_offset.to(dev))
    want = O.pointcept_fps(xyz.numpy(), offset.numpy(), new_offset.numpy())
    np.testing.assert_array_equal(samples.cpu().numpy(), want)
    new_xyz = xyz[torch.as_tensor(want).long()]
    idx, dist = pointcept.knn_query(16, xyz.to(dev), offset.to(dev), new_xyz.to(dev),
                                    new_offset.to(dev))
    wi, wd = O.pointcept_knn(16, xyz.numpy(), offset.numpy(), new_xyz.numpy(),
                             new_offset.numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), wi)
    np.testing.assert_array_equal(dist.cpu().numpy(), wd)
