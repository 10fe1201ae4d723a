"""PyTorch3D-style Ball Query adapter (mps_pointops/pytorch3d.py of
gamzerA/mps-pointops, tests/test_pytorch3d_adapter.py) on CUDA tensors:
the reference tests' known answers, plus the oracle on ragged batches."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mps_pointops.pytorch3d import KNN, ball_query
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_defaults_named_fields_and_zero_padded_neighbors(cuda_device):  # :13-33
    queries = torch.zeros((1, 1, 3), device=cuda_device)
    points = torch.tensor([[[0.125, 0.0, 0.0], [2.0, 0.0, 0.0]]], device=cuda_device)
    result = ball_query(queries, points)
    assert isinstance(result, KNN) and result._fields == ("dists", "idx", "knn")
    assert result.dists.shape == result.idx.shape == (1, 1, 500)
    assert result.knn.shape == (1, 1, 500, 3)
    assert result.dists.dtype == torch.float32 and result.idx.dtype == torch.int64
    assert result.idx[0, 0, 0].item() == 0 and torch.all(result.idx[0, 0, 1:] == -1)
    assert result.dists[0, 0, 0].item() == 0.015625 and torch.all(result.dists[0, 0, 1:] == 0)
    assert torch.equal(result.knn[0, 0, 0], points[0, 0])
    assert torch.all(result.knn[0, 0, 1:] == 0)


def test_ragged_lengths_first_k_return_nn_and_cube_hint(cuda_device):  # :36-69
    q = torch.tensor([[[0.0, 0, 0], [0.0, 0, 0]], [[3.0, 0, 0], [0.0, 0, 0]]], device=cuda_device)
    p = torch.tensor([[[0.5, 0, 0], [0.25, 0, 0], [0.125, 0, 0], [2.0, 0, 0]],
                      [[0.125, 0, 0], [0.25, 0, 0], [2.0, 0, 0], [3.0, 0, 0]]], device=cuda_device)
    l1 = torch.tensor([1, 2], device=cuda_device)
    l2 = torch.tensor([2, 1], device=cuda_device)
    default = ball_query(q, p, l1, l2, 3, 1.0, True, False)
    cube = ball_query(q, p, l1, l2, 3, 1.0, True, True)
    no_nn = ball_query(q, p, l1, l2, 3, 1.0, False, True)
    assert default.idx.tolist() == [[[0, 1, -1], [-1, -1, -1]], [[-1, -1, -1], [0, -1, -1]]]
    assert default.dists.tolist() == [[[0.25, 0.0625, 0], [0, 0, 0]], [[0, 0, 0], [0.015625, 0, 0]]]
    assert torch.equal(cube.idx, default.idx) and torch.equal(cube.dists, default.dists)
    assert no_nn.knn is None
    assert default.knn[0, 0, 0, 0].item() == 0.5 and default.knn[0, 0, 1, 0].item() == 0.25
    assert torch.all(default.knn[default.idx == -1] == 0)


@pytest.mark.parametrize("batch,query_count,point_count,k",
                         [(1, 2, 0, 3), (1, 2, 2, 0), (1, 0, 2, 3), (0, 2, 2, 3)])
def test_empty_dimensions(cuda_device, batch, query_count, point_count, k):  # :72-87
    queries = torch.zeros((batch, query_count, 3), device=cuda_device)
    points = torch.zeros((batch, point_count, 3), device=cuda_device)
    result = ball_query(queries, points, K=k, radius=1.0)
    assert result.dists.shape == result.idx.shape == (batch, query_count, k)
    assert result.knn.shape == (batch, query_count, k, 3)
    assert torch.all(result.idx == -1) and torch.all(result.dists == 0)
    assert torch.all(result.knn == 0)


def test_coordinate_gradients_include_returned_neighbors(cuda_device):  # :90-103
    queries = torch.zeros((1, 1, 3), device=cuda_device, requires_grad=True)
    points = torch.tensor([[[0.25, 0.0, 0.0]]], device=cuda_device, requires_grad=True)
    result = ball_query(queries, points, K=2, radius=1.0)
    (result.dists.sum() + result.knn.sum()).backward()
    assert queries.grad.tolist() == [[[-0.5, 0.0, 0.0]]]
    assert points.grad.tolist() == [[[1.5, 1.0, 1.0]]]


@pytest.mark.parametrize("point_count,k", [(0, 2), (2, 0)])
def test_empty_neighbor_gather_keeps_zero_gradient(cuda_device, point_count, k):  # :106-118
    queries = torch.zeros((1, 1, 3), device=cuda_device)
    points = torch.zeros((1, point_count, 3), device=cuda_device, requires_grad=True)
    result = ball_query(queries, points, K=k, radius=1.0)
    result.knn.sum().backward()
    assert points.grad is not None and torch.all(points.grad == 0)


def test_rejects_unsupported_dtype_and_invalid_lengths(cuda_device):  # :121-134
    points = torch.zeros((1, 2, 3), device=cuda_device)
    with pytest.raises(TypeError, match="float32"):
        ball_query(points.half(), points.half(), K=1, radius=1.0)
    with pytest.raises(ValueError, match="lengths1|query_lengths"):
        ball_query(points, points, lengths1=torch.tensor([3], device=cuda_device), K=1, radius=1.0)
    with pytest.raises(TypeError, match="bool"):
        ball_query(points, points, K=1, radius=1.0, skip_points_outside_cube=1)


def test_ragged_batch_against_oracle(cuda_device):
    g = torch.Generator().manual_seed(12)
    p1, p2 = torch.rand(3, 200, 3, generator=g), torch.rand(3, 900, 3, generator=g)
    l1, l2 = torch.tensor([200, 37, 0]), torch.tensor([900, 11, 500])
    res = ball_query(p1.to(cuda_device), p2.to(cuda_device), l1.to(cuda_device),
                     l2.to(cuda_device), K=24, radius=0.15)
    d2, idx = O.ball_query(p1.numpy(), p2.numpy(), 0.15, 24, l1.numpy(), l2.numpy())
    np.testing.assert_array_equal(res.idx.cpu().numpy(), idx)
    np.testing.assert_array_equal(res.dists.cpu().numpy(), d2)
    gathered = p2.numpy()[np.arange(3)[:, None, None], np.maximum(idx, 0)]  # (3, 200, 24, 3)
    want_nn = np.where((idx >= 0)[..., None], gathered, np.float32(0.0))
    np.testing.assert_array_equal(res.knn.cpu().numpy(), want_nn)
