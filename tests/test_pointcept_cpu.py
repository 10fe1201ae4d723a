"""Pointcept ``pointops`` subset on the host: the oracle pinned to the
reference's own CPU results (tests/golden/pointcept.npz, generated from
mps_pointops/pointcept.py by tests/golden/make_golden.py), the validation
messages and the optional ``pointops`` registration of
gamzerA/mps-pointops tests/test_pointcept.py:181-205, and the loud refusal
of CPU computation."""

from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import compat, pointcept
from oracle import oracle as O


def test_oracle_matches_reference_knn_query():
    """Indices bit-exact; distances within one float32 ulp.  The reference's
    CPU distances come from torch's CPU float32 sqrt, which is not correctly
    rounded in near-halfway cases (e.g. sqrt(0.332381) gives 0.57652491 where
    the nearest float32 is 0.57652497); the oracle uses IEEE sqrt, like the
    CUDA kernels."""
    c = golden("pointcept")
    for k in (1, 3, 16, 50):
        idx, dist = O.pointcept_knn(k, c["x"], c["offset"], c["y"], c["new_offset"])
        np.testing.assert_array_equal(idx, c[f"knn_k{k}"]["idx"], err_msg=f"k={k}")
        np.testing.assert_allclose(dist, c[f"knn_k{k}"]["dist"], rtol=2.4e-7, atol=0,
                                   err_msg=f"k={k}")
        assert (idx == -1).any() and (dist[idx == -1] == np.float32(1e5)).all()
    idx, dist = O.pointcept_knn(12, c["ties"]["x"], c["offset"])
    np.testing.assert_array_equal(idx, c["ties"]["idx"])
    np.testing.assert_allclose(dist, c["ties"]["dist"], rtol=2.4e-7, atol=0)


def test_oracle_matches_reference_fps():
    c = golden("pointcept")
    got = O.pointcept_fps(c["fps"]["x"], c["offset"], c["fps"]["new_offset"])
    assert got.dtype == np.int32
    np.testing.assert_array_equal(got, c["fps"]["idx"])


def test_oracle_known_answers():
    """tests/test_pointcept.py:20-30, 34-50, 53-64, 67-79 of the reference."""
    xyz = np.array([[0., 0, 0], [1., 0, 0], [4., 0, 0], [9., 0, 0],
                    [10., 0, 0], [11., 0, 0], [15., 0, 0]], np.float32)
    assert O.pointcept_fps(xyz, [4, 7], [2, 4]).tolist() == [0, 3, 4, 6]
    xyz = np.array([[0., 0, 0], [2., 0, 0], [10., 0, 0], [12., 0, 0], [14., 0, 0]], np.float32)
    q = np.array([[0.5, 0, 0], [11., 0, 0]], np.float32)
    idx, dist = O.pointcept_knn(4, xyz, [2, 5], q, [1, 2])
    assert idx.tolist() == [[0, 1, -1, -1], [2, 3, 4, -1]]
    np.testing.assert_allclose(dist, [[0.5, 1.5, 1e5, 1e5], [1., 1., 3., 1e5]], rtol=1e-6)
    x = np.arange(16, dtype=np.float32) * 0.25
    line = np.stack((x, np.zeros_like(x), np.zeros_like(x)), axis=1)
    idx, _ = O.pointcept_knn(8, line, [16])
    assert idx[2].tolist() == [2, 1, 3, 0, 4, 5, 6, 7]
    far = np.array([[99_999., 0, 0], [100_000., 0, 0], [100_001., 0, 0]], np.float32)
    idx, dist = O.pointcept_knn(3, far, [3], np.zeros((1, 3), np.float32), [1])
    assert idx.tolist() == [[0, -1, -1]]
    assert dist.tolist() == [[99_999., 100_000., 100_000.]]


def test_validation_messages_and_cpu_refusal():
    xyz = torch.zeros((3, 3))
    with pytest.raises(ValueError, match="end at"):
        pointcept.farthest_point_sampling(xyz, torch.tensor([2]), torch.tensor([1]))
    with pytest.raises(ValueError, match="more FPS"):
        pointcept.farthest_point_sampling(xyz, torch.tensor([3]), torch.tensor([4]))
    with pytest.raises(ValueError, match="nondecreasing"):
        pointcept.knn_query(2, torch.zeros((3, 3)), torch.tensor([2, 1, 3]))
    with pytest.raises(ValueError, match="shape \\(N, 3\\)"):
        pointcept.knn_query(2, torch.zeros((3, 2)), torch.tensor([3]))
    with pytest.raises(ValueError, match="provided together"):
        pointcept.knn_query(2, xyz, torch.tensor([3]), new_xyz=xyz)
    with pytest.raises(ValueError, match="nsample"):
        pointcept.knn_query(-1, xyz, torch.tensor([3]))
    with pytest.raises(ValueError, match="same batch count"):
        pointcept.knn_query(2, xyz, torch.tensor([3]), xyz, torch.tensor([1, 3]))
    with pytest.raises(ValueError, match="out-of-range"):
        pointcept.grouping(torch.tensor([[3]]), torch.zeros((3, 2)), xyz)
    with pytest.raises(ValueError, match="required when idx is absent"):
        pointcept.knn_query_and_group(torch.zeros((3, 2)), xyz)
    # Empty results need no device; anything else refuses CPU tensors.
    assert pointcept.farthest_point_sampling(xyz, torch.tensor([3]), torch.tensor([0])).numel() == 0
    idx, dist = pointcept.knn_query(0, xyz, torch.tensor([3]))
    assert idx.shape == (3, 0) and idx.dtype == torch.int32 and dist.dtype == torch.float32
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        pointcept.farthest_point_sampling(xyz, torch.tensor([3]), torch.tensor([2]))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        pointcept.knn_query(2, xyz, torch.tensor([3]))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        pointcept.grouping(torch.tensor([[0, -1]]), torch.zeros((3, 2)), xyz)


def test_explicit_optional_registration():
    names = ("pointnet2_ops", "pointnet2_ops.pointnet2_utils", "knn_cuda", "torch_cluster",
             "pointops")
    saved = {name: sys.modules.pop(name) for name in names if name in sys.modules}
    try:
        assert "pointops" not in compat.install()
        assert "pointops" in compat.install(force=True, pointcept=True)
        import pointops

        assert pointops.knn_query is pointcept.knn_query
        assert pointops.interpolation is pointcept.interpolation
        assert pointops.farthest_point_sampling is pointcept.farthest_point_sampling
    finally:
        for name in names:
            sys.modules.pop(name, None)
        sys.modules.update(saved)
