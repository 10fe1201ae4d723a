"""Host-side API behaviour that needs no GPU: validation order, exception
types and messages of the reference (tests in gamzerA/mps-pointops
tests/test_fps.py, test_knn.py, test_pointnet2.py, test_ball_query_api.py,
test_chamfer.py, test_compat.py), and the loud refusal of CPU tensors."""

from __future__ import annotations

import sys

import pytest
import torch

import mps_pointops
from mps_pointops import compat
from mps_pointops._ball_query_cuda import _checked_radius_and_k
from mps_pointops.chamfer import chamfer_distance
from mps_pointops.pointnet2 import three_interpolate, three_nn


def test_cpu_tensors_fail_loudly():
    xyz = torch.rand(1, 20, 3)
    for call in (lambda: mps_pointops.furthest_point_sample(xyz, 4),
                 lambda: mps_pointops.knn(xyz, xyz, 3),
                 lambda: mps_pointops.ball_query(xyz, xyz, 0.5, 3),
                 lambda: three_nn(xyz, xyz),
                 lambda: chamfer_distance(xyz, xyz),
                 lambda: compat.furthest_point_sample(xyz, 4),
                 lambda: compat.ball_query(0.5, 3, xyz, xyz)):
        with pytest.raises(RuntimeError, match="CUDA tensors only"):
            call()


def test_fps_validation():  # tests/test_fps.py:71-80, 157-159
    with pytest.raises(ValueError):
        mps_pointops.furthest_point_sample(torch.randn(10, 3), 4)
    with pytest.raises(ValueError):
        mps_pointops.furthest_point_sample(torch.randn(1, 0, 3), 4)
    with pytest.raises(IndexError):
        mps_pointops.furthest_point_sample(torch.randn(1, 10, 3), 4, start_idx=10)
    with pytest.raises(ValueError, match="strategy"):
        mps_pointops.furthest_point_sample(torch.randn(1, 8, 3), 2, strategy="unknown")


def test_knn_validation():  # tests/test_knn.py:94-106
    ref = torch.randn(1, 300, 3)
    with pytest.raises(ValueError):
        mps_pointops.knn(ref, ref, 301)
    with pytest.raises(ValueError):
        mps_pointops.knn(ref, torch.randn(2, 300, 3), 4)
    with pytest.raises(ValueError, match="D >= 1"):
        mps_pointops.knn(ref[:, :, :0], ref[:, :, :0], 0)
    with pytest.raises(ValueError, match="ref must have shape"):
        mps_pointops.knn(torch.zeros(1, 3, 64), torch.zeros(1, 3, 128), 2)


@pytest.mark.parametrize("radius", [-0.1, float("inf"), float("nan"), 1e-40, 1e39, True])
def test_ball_query_rejects_bad_radius(radius):  # tests/test_ball_query_api.py:37-42
    xyz = torch.rand(1, 20, 3)
    with pytest.raises(ValueError):
        mps_pointops.ball_query(xyz[:, :4], xyz, radius, 4)


@pytest.mark.parametrize("K", [-1, 1.5, True])
def test_ball_query_rejects_bad_k(K):  # tests/test_ball_query_api.py:45-50
    xyz = torch.rand(1, 20, 3)
    with pytest.raises(ValueError):
        mps_pointops.ball_query(xyz[:, :4], xyz, 0.5, K)


def test_radius_square_rounding_known_answer():  # tests/test_ball_query_mps.py:248-261
    import struct
    r32, r2 = _checked_radius_and_k(0.1, 1)
    assert struct.unpack("<I", struct.pack("<f", r2))[0] == 0x3C23D70B
    with pytest.raises(ValueError, match="2\\*\\*-112"):
        _checked_radius_and_k(float(torch.nextafter(torch.tensor(2.0**-112),
                                                    torch.tensor(0.0))), 1)


def test_pointnet2_validation():  # tests/test_pointnet2.py:151-165
    points = torch.zeros((1, 2, 3))
    with pytest.raises(ValueError, match="at least 3"):
        three_nn(points, points)
    with pytest.raises(TypeError, match="float32"):
        three_nn(points.half(), torch.zeros((1, 3, 3)).half())
    with pytest.raises(ValueError, match="batch"):
        three_nn(points, torch.zeros((2, 3, 3)))
    with pytest.raises(TypeError, match="indices"):
        three_interpolate(torch.zeros((1, 2, 3)), torch.zeros((1, 2, 3)), torch.ones((1, 2, 3)))
    with pytest.raises(ValueError, match="source point"):
        three_interpolate(torch.zeros((1, 2, 0)), torch.zeros((1, 2, 3), dtype=torch.int32),
                          torch.ones((1, 2, 3)))
    with pytest.raises(IndexError):
        three_interpolate(torch.zeros((1, 2, 4)), torch.tensor([[[0, -1, 1]]], dtype=torch.int32),
                          torch.ones((1, 1, 3)))


def test_chamfer_validation():  # tests/test_chamfer.py:285-304, test_chamfer_nd.py:98-108
    x = torch.zeros((1, 2, 3))
    y = torch.ones((1, 2, 3))
    with pytest.raises(ValueError, match="batch_reduction"):
        chamfer_distance(x, y, point_reduction=None)
    with pytest.raises(ValueError, match="1 or 2 norm"):
        chamfer_distance(x, y, norm=3)
    with pytest.raises(ValueError, match="Normals must be None"):
        chamfer_distance(x, y, x_normals=x, point_reduction="max")
    with pytest.raises(ValueError, match="D >= 1"):
        chamfer_distance(torch.empty((1, 2, 0)), torch.empty((1, 2, 0)))
    with pytest.raises(TypeError):
        chamfer_distance(x.int(), y.int())


NAMES = ["pointnet2_ops", "pointnet2_ops.pointnet2_utils", "knn_cuda", "torch_cluster"]


@pytest.fixture
def installed():
    saved = {n: sys.modules.pop(n) for n in NAMES if n in sys.modules}
    compat.install(force=True)
    yield
    for n in NAMES:
        sys.modules.pop(n, None)
    sys.modules.update(saved)


def test_install_serves_imports(installed):  # tests/test_compat.py:28-41
    from knn_cuda import KNN
    from pointnet2_ops import pointnet2_utils
    import pointnet2_ops.pointnet2_utils as direct

    from torch_cluster import fps, knn as flat_knn, knn_graph, radius, radius_graph

    assert direct is pointnet2_utils
    assert pointnet2_utils.furthest_point_sample is compat.furthest_point_sample
    assert pointnet2_utils.ball_query is compat.ball_query
    assert KNN is compat.KNN
    assert fps is compat.flat.fps and flat_knn is compat.flat.knn
    assert radius is compat.flat.radius
    assert knn_graph is compat.flat.knn_graph and radius_graph is compat.flat.radius_graph
    assert compat.importlib.util.find_spec("torch_cluster") is not None


def test_install_leaves_existing_modules_alone(installed):  # tests/test_compat.py:44-52
    marker = object()
    sys.modules["knn_cuda"] = marker
    assert "knn_cuda" not in compat.install()
    assert sys.modules["knn_cuda"] is marker

    sys.modules["torch_cluster"] = marker
    assert "torch_cluster" not in compat.install()
    assert sys.modules["torch_cluster"] is marker


def test_gather_and_grouping_operations():  # tests/test_compat.py:121-137
    features = torch.randn(2, 4, 30)
    idx = torch.randint(0, 30, (2, 7), dtype=torch.int32)
    out = compat.gather_operation(features, idx)
    assert out.shape == (2, 4, 7)
    assert torch.equal(out[1, :, 3], features[1, :, idx[1, 3]])
    gidx = torch.randint(0, 30, (2, 7, 5), dtype=torch.int32)
    out = compat.grouping_operation(features, gidx)
    assert out.shape == (2, 4, 7, 5)
    assert torch.equal(out[0, :, 6, 2], features[0, :, gidx[0, 6, 2]])
    f = torch.randn(1, 3, 10, requires_grad=True)
    compat.gather_operation(f, torch.tensor([[2, 2, 5]])).sum().backward()
    assert f.grad[0, 0].tolist() == [0, 0, 2, 0, 0, 1, 0, 0, 0, 0]
