"""SpatialIndex argument checks (mps_pointops/spatial.py:96-136 of the reference)."""

from __future__ import annotations

import pytest
import torch

from mps_pointops.spatial import SpatialIndex


def test_constructor_checks():
    pts = torch.rand(10, 3)
    with pytest.raises(ValueError, match=r"shape \[N, 3\]"):
        SpatialIndex(torch.rand(10, 2))
    with pytest.raises(ValueError, match="backend"):
        SpatialIndex(pts, backend="tree")
    with pytest.raises(ValueError, match="origin"):
        SpatialIndex(pts, origin=torch.zeros(2))
    with pytest.raises(ValueError, match="cell_size"):
        SpatialIndex(pts, cell_size=0.0)
    index = SpatialIndex(pts, backend="scan")
    with pytest.raises(ValueError, match=r"shape \[Q, 3\]"):
        index.knn(torch.rand(3, 2), 1)
    with pytest.raises(TypeError, match="same dtype"):
        index.knn(pts.double(), 1)
    with pytest.raises(ValueError, match="k must be in"):
        index.knn(pts, 11)
    with pytest.raises(ValueError, match="parallel_microtrees"):
        index.knn(pts, 1, parallel_microtrees=True)
    with pytest.raises(ValueError, match="grid backend needs float32 CUDA"):
        SpatialIndex(pts, backend="grid").knn(pts, 1)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        index.knn(pts, 1)
    assert SpatialIndex(pts)._selected_backend(4, None) == "scan"   # CPU -> scan
