"""mps_pointops for NVIDIA B200 (sm_100a).

A drop-in for the point-cloud hot path of gamzerA/mps-pointops v1.0.0
(mps_pointops/__init__.py:3-13): farthest point sampling, kNN (xyz and
feature space), ball query, three_nn / three_interpolate, squared-L2
Chamfer distance, the flat (ragged-batch) torch_cluster API, the Pointcept
``pointops`` subset and the grid-accelerated ``SpatialIndex``, computed by the
hand-written CUDA kernels of
libmpo_b200.so (C ABI: include/mpo_b200.h).  CUDA tensors only; there is no
CPU or library fallback.
"""

from . import compat, dist, flat, grouping, pointcept, pyg
from .chamfer import chamfer_distance
from .ops import ball_query, furthest_point_sample, knn
from .pointnet2 import three_interpolate, three_nn
from .spatial import SpatialIndex

__all__ = [
    "ball_query", "chamfer_distance", "compat", "dist", "flat", "furthest_point_sample",
    "grouping", "knn", "pointcept", "pyg", "three_interpolate", "three_nn", "SpatialIndex",
]
__version__ = "1.0.0+b200"
