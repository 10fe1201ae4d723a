"""Stand-ins for ``pointnet2_ops`` and ``knn_cuda`` backed by the B200 kernels.

Drop-in for the pointnet2_ops / knn_cuda part of ``mps_pointops.compat`` of
gamzerA/mps-pointops v1.0.0 (mps_pointops/compat.py:53-172)::

    import mps_pointops.compat
    mps_pointops.compat.install()

    from pointnet2_ops import pointnet2_utils   # served by mps_pointops
    from knn_cuda import KNN

``install()`` registers ``pointnet2_ops``, ``pointnet2_ops.pointnet2_utils``,
``knn_cuda`` and ``torch_cluster`` in ``sys.modules``; a name that is already
importable (the real package) is left alone unless ``force=True``.  The
``torch_cluster`` stand-in serves ``fps``, ``knn``, ``radius``, ``knn_graph``
and ``radius_graph`` from :mod:`mps_pointops.flat`; the reference's clustering
and random-walk entries (``grid_cluster``, ``graclus_cluster``,
``random_walk``, ``nearest``) are not part of this build.  ``pointcept=True``
also registers the Pointcept v1.2.1 ``pointops`` subset of
:mod:`mps_pointops.pointcept` (compat.py:161-171).

The pointnet2_ops FPS and ball query run as fused kernels here: FPS writes its
int32 indices directly, and the ball query applies pointnet2's first-hit
padding inside the search kernel.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from importlib.machinery import ModuleSpec

import torch
from torch import Tensor

from . import _native as N
from . import flat, grouping, ops
from . import pointcept as pointcept_ops
from ._ball_query_cuda import _checked_radius_and_k


# ---------------------------------------------------------------- pointnet2_ops


def furthest_point_sample(xyz: Tensor, npoint: int) -> Tensor:
    """Like ``pointnet2_ops.pointnet2_utils.furthest_point_sample``
    (mps_pointops/compat.py:53-59): (B, N, 3) float32 -> (B, npoint) int32,
    starting at index 0 and never picking points with x^2 + y^2 + z^2 <= 1e-3."""
    out = ops._fps(xyz, npoint, 0, True, "auto", out_dtype=torch.int32)
    out._mpo_index_bound = xyz.shape[1]  # valid indices: gather_operation skips its check
    return out


# gather_operation / grouping_operation (mps_pointops/compat.py:62-73) run on
# the grouping kernels for float32 CUDA tensors; QueryAndGroup / GroupAll are
# the pointnet2_ops modules on the fused grouping kernel.
gather_operation = grouping.gather_operation
grouping_operation = grouping.grouping_operation
QueryAndGroup = grouping.QueryAndGroup
GroupAll = grouping.GroupAll


def ball_query(radius: float, nsample: int, xyz: Tensor, new_xyz: Tensor) -> Tensor:
    """Like ``pointnet2_utils.ball_query`` (mps_pointops/compat.py:76-85):
    (B, N, 3), (B, npoint, 3) -> (B, npoint, nsample) int32 holding the first
    ``nsample`` points in input order with squared distance < radius**2;
    empty slots repeat the first hit, and a query without hits is all zeros."""
    _, radius_sq = _checked_radius_and_k(radius, nsample)
    if xyz.dim() != 3 or new_xyz.dim() != 3 or xyz.shape[-1] != 3 or new_xyz.shape[-1] != 3:
        raise ValueError("query and ref must have shapes (B, M, 3) and (B, N, 3)")
    if xyz.shape[0] != new_xyz.shape[0]:
        raise ValueError("query and ref must have the same batch size")
    if xyz.device != new_xyz.device:
        raise ValueError(f"query and ref are on different devices: {new_xyz.device} and {xyz.device}")
    N.require_cuda(xyz, "ball_query")
    if xyz.dtype != torch.float32 or new_xyz.dtype != torch.float32:
        # Other dtypes take the general path (float16 is widened exactly).
        _, idx = ops.ball_query(new_xyz, xyz, radius, nsample)
        first = idx[..., :1].clamp(min=0)
        return torch.where(idx >= 0, idx, first).int()
    B, Np, _ = xyz.shape
    npoint = new_xyz.shape[1]
    out = torch.empty((B, npoint, nsample), dtype=torch.int32, device=xyz.device)
    if out.numel():
        a, q = xyz.contiguous(), new_xyz.contiguous()
        with N.on_device(xyz.device):
            N.check(N.lib().mpo_ball_query_pointnet2(N.ptr(a), N.ptr(q), B, Np, npoint, nsample,
                                                     radius_sq, N.ptr(out),
                                                     N.stream(xyz.device)), "ball_query")
    # Every index lies in [0, N) (or is 0): grouping_operation can skip its
    # bounds check on this tensor.
    out._mpo_index_bound = Np
    return out


# ---------------------------------------------------------------- knn_cuda


class KNN(torch.nn.Module):
    """Like ``knn_cuda.KNN`` (mps_pointops/compat.py:91-112).

    With ``transpose_mode=True`` ``ref`` is (B, N, D) and ``query`` (B, M, D)
    and both outputs are (B, M, k); otherwise inputs are (B, D, N) / (B, D, M)
    and outputs (B, k, M).  ``dist`` is Euclidean.  No gradients flow.
    """

    def __init__(self, k: int, transpose_mode: bool = False):
        super().__init__()
        self.k = k
        self.transpose_mode = transpose_mode

    def forward(self, ref: Tensor, query: Tensor) -> tuple[Tensor, Tensor]:
        if not self.transpose_mode:
            ref, query = ref.transpose(1, 2), query.transpose(1, 2)
        with torch.no_grad():
            dist, idx = ops.knn(query.float(), ref.float(), self.k)
        if not self.transpose_mode:
            dist, idx = dist.transpose(1, 2), idx.transpose(1, 2)
        return dist, idx


# ---------------------------------------------------------------- install


def _module(name: str, **attrs) -> types.ModuleType:
    module = types.ModuleType(name)
    module.__dict__.update(attrs)
    module.__spec__ = ModuleSpec(name, loader=None, is_package="__path__" in attrs)
    return module


def install(force: bool = False, *, pointcept: bool = False) -> list[str]:
    """Register the stand-ins in ``sys.modules``; returns the names added."""
    pointnet2_utils = _module(
        "pointnet2_ops.pointnet2_utils",
        furthest_point_sample=furthest_point_sample,
        gather_operation=gather_operation,
        grouping_operation=grouping_operation,
        ball_query=ball_query,
        QueryAndGroup=QueryAndGroup,
        GroupAll=GroupAll,
    )
    packages = {
        "pointnet2_ops": {
            "pointnet2_ops": _module("pointnet2_ops", pointnet2_utils=pointnet2_utils, __path__=[]),
            "pointnet2_ops.pointnet2_utils": pointnet2_utils,
        },
        "knn_cuda": {"knn_cuda": _module("knn_cuda", KNN=KNN)},
        "torch_cluster": {
            "torch_cluster": _module(
                "torch_cluster",
                fps=flat.fps,
                knn=flat.knn,
                radius=flat.radius,
                knn_graph=flat.knn_graph,
                radius_graph=flat.radius_graph,
            )
        },
    }
    if pointcept:
        packages["pointops"] = {
            "pointops": _module(
                "pointops",
                farthest_point_sampling=pointcept_ops.farthest_point_sampling,
                knn_query=pointcept_ops.knn_query,
                grouping=pointcept_ops.grouping,
                knn_query_and_group=pointcept_ops.knn_query_and_group,
                interpolation=pointcept_ops.interpolation,
            ),
        }
    installed = []
    for top, modules in packages.items():
        if not force and (top in sys.modules or importlib.util.find_spec(top) is not None):
            continue
        sys.modules.update(modules)
        installed.extend(modules)
    return installed
