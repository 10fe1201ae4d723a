"""PyTorch3D-style Ball Query call surface on the B200 kernels.

Drop-in for ``mps_pointops.pytorch3d`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/pytorch3d.py:1-125): ``ball_query(p1, p2, lengths1, lengths2,
K, radius, return_nn, skip_points_outside_cube)`` returning
``KNN(dists, idx, knn)``, with the same argument checks and messages.  The
search is the first-K ball query of ``mps_pointops.ball_query`` (the
``mpo_ball_query`` kernel, ragged lengths honoured on the device); the
returned neighbour coordinates come from the native row gather
(``mpo_gather_rows``: zero rows for ``-1`` slots, gradients to ``p2``).  Import it
explicitly: ``from mps_pointops.pytorch3d import ball_query``.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from . import _native as N
from ._rows import GatherRows
from ._ball_query_cuda import _checked_radius_and_k
from ._ball_query_cuda import ball_query as _cuda_ball_query


class KNN(NamedTuple):
    """PyTorch3D-style ``(dists, idx, knn)`` result."""

    dists: torch.Tensor
    idx: torch.Tensor
    knn: torch.Tensor | None


def ball_query(
    p1: torch.Tensor,
    p2: torch.Tensor,
    lengths1: torch.Tensor | None = None,
    lengths2: torch.Tensor | None = None,
    K: int = 500,
    radius: float = 0.2,
    return_nn: bool = True,
    skip_points_outside_cube: bool = False,
) -> KNN:
    """Find the first ``K`` points of ``p2`` inside each ``p1`` ball
    (mps_pointops/pytorch3d.py:67-125).

    ``p1`` (B, Q, 3) and ``p2`` (B, P, 3) are float32 CUDA tensors; lengths,
    when given, are int64 (B,) tensors on the same device.  ``dists`` holds
    squared distances, ``idx`` point indices in input order with ``-1``
    padding, and ``knn`` (when ``return_nn``) the gathered coordinates with
    zero padding.  ``skip_points_outside_cube`` is accepted as a hint and does
    not change the result.
    """
    if not isinstance(p1, torch.Tensor) or not isinstance(p2, torch.Tensor):
        raise TypeError("p1 and p2 must be torch.Tensor values")
    if p1.ndim != 3 or p2.ndim != 3 or p1.shape[-1] != 3 or p2.shape[-1] != 3:
        raise ValueError("p1 and p2 must have shapes (B, Q, 3) and (B, P, 3)")
    if p1.shape[0] != p2.shape[0]:
        raise ValueError("p1 and p2 must have the same batch dimension")
    if p1.device != p2.device:
        raise ValueError("p1 and p2 must be on the same device")
    if p1.dtype != torch.float32 or p2.dtype != torch.float32:
        raise TypeError("PyTorch3D-style Ball Query currently requires float32 coordinates")
    if not isinstance(return_nn, bool) or not isinstance(skip_points_outside_cube, bool):
        raise TypeError("return_nn and skip_points_outside_cube must be bool")
    _checked_radius_and_k(radius, K)
    N.require_cuda(p1, "pytorch3d.ball_query")
    result = _cuda_ball_query(p1, p2, radius=radius, k=K, query_lengths=lengths1,
                              point_lengths=lengths2)
    dists, idx = result.distances, result.indices
    # Neighbour coordinates: one native gather, zero rows for -1 slots,
    # gradients scattered back to p2 (mpo_gather_rows).
    knn = GatherRows.apply(p2, idx) if return_nn else None
    return KNN(dists=dists, idx=idx, knn=knn)


__all__ = ["KNN", "ball_query"]
