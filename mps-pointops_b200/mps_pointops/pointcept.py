"""Pointcept v1.2.1 ``pointops`` subset (Point Transformer V1) on B200.

Drop-in for ``mps_pointops.pointcept`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/pointcept.py:1-246): ``farthest_point_sampling``, ``knn_query``,
``grouping``, ``knn_query_and_group`` and ``interpolation`` with the same
signatures, return types, padding rules and validation messages.
Coordinates and features are flat point rows; offsets are inclusive
cumulative counts per batch (``[4, 9]`` = rows 0-3 and 4-8).

Where the reference loops over the batches in Python and calls its
per-cloud FPS and kNN once per batch (pointcept.py:77-165), this module
issues ONE flat launch for all batches: ``mpo_flat_fps`` (starts at each
batch's first point) and ``mpo_flat_knn`` (lowest index on equal squared
distances, non-finite distances dropped).  The padding rules of the
upstream CUDA heap stay as the reference states them (pointcept.py:17-18,
141-153): a slot is valid only when its squared distance, recomputed from
the selected coordinates as ((dx*dx + dy*dy) + dz*dz), is below 1e10;
missing slots hold index -1 and distance 1e5.  Grouping is one native row
gather per part written into the concatenated output in place
(``mpo_gather_rows``: relative coordinates, then features, zero rows for -1
slots), and interpolation one native pass that forms the inverse-distance
weights and their weighted sum (``mpo_flat_interpolate``), with native
scatter backwards (pointcept.py:168-243).

Inputs are validated as the reference does (shape, dtype, offsets) on CPU
or CUDA tensors; the computation itself runs on CUDA only and raises
``RuntimeError`` for tensors on any other device.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _native as N
from . import flat
from ._rows import FlatInterpolate, GroupRows

_PAD_SQUARED_DISTANCE = 1e10  # the upstream CUDA heap's strict ceiling
_PAD_DISTANCE = 100_000.0  # sqrt(1e10): the upstream unfilled distance
_CUDA_KNN_MAX_K = 256


def _points(value: Tensor, name: str) -> None:
    if not isinstance(value, Tensor) or value.ndim != 2 or value.shape[1] != 3:
        raise ValueError(f"{name} must be a tensor of shape (N, 3)")
    if value.dtype != torch.float32 or value.device.type not in ("cpu", "cuda"):
        raise ValueError(f"{name} must be float32 on CPU or CUDA")


def _offsets(value: Tensor, count: int | None, device: torch.device, name: str) -> list[int]:
    """Inclusive cumulative ends -> [0, *ends] on the host (pointcept.py:46-56)."""
    if not isinstance(value, Tensor) or value.ndim != 1 or value.dtype not in (torch.int32,
                                                                                 torch.int64):
        raise ValueError(f"{name} must be a one-dimensional int32/int64 tensor")
    if value.device != device:
        raise ValueError(f"{name} must be on {device}")
    ends = value.tolist()
    if count is not None and ((ends and ends[-1] != count) or (not ends and count != 0)):
        raise ValueError(f"{name} must end at its point count ({count})")
    if any(end < start for start, end in zip((0, *ends[:-1]), ends)):
        raise ValueError(f"{name} must be nondecreasing and nonnegative")
    return [0, *ends]


def _pairs(xyz: Tensor, offset: Tensor, new_xyz: Tensor | None,
           new_offset: Tensor | None) -> tuple[Tensor, list[int], list[int]]:
    _points(xyz, "xyz")
    if new_xyz is None and new_offset is None:
        new_xyz, new_offset = xyz, offset
    elif new_xyz is None or new_offset is None:
        raise ValueError("new_xyz and new_offset must be provided together")
    _points(new_xyz, "new_xyz")
    if xyz.device != new_xyz.device:
        raise ValueError("xyz and new_xyz must be on the same device")
    ref_ends = _offsets(offset, len(xyz), xyz.device, "offset")
    query_ends = _offsets(new_offset, len(new_xyz), xyz.device, "new_offset")
    if len(ref_ends) != len(query_ends):
        raise ValueError("offset and new_offset must have the same batch count")
    return new_xyz, ref_ends, query_ends


def farthest_point_sampling(xyz: Tensor, offset: Tensor, new_offset: Tensor) -> Tensor:
    """Global int32 FPS indices, each batch starting at its first point
    (pointcept.py:77-98).  ``offset`` and ``new_offset`` are same-length
    cumulative int32/int64 vectors; a batch may request at most its point
    count.  Equal distances go to the smaller index.  One flat launch serves
    every batch."""
    _points(xyz, "xyz")
    source = _offsets(offset, len(xyz), xyz.device, "offset")
    target = _offsets(new_offset, None, xyz.device, "new_offset")
    if len(source) != len(target):
        raise ValueError("offset and new_offset must have the same batch count")
    for lo, hi, out_lo, out_hi in zip(source, source[1:], target, target[1:]):
        if out_hi - out_lo > hi - lo:
            raise ValueError("a batch requests more FPS samples than input points")
    total = target[-1]
    if total == 0:
        return torch.empty(0, dtype=torch.int32, device=xyz.device)
    N.require_cuda(xyz, "pointcept.farthest_point_sampling")
    device = xyz.device
    segments = len(source) - 1
    max_len = max(hi - lo for lo, hi in zip(source, source[1:]))
    ptr = torch.tensor(source, dtype=torch.long).to(device, non_blocking=True)
    out_ptr = torch.tensor(target, dtype=torch.long).to(device, non_blocking=True)
    starts = torch.zeros(segments, dtype=torch.long, device=device)
    out = torch.empty(total, dtype=torch.long, device=device)
    status = torch.empty(1, dtype=torch.int32, device=device)
    points = xyz.contiguous()
    with N.on_device(device):
        lib = N.lib()
        ws_bytes = int(lib.mpo_flat_fps_workspace_bytes(segments, max_len))
        ws = N.workspace(ws_bytes, device)
        N.check(lib.mpo_flat_fps(N.ptr(points), N.ptr(ptr), N.ptr(out_ptr), N.ptr(starts),
                                 segments, len(xyz), total, max_len, N.ptr(out), N.ptr(status),
                                 N.ptr(ws), ws_bytes, N.stream(device)),
                "pointcept farthest_point_sampling")
    if max_len > 8192:
        flat._raise_status(status, "fps")
    return out.to(torch.int32)


def _selected_squared(query: Tensor, refs: Tensor, idx: Tensor) -> Tensor:
    """((dx*dx + dy*dy) + dz*dz) of each query and its selected rows, each
    operation rounded on its own (pointcept.py:146-149); idx must be >= 0."""
    delta = query[:, None, :] - refs[idx]
    squared = delta[..., 0] * delta[..., 0]
    squared = squared + delta[..., 1] * delta[..., 1]
    return squared + delta[..., 2] * delta[..., 2]


def knn_query(nsample: int, xyz: Tensor, offset: Tensor, new_xyz: Tensor | None = None,
              new_offset: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """Global int32 neighbours and float32 Euclidean distances, (M, nsample)
    (pointcept.py:101-165).

    Neighbours are in ascending (squared distance, index) order within each
    query's batch.  A slot without a neighbour -- fewer references in the
    batch, an empty reference batch, a non-finite distance, or a squared
    distance of at least 1e10 -- holds index -1 and distance 1e5.  The result
    carries no autograd history.
    """
    if isinstance(nsample, bool) or not isinstance(nsample, int) or nsample < 0:
        raise ValueError("nsample must be a nonnegative integer")
    new_xyz, source, target = _pairs(xyz, offset, new_xyz, new_offset)
    if nsample > _CUDA_KNN_MAX_K and xyz.device.type == "cuda":
        raise ValueError(f"CUDA kNN supports at most {_CUDA_KNN_MAX_K} neighbors")
    device = xyz.device
    queries = len(new_xyz)
    if queries == 0 or nsample == 0:
        return (torch.empty((queries, nsample), dtype=torch.int32, device=device),
                torch.empty((queries, nsample), dtype=torch.float32, device=device))
    N.require_cuda(xyz, "pointcept.knn_query")
    with torch.no_grad():
        if len(xyz) == 0:
            return (torch.full((queries, nsample), -1, dtype=torch.int32, device=device),
                    torch.full((queries, nsample), _PAD_DISTANCE, dtype=torch.float32,
                               device=device))
        refs = xyz.detach().contiguous()
        query = new_xyz.detach().contiguous()
        ptr_x = torch.tensor(source, dtype=torch.long).to(device, non_blocking=True)
        ptr_y = torch.tensor(target, dtype=torch.long).to(device, non_blocking=True)
        # Offsets were validated on the host above.
        idx = flat.knn_indices(refs, query, ptr_x, ptr_y, nsample, check=False)
        selected = idx >= 0
        squared = _selected_squared(query, refs, torch.where(selected, idx, 0))
        valid = selected & (squared < _PAD_SQUARED_DISTANCE)
        dist = torch.where(valid, torch.sqrt(squared), _PAD_DISTANCE)
        return torch.where(valid, idx, -1).to(torch.int32), dist


def grouping(idx: Tensor, feat: Tensor, xyz: Tensor, new_xyz: Tensor | None = None,
             with_xyz: bool = False) -> Tensor:
    """Gather (N, C) features into (M, K, C), zero for ``-1`` slots; with
    ``with_xyz`` the relative positions come first, (M, K, 3 + C)
    (pointcept.py:168-203).  Gradients reach the features and, for valid
    slots, both point sets."""
    _points(xyz, "xyz")
    if not isinstance(feat, Tensor) or feat.ndim != 2 or len(feat) != len(xyz):
        raise ValueError("feat must have shape (N, C) matching xyz")
    if feat.dtype != torch.float32 or feat.device != xyz.device:
        raise ValueError("feat must be float32 on the xyz device")
    if not isinstance(idx, Tensor) or idx.ndim != 2 or idx.dtype not in (torch.int32,
                                                                         torch.int64):
        raise ValueError("idx must be a two-dimensional int32/int64 tensor")
    if idx.device != xyz.device:
        raise ValueError("idx must be on the xyz device")
    if bool(((idx < -1) | (idx >= len(xyz))).any()):
        raise ValueError("idx contains an out-of-range point index")
    N.require_cuda(xyz, "pointcept.grouping")
    if with_xyz:
        if new_xyz is None:
            new_xyz = xyz
        _points(new_xyz, "new_xyz")
        if new_xyz.device != xyz.device or len(new_xyz) != len(idx):
            raise ValueError("new_xyz must have one row per idx row on the xyz device")
    # One native gather per part, written into the concatenated output in
    # place (mpo_gather_rows): relative coordinates, then the features.
    return GroupRows.apply(feat, xyz, new_xyz if with_xyz else xyz, idx, with_xyz)


def knn_query_and_group(feat: Tensor, xyz: Tensor, offset: Tensor | None = None,
                        new_xyz: Tensor | None = None, new_offset: Tensor | None = None,
                        idx: Tensor | None = None, nsample: int | None = None,
                        with_xyz: bool = False) -> tuple[Tensor, Tensor]:
    """kNN when ``idx`` is absent, then ``grouping`` (pointcept.py:206-216)."""
    if idx is None:
        if offset is None or nsample is None:
            raise ValueError("offset and nsample are required when idx is absent")
        idx, _ = knn_query(nsample, xyz, offset, new_xyz, new_offset)
    return grouping(idx, feat, xyz, new_xyz, with_xyz), idx


def interpolation(xyz: Tensor, new_xyz: Tensor, feat: Tensor, offset: Tensor,
                  new_offset: Tensor, k: int = 3) -> Tensor:
    """Inverse-distance interpolation of (N, C) features to the new points
    over their k nearest (pointcept.py:219-243).  ``-1`` neighbours weigh
    zero; a query whose reference batch is empty gets zeros.  The weights are
    fixed for autograd (no coordinate gradient)."""
    if not isinstance(feat, Tensor) or feat.ndim != 2 or len(feat) != len(xyz):
        raise ValueError("feat must have shape (N, C) matching xyz")
    if feat.dtype != torch.float32 or feat.device != xyz.device:
        raise ValueError("feat must be float32 on the xyz device")
    idx, dist = knn_query(k, xyz, offset, new_xyz, new_offset)
    # Weights and the weighted sum in one native pass (mpo_flat_interpolate).
    return FlatInterpolate.apply(feat, idx, dist)


__all__ = [
    "farthest_point_sampling", "knn_query", "grouping", "knn_query_and_group",
    "interpolation",
]
