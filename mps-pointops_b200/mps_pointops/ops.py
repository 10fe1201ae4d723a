"""Point-cloud search ops on B200: FPS, kNN and ball query.

Drop-in for ``mps_pointops.ops`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/ops.py:53-227): the same signatures, defaults, return types,
validation order, exception types and messages.  Where the reference sends
MPS tensors to Metal kernels, this module sends CUDA tensors to the sm_100a
kernels of libmpo_b200.so through the C ABI in include/mpo_b200.h.  Tensors on
any other device are rejected after validation with ``RuntimeError`` -- this
build does not compute on the CPU.
"""

from __future__ import annotations

from typing import Literal

import torch
from torch import Tensor

from . import _native as N
from ._ball_query_cuda import _checked_radius_and_k, ball_query as _cuda_ball_query

# The CUDA kernels rank at most this many neighbours per query
# (the reference's Metal limit, mps_pointops/ops.py:28-30).
_KNN_MAX_K = 256
_FPS_STRATEGIES = {"auto": 0, "single": 1, "multigroup": 2}


def furthest_point_sample(
    xyz: Tensor,
    npoint: int,
    start_idx: int = 0,
    skip_near_origin: bool = False,
    *,
    strategy: Literal["auto", "single", "multigroup"] = "auto",
) -> Tensor:
    """Farthest point sampling (mps_pointops/ops.py:53-141).

    Sampling starts at ``start_idx``; each next sample is the point whose
    squared distance to the samples so far is largest, ties going to the
    smaller index; once every point has been taken, index 0 repeats.

    Args:
        xyz: (B, N, 3) float32 CUDA tensor.
        npoint: number of samples.
        start_idx: first sampled index.
        skip_near_origin: never pick points with x^2 + y^2 + z^2 <= 1e-3
            (other than the start), like pointnet2_ops.
        strategy: ``auto`` picks by size (one CTA per cloud up to 8192 points,
            a cooperative CTA group above); ``single`` forces the one-CTA path
            and ``multigroup`` the CTA-group path, for measurement.

    Returns:
        (B, npoint) int64 indices.
    """
    return _fps(xyz, npoint, start_idx, skip_near_origin, strategy, out_dtype=torch.long)


def _fps(xyz, npoint, start_idx, skip_near_origin, strategy, out_dtype):
    if xyz.dim() != 3 or xyz.shape[-1] != 3:
        raise ValueError(f"xyz must have shape (B, N, 3), got {tuple(xyz.shape)}")
    if strategy not in _FPS_STRATEGIES:
        raise ValueError(f"strategy must be auto, single, or multigroup, got {strategy!r}")
    B, Np, _ = xyz.shape
    if npoint < 0:
        raise ValueError(f"npoint must be >= 0, got {npoint}")
    if npoint > 0 and Np == 0:
        raise ValueError("cannot sample from an empty point cloud")
    if npoint > 0 and not 0 <= start_idx < Np:
        raise IndexError(f"start_idx {start_idx} is out of range for {Np} points")
    N.require_cuda(xyz, "furthest_point_sample")
    if xyz.dtype != torch.float32:
        raise TypeError(f"xyz must be float32 on CUDA, got {xyz.dtype}")
    if strategy == "multigroup" and B > 1 and npoint > 1:
        raise ValueError("multigroup FPS requires batch size 1; use auto or single for batches")
    if strategy == "single" and Np > 8192:
        raise ValueError("single-CTA FPS holds at most 8192 points; use auto or multigroup")
    out = torch.empty((B, npoint), dtype=out_dtype, device=xyz.device)
    if B == 0 or npoint == 0:
        return out
    xyz = xyz.contiguous()
    code = _FPS_STRATEGIES[strategy]
    lib = N.lib()
    with N.on_device(xyz.device):
        ws = N.workspace(lib.mpo_fps_workspace_bytes(B, Np, npoint, code), xyz.device)
        N.check(lib.mpo_fps(N.ptr(xyz), B, Np, npoint, start_idx, int(bool(skip_near_origin)),
                            int(out_dtype == torch.int32), code, N.ptr(out), None, N.ptr(ws),
                            0 if ws is None else ws.numel(), N.stream(xyz.device)),
                "furthest_point_sample")
    return out


def knn(query: Tensor, ref: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """Brute-force k nearest neighbours in coordinate or feature space
    (mps_pointops/ops.py:144-205).

    Neighbours are sorted by float32 squared distance (accumulated in
    dimension order, no FMA), then by index; distances are Euclidean, the
    square root taken after selection.  ``k`` is at most 256.  No gradients.

    Args:
        query: (B, M, D) float32, D >= 1.
        ref: (B, N, D) float32.
        k: number of neighbours, 0 <= k <= N.

    Returns:
        dist (B, M, k) float32 and idx (B, M, k) int64.
    """
    if query.dim() != 3 or query.shape[-1] < 1:
        raise ValueError(f"query must have shape (B, M, D) with D >= 1, got {tuple(query.shape)}")
    if ref.dim() != 3 or ref.shape[-1] != query.shape[-1]:
        raise ValueError(f"ref must have shape (B, N, {query.shape[-1]}), got {tuple(ref.shape)}")
    if query.device != ref.device:
        raise ValueError(f"query and ref are on different devices: {query.device} and {ref.device}")
    if query.shape[0] != ref.shape[0]:
        raise ValueError(f"batch sizes differ: {query.shape[0]} and {ref.shape[0]}")
    B, M, D = query.shape
    Nr = ref.shape[1]
    if not 0 <= k <= Nr:
        raise ValueError(f"k must be in [0, {Nr}], got {k}")
    N.require_cuda(query, "knn")
    if query.dtype != torch.float32 or ref.dtype != torch.float32:
        raise TypeError(f"query and ref must be float32 on CUDA, got {query.dtype} and {ref.dtype}")
    if k > _KNN_MAX_K:
        raise ValueError(f"k must be at most {_KNN_MAX_K} on CUDA, got {k}; use CPU for larger k")
    if M >= 2**31 or Nr >= 2**31:
        raise ValueError("M and N must each be below 2**31 for the CUDA kNN kernel")
    dist = torch.empty(B, M, k, dtype=torch.float32, device=query.device)
    idx = torch.empty(B, M, k, dtype=torch.long, device=query.device)
    if B == 0 or M == 0 or k == 0:
        return dist, idx
    query, ref = query.contiguous(), ref.contiguous()
    with N.on_device(query.device):
        lib = N.lib()
        ws_bytes = int(lib.mpo_knn_workspace_bytes(B, M, Nr, D, k))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=query.device) if ws_bytes else None
        N.check(lib.mpo_knn(N.ptr(query), N.ptr(ref), B, M, Nr, D, k, N.ptr(dist), N.ptr(idx),
                            None, N.ptr(ws), ws_bytes, N.stream(query.device)), "knn")
    return dist, idx


def ball_query(query: Tensor, ref: Tensor, radius: float, K: int) -> tuple[Tensor, Tensor]:
    """First-K radius search with squared distances and -1 padded indices
    (mps_pointops/ops.py:208-227).

    Shapes (B, M, 3), (B, N, 3) -> (B, M, K).  The radius and K rules are
    checked before the device, so every device accepts and rejects the same
    arguments.  CUDA float32/float16 inputs use the native kernel and support
    coordinate gradients.
    """
    _checked_radius_and_k(radius, K)
    if query.device.type == "cuda" or ref.device.type == "cuda":
        result = _cuda_ball_query(query, ref, radius=radius, k=K)
        return result.distances, result.indices
    if query.dim() != 3 or ref.dim() != 3 or query.shape[-1] != 3 or ref.shape[-1] != 3:
        raise ValueError("query and ref must have shapes (B, M, 3) and (B, N, 3)")
    if query.shape[0] != ref.shape[0]:
        raise ValueError("query and ref must have the same batch size")
    if query.device != ref.device:
        raise ValueError(f"query and ref are on different devices: {query.device} and {ref.device}")
    N.require_cuda(query, "ball_query")
    raise AssertionError("unreachable")  # pragma: no cover
