"""PointNet++ three-neighbour search and weighted feature propagation on B200.

Drop-in for ``mps_pointops.pointnet2`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/pointnet2.py:30-214): the same shapes (those of
``pointnet2_ops.pointnet2_utils``), validation, error types and autograd
contract, computed by the sm_100a kernels of libmpo_b200.so.
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import _native as N

_MAX_INDEX = (1 << 31) - 1


def _validate_three_nn(unknown: Tensor, known: Tensor) -> tuple[int, int, int]:
    """mps_pointops/pointnet2.py:30-51."""
    if not isinstance(unknown, Tensor) or not isinstance(known, Tensor):
        raise TypeError("unknown and known must be tensors")
    if unknown.ndim != 3 or unknown.shape[-1] != 3:
        raise ValueError("unknown must have shape (B, N, 3)")
    if known.ndim != 3 or known.shape[-1] != 3:
        raise ValueError("known must have shape (B, M, 3)")
    if unknown.shape[0] != known.shape[0]:
        raise ValueError("unknown and known must have the same batch size")
    if unknown.device != known.device:
        raise ValueError("unknown and known must be on the same device")
    if unknown.dtype != torch.float32 or known.dtype != torch.float32:
        raise TypeError("unknown and known must be float32")
    batch, queries, _ = unknown.shape
    points = known.shape[1]
    if batch and queries and points < 3:
        raise ValueError("three_nn needs at least 3 known points for nonempty queries")
    if points > _MAX_INDEX:
        raise ValueError("three_nn supports at most 2**31-1 known points")
    if batch * queries > (1 << 32) - 1:
        raise ValueError("three_nn query count exceeds the native index range")
    return batch, queries, points


def three_nn(unknown: Tensor, known: Tensor) -> tuple[Tensor, Tensor]:
    """Three nearest known points of every unknown point (pointnet2.py:75-100).

    ``unknown`` (B,N,3) and ``known`` (B,M,3) float32 CUDA tensors, M >= 3
    whenever B*N > 0.  Returns Euclidean distances (B,N,3) float32 and known
    indices (B,N,3) int32, ordered by squared distance with the smaller index
    first on equal squared distances.  No coordinate gradient.
    """
    batch, queries, points = _validate_three_nn(unknown, known)
    N.require_cuda(unknown, "three_nn")
    distances = torch.empty((batch, queries, 3), dtype=torch.float32, device=unknown.device)
    indices = torch.empty((batch, queries, 3), dtype=torch.int32, device=unknown.device)
    if batch * queries:
        u, k = unknown.detach().contiguous(), known.detach().contiguous()
        with N.on_device(unknown.device):
            N.check(N.lib().mpo_three_nn(N.ptr(u), N.ptr(k), batch, queries, points,
                                         N.ptr(distances), N.ptr(indices),
                                         N.stream(unknown.device)), "three_nn")
    return distances, indices


def _validate_interpolate(features: Tensor, indices: Tensor, weights: Tensor):
    """mps_pointops/pointnet2.py:103-132, except the bounds check on the
    caller-supplied indices, which _queue_index_check runs on the device."""
    if not all(isinstance(t, Tensor) for t in (features, indices, weights)):
        raise TypeError("features, indices, and weights must be tensors")
    if features.ndim != 3:
        raise ValueError("features must have shape (B, C, M)")
    if indices.ndim != 3 or indices.shape[-1] != 3:
        raise ValueError("indices must have shape (B, N, 3)")
    if weights.shape != indices.shape:
        raise ValueError("weights must have the same (B, N, 3) shape as indices")
    if features.shape[0] != indices.shape[0]:
        raise ValueError("features and indices must have the same batch size")
    if features.device != indices.device or features.device != weights.device:
        raise ValueError("features, indices, and weights must be on the same device")
    if features.dtype != torch.float32 or weights.dtype != torch.float32:
        raise TypeError("features and weights must be float32")
    if indices.dtype not in (torch.int32, torch.int64):
        raise TypeError("indices must be int32 or int64")
    batch, channels, points = features.shape
    queries = indices.shape[1]
    if batch and queries and points == 0:
        raise ValueError("nonempty interpolation requires at least one source point")
    if points > _MAX_INDEX:
        raise ValueError("three_interpolate supports at most 2**31-1 source points")
    if batch * channels * queries > (1 << 32) - 1:
        raise ValueError("three_interpolate output exceeds the native index range")
    return batch, channels, points, queries


class _PendingIndexCheck:
    """Device-side version of the reference's bounds check
    (mps_pointops/pointnet2.py:130-131): the flag is copied to pinned memory
    behind the check kernel, and read (waiting for that copy only) once the
    interpolation has been queued; its kernels skip out-of-range indices."""

    def __init__(self, indices: Tensor, points: int):
        self.points = points
        self.host = None
        if not indices.numel():
            return
        flag = torch.empty(1, dtype=torch.int32, device=indices.device)
        idx = indices.contiguous()
        with N.on_device(indices.device):
            N.check(N.lib().mpo_index_check(N.ptr(idx), 1 if idx.dtype == torch.int64 else 0,
                                            idx.numel(), points, N.ptr(flag),
                                            N.stream(indices.device)), "index check")
            self.host = torch.empty(1, dtype=torch.int32, pin_memory=True)
            self.host.copy_(flag, non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(torch.cuda.current_stream(indices.device))

    def raise_if_bad(self) -> None:
        if self.host is None:
            return
        self.event.synchronize()
        if int(self.host[0]):
            raise IndexError(f"indices must lie in [0, {self.points})")


class _ThreeInterpolate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, features: Tensor, indices: Tensor, weights: Tensor) -> Tensor:
        batch, channels, points = features.shape
        queries = indices.shape[1]
        output = torch.empty((batch, channels, queries), dtype=torch.float32,
                             device=features.device)
        if output.numel():
            f = features.contiguous()
            with N.on_device(features.device):
                N.check(N.lib().mpo_three_interpolate(
                    N.ptr(f), N.ptr(indices), N.ptr(weights), batch, channels, points, queries,
                    N.ptr(output), N.stream(features.device)), "three_interpolate")
        ctx.save_for_backward(indices, weights)
        ctx.points = points
        ctx.channels = channels
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        if grad_output is None:
            return None, None, None
        indices, weights = ctx.saved_tensors
        batch, queries, _ = indices.shape
        grad_features = None
        if ctx.needs_input_grad[0]:
            grad_features = torch.empty((batch, ctx.channels, ctx.points), dtype=torch.float32,
                                        device=indices.device)
            g = grad_output.contiguous()
            with N.on_device(indices.device):
                N.check(N.lib().mpo_three_interpolate_backward(
                    N.ptr(g), N.ptr(indices), N.ptr(weights), batch, ctx.channels, ctx.points,
                    queries, N.ptr(grad_features), N.stream(indices.device)),
                    "three_interpolate backward")
        # The original PointNet++ wrapper returns an explicit zero weight
        # gradient (mps_pointops/pointnet2.py:187).
        grad_weights = torch.zeros_like(weights) if ctx.needs_input_grad[2] else None
        return grad_features, None, grad_weights


def three_interpolate(features: Tensor, indices: Tensor, weights: Tensor) -> Tensor:
    """Interpolate (B,C,M) features at (B,N,3) source indices (pointnet2.py:191-211).

    out[b,c,n] = ((F[b,c,I0]*W0 + F[b,c,I1]*W1) + F[b,c,I2]*W2).  Backward
    accumulates grad_out*W at the selected sources (repeats summed, float
    atomics, so low bits may vary run to run); the weight gradient is an
    explicit zero tensor.  The index bounds check runs on the device and is
    read once the interpolation is queued (IndexError as in the reference).
    """
    _, _, points, _ = _validate_interpolate(features, indices, weights)
    if features.device.type != "cuda" and indices.numel():
        # Same order as the reference: the bounds error before the device error.
        if torch.any((indices < 0) | (indices >= points)).item():
            raise IndexError(f"indices must lie in [0, {points})")
    N.require_cuda(features, "three_interpolate")
    pending = _PendingIndexCheck(indices, points)
    index32 = indices.contiguous() if indices.dtype == torch.int32 else indices.to(torch.int32)
    out = _ThreeInterpolate.apply(features, index32, weights.contiguous())
    pending.raise_if_bad()
    return out


__all__ = ["three_nn", "three_interpolate"]
