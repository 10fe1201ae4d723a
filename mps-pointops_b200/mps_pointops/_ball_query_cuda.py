"""First-K radius search (ball query) on B200.

Drop-in for the reference's ``mps_pointops._ball_query_mps`` core
(mps_pointops/_ball_query_mps.py:73-273): the same public function
``ball_query(queries, points, *, radius, k, query_lengths, point_lengths)``,
result type, validation and error messages, with "CUDA" in place of "MPS".

Membership follows the reference's CPU path (mps_pointops/reference.py:83-121):
``((dx*dx + dy*dy) + dz*dz) < fl32(fl32(r) * fl32(r))`` in float32, every
operation rounded on its own, so non-finite coordinates never match.  float16
inputs are widened to float32 (exactly) before the search; distances are
float32 either way.
"""

from __future__ import annotations

import math
import struct
from typing import NamedTuple

import torch

from . import _native as N

_MIN_SUPPORTED_RADIUS_F32 = 2.0**-112


class BallQueryResult(NamedTuple):
    """Squared distances and indices, both shaped ``(B, Q, K)``."""

    distances: torch.Tensor
    indices: torch.Tensor


def _checked_radius_and_k(radius: float, k: int) -> tuple[float, float]:
    """Validate ``radius`` and ``k`` (mps_pointops/_ball_query_mps.py:87-119).

    Returns ``(radius_f32, radius_squared)`` where radius_f32 is the radius
    rounded to float32 and radius_squared = fl32(radius_f32 * radius_f32).
    """
    if not isinstance(k, int) or isinstance(k, bool) or k < 0 or k > (1 << 63) - 1:
        raise ValueError("k must be a non-negative integer")
    if not isinstance(radius, (int, float)) or isinstance(radius, bool):
        raise ValueError("radius must be a finite non-negative number")
    try:
        radius = float(radius)
    except OverflowError as exc:
        raise ValueError("radius must be a finite non-negative number") from exc
    if not math.isfinite(radius) or radius < 0:
        raise ValueError("radius must be a finite non-negative number")
    try:
        radius_f32 = struct.unpack("f", struct.pack("f", radius))[0]
    except OverflowError as exc:
        raise ValueError("radius must fit in float32") from exc
    if not math.isfinite(radius_f32) or (radius > 0 and radius_f32 < _MIN_SUPPORTED_RADIUS_F32):
        raise ValueError("positive radius must round to a normal float32 value at least 2**-112")
    # Two binary32 values multiply exactly in binary64; packing rounds once.
    radius_squared = float(radius_f32) * float(radius_f32)
    try:
        radius_squared = struct.unpack("f", struct.pack("f", radius_squared))[0]
    except OverflowError:
        radius_squared = math.inf
    return radius_f32, radius_squared


def _lengths_or_none(lengths, *, batch: int, count: int, device: torch.device, name: str):
    """mps_pointops/_ball_query_mps.py:73-84; ``None`` means every row is valid."""
    if lengths is None:
        return None
    if not isinstance(lengths, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor or None")
    if lengths.shape != (batch,) or lengths.dtype != torch.int64 or lengths.device != device:
        raise ValueError(f"{name} must have shape ({batch},), int64 dtype and device {device}")
    if torch.any((lengths < 0) | (lengths > count)).item():
        raise ValueError(f"{name} values must lie in [0, {count}]")
    return lengths.contiguous()


# Large searches run their queries in Morton order of their coordinates.
# The kernel scans the reference points in input order and stops a query at
# its K-th hit; the 8 queries of a CTA share each reference tile, so the CTA
# runs as long as its slowest query.  Neighbouring queries have similar local
# densities and therefore similar scan lengths: at BASELINE config 5 (131,072
# clustered queries, 2^20 points) the kernel takes 20.7 ms in Morton order
# against 29.1 ms in input order (22.2 ms with the ordering and the
# scatter back).  Each query's result does not depend on the others, so the
# outputs are identical.  Ragged query counts keep the input order (a
# query's validity is its position).
_ORDER_MIN_QUERIES = 16384
_ORDER_MIN_POINTS = 65536


def _morton_order(q: torch.Tensor) -> torch.Tensor:
    """(B, M, 3) -> (B, M) int64: each cloud's queries sorted by a 30-bit
    Morton code of their coordinates (non-finite coordinates count as 0)."""
    x = torch.nan_to_num(q.detach(), nan=0.0, posinf=0.0, neginf=0.0)
    lo = x.amin(dim=1, keepdim=True)
    hi = x.amax(dim=1, keepdim=True)
    v = ((x - lo) * (1023.0 / (hi - lo).clamp_min(1e-30))).clamp_(0, 1023).to(torch.int64)

    def spread(t):  # 10 bits -> every third bit
        t = (t | (t << 16)) & 0x030000FF
        t = (t | (t << 8)) & 0x0300F00F
        t = (t | (t << 4)) & 0x030C30C3
        return (t | (t << 2)) & 0x09249249

    code = spread(v[..., 0]) | (spread(v[..., 1]) << 1) | (spread(v[..., 2]) << 2)
    return torch.argsort(code, dim=1)


class _BallQuery(torch.autograd.Function):
    @staticmethod
    def forward(ctx, queries, points, query_lengths, point_lengths, radius_sq, k):
        batch, query_count, _ = queries.shape
        point_count = points.shape[1]
        q32 = queries if queries.dtype == torch.float32 else queries.float()
        p32 = points if points.dtype == torch.float32 else points.float()
        order = None
        if (query_lengths is None and query_count >= _ORDER_MIN_QUERIES
                and point_count >= _ORDER_MIN_POINTS and k > 0):
            order = _morton_order(q32)
            q32 = torch.gather(q32, 1, order.unsqueeze(-1).expand(-1, -1, 3))
        indices = torch.empty((batch, query_count, k), device=queries.device, dtype=torch.int64)
        distances = torch.empty((batch, query_count, k), device=queries.device, dtype=torch.float32)
        if indices.numel():
            with N.on_device(queries.device):
                N.check(N.lib().mpo_ball_query(
                    N.ptr(q32), N.ptr(p32), N.ptr(query_lengths), N.ptr(point_lengths), batch,
                    query_count, point_count, k, radius_sq, N.ptr(distances), N.ptr(indices),
                    N.stream(queries.device)), "ball_query")
            if order is not None:  # back to the callers' query order
                slots = order.unsqueeze(-1).expand(-1, -1, k)
                distances = torch.empty_like(distances).scatter_(1, slots, distances)
                indices = torch.empty_like(indices).scatter_(1, slots, indices)
        ctx.save_for_backward(queries, points, indices)
        ctx.mark_non_differentiable(indices)
        return distances, indices

    @staticmethod
    def backward(ctx, grad_distances, grad_indices):
        if grad_distances is None:
            return None, None, None, None, None, None
        queries, points, indices = ctx.saved_tensors
        batch, query_count, k = indices.shape
        if not indices.numel() or points.shape[1] == 0:
            return torch.zeros_like(queries), torch.zeros_like(points), None, None, None, None
        if torch.is_grad_enabled():
            # Higher-order gradients: the same formula as a differentiable
            # tensor expression (mps_pointops/_ball_query_mps.py:168-203).
            return _differentiable_backward(ctx, queries, points, indices, grad_distances)
        q32 = queries.float().contiguous()
        p32 = points.float().contiguous()
        g = grad_distances.float().contiguous()
        gq = torch.empty_like(q32) if ctx.needs_input_grad[0] else None
        gp = torch.empty_like(p32) if ctx.needs_input_grad[1] else None
        with N.on_device(queries.device):
            N.check(N.lib().mpo_ball_query_backward(
                N.ptr(g), N.ptr(q32), N.ptr(p32), N.ptr(indices), batch, query_count,
                points.shape[1], k, N.ptr(gq), N.ptr(gp), N.stream(queries.device)),
                "ball_query backward")
        gq = None if gq is None else gq.to(queries.dtype)
        gp = None if gp is None else gp.to(points.dtype)
        return gq, gp, None, None, None, None


def _differentiable_backward(ctx, queries, points, indices, grad_distances):
    batch, query_count, k = indices.shape
    valid = indices >= 0
    safe = indices.clamp_min(0)
    gathered = points.float().gather(1, safe.reshape(batch, -1, 1).expand(-1, -1, 3))
    gathered = gathered.reshape(batch, query_count, k, 3)
    delta = queries.float().unsqueeze(2) - gathered
    delta = torch.where(valid.unsqueeze(-1), delta, torch.zeros_like(delta))
    coeff = (2.0 * torch.where(valid, grad_distances, torch.zeros_like(grad_distances))).unsqueeze(-1)
    contrib = coeff * delta
    gq = contrib.sum(dim=2).to(queries.dtype) if ctx.needs_input_grad[0] else None
    gp = None
    if ctx.needs_input_grad[1]:
        gp = torch.zeros_like(points, dtype=torch.float32).scatter_add(
            1, safe.reshape(batch, -1, 1).expand(-1, -1, 3), -contrib.reshape(batch, -1, 3))
        gp = gp.to(points.dtype)
    return gq, gp, None, None, None, None


def ball_query(
    queries: torch.Tensor,
    points: torch.Tensor,
    *,
    radius: float,
    k: int,
    query_lengths: torch.Tensor | None = None,
    point_lengths: torch.Tensor | None = None,
) -> BallQueryResult:
    """Find the first ``k`` points strictly inside each radius
    (mps_pointops/_ball_query_mps.py:206-273).

    ``queries`` (B,Q,3) and ``points`` (B,P,3) are float32 or float16 CUDA
    tensors.  The output is ordered by point index, not distance; missing
    neighbours have index -1 and squared distance 0.  Gradients of valid
    squared distances reach both coordinate tensors; indices are not
    differentiable.  Supplying lengths checks their bounds with one
    device-to-host synchronisation.  The radius is rounded to float32 and must
    then be zero or at least 2**-112.
    """
    if not isinstance(queries, torch.Tensor) or not isinstance(points, torch.Tensor):
        raise TypeError("queries and points must be torch.Tensor values")
    if queries.ndim != 3 or points.ndim != 3 or queries.shape[-1] != 3 or points.shape[-1] != 3:
        raise ValueError("queries and points must have shapes (B, Q, 3) and (B, P, 3)")
    if queries.shape[0] != points.shape[0]:
        raise ValueError("queries and points must have the same batch size")
    if queries.device.type != "cuda" or points.device != queries.device:
        raise ValueError("queries and points must be on the same CUDA device")
    if queries.dtype not in (torch.float32, torch.float16) or points.dtype != queries.dtype:
        raise TypeError("queries and points must have the same float32 or float16 dtype")
    _, radius_squared = _checked_radius_and_k(radius, k)
    N.require_cuda(queries, "ball_query")
    batch, query_count, _ = queries.shape
    point_count = points.shape[1]
    if batch > 65535:
        raise ValueError("batch size must be at most 65535 for the CUDA kernel")
    query_lengths = _lengths_or_none(query_lengths, batch=batch, count=query_count,
                                     device=queries.device, name="query_lengths")
    point_lengths = _lengths_or_none(point_lengths, batch=batch, count=point_count,
                                     device=queries.device, name="point_lengths")
    distances, indices = _BallQuery.apply(queries.contiguous(), points.contiguous(),
                                          query_lengths, point_lengths, radius_squared, k)
    return BallQueryResult(distances=distances, indices=indices)
