"""Bidirectional Chamfer loss (squared L2 and L1) on B200.

Drop-in for ``mps_pointops.chamfer.chamfer_distance`` of gamzerA/mps-pointops
v1.0.0 (mps_pointops/chamfer.py:342-488): PyTorch3D argument conventions --
lengths, per-cloud weights, point/batch reductions, single-directional loss,
normals (D == 3) and PyTorch3D ``Pointclouds`` inputs -- with the same
validation and error messages.  The nearest-neighbour search and its backward
run in the sm_100a kernels of libmpo_b200.so; the reductions over the
per-point distances are tensor ops on the device.

Scope of this build: float32 and float64 CUDA tensors, ``norm=2`` and
``norm=1`` (L1, on ``mpo_chamfer_nearest_l1``); float64 runs the same search
and backward in double (``mpo_chamfer_nearest_f64``,
``mpo_chamfer_backward_f64``).
"""

from __future__ import annotations

from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import _native as N

PointReduction = Literal["mean", "sum", "max"] | None
BatchReduction = Literal["mean", "sum"] | None


def _unpack_cloud(points, lengths, normals, name):
    """PyTorch3D ``Pointclouds`` precedence (mps_pointops/chamfer.py:32-48)."""
    if isinstance(points, Tensor):
        return points, lengths, normals
    try:
        from pytorch3d.structures import Pointclouds
    except ImportError as exc:
        raise TypeError(
            f"{name} must be a tensor, or a PyTorch3D Pointclouds object "
            "(install PyTorch3D for Pointclouds inputs)"
        ) from exc
    if not isinstance(points, Pointclouds):
        raise TypeError(f"{name} must be a tensor or a PyTorch3D Pointclouds object")
    return points.points_padded(), points.num_points_per_cloud(), points.normals_padded()


def _validate_normals(points: Tensor, normals: Tensor | None, name: str) -> None:
    if normals is None:
        return
    if not isinstance(normals, Tensor) or normals.shape != points.shape:
        raise ValueError(f"{name} must have the same (B, P, 3) shape as its points")
    if normals.device != points.device or normals.dtype != points.dtype:
        raise ValueError(f"{name} must match its points' device and dtype")


class _PendingCheck:
    """Flags of mpo_chamfer_check_inputs copied to pinned host memory
    asynchronously; ``raise_if_bad`` waits for that copy only, so the device
    work queued after the check keeps running while the host reads them."""

    def __init__(self, flags_host: Tensor, event: torch.cuda.Event, P: int, Q: int):
        self.flags, self.event, self.P, self.Q = flags_host, event, P, Q

    def raise_if_bad(self) -> None:
        self.event.synchronize()
        bad_x, bad_y, bad_lx, bad_ly = self.flags.tolist()
        if bad_lx:
            raise ValueError(f"x_lengths must lie in [0, {self.P}]")
        if bad_ly:
            raise ValueError(f"y_lengths must lie in [0, {self.Q}]")
        if bad_x:
            raise ValueError("valid x coordinates must be finite")
        if bad_y:
            raise ValueError("valid y coordinates must be finite")


def _validate_clouds(x, y, x_lengths, y_lengths, defer: bool = False):
    """mps_pointops/chamfer.py:79-110: shapes, dtype, lengths in range and
    finite valid coordinates -- here one native check.  The check and the
    copy of its flags to pinned host memory run on a side stream that first
    waits for the caller's stream (the inputs as the caller sees them), so
    the search queued next starts at once, beside the check.  With ``defer``
    the result is returned as a _PendingCheck to be raised after the search
    has been queued (the kernels clamp lengths and are memory-safe on the
    inputs the check rejects, so queuing them first is safe); otherwise it is
    raised here."""
    if x.ndim != 3 or y.ndim != 3 or x.shape[-1] < 1 or y.shape[-1] != x.shape[-1]:
        raise ValueError("x and y must have shapes (B, P, D) and (B, Q, D) with D >= 1")
    if x.shape[0] != y.shape[0]:
        raise ValueError("x and y must have the same batch size")
    if x.device != y.device or x.dtype != y.dtype:
        raise ValueError("x and y must have the same device and dtype")
    if x.dtype not in (torch.float32, torch.float64):
        raise TypeError("Chamfer inputs must be float32 (or float64 outside MPS)")
    N.require_cuda(x, "chamfer_distance")
    B, P, D = x.shape
    Q = y.shape[1]
    for value, count, name in ((x_lengths, P, "x_lengths"), (y_lengths, Q, "y_lengths")):
        if value is not None and (value.shape != (B,) or value.dtype != torch.long
                                  or value.device != x.device):
            raise ValueError(f"{name} must be an int64 tensor of shape ({B},) on {x.device}")
    lx = None if x_lengths is None else x_lengths.contiguous()
    ly = None if y_lengths is None else y_lengths.contiguous()
    xc, yc = x.detach().contiguous(), y.detach().contiguous()
    with N.on_device(x.device):
        side = N.side_stream(x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            if x.dtype == torch.float32:
                flags = torch.empty(4, dtype=torch.int32, device=x.device)
                N.check(N.lib().mpo_chamfer_check_inputs(N.ptr(xc), N.ptr(yc), N.ptr(lx),
                                                         N.ptr(ly), B, P, Q, D, N.ptr(flags),
                                                         N.stream(x.device)),
                        "chamfer input check")
            else:
                # float64: the same four flags from device tensor ops (the
                # native check reads float32).
                flags = torch.stack([*_bad_side(xc, lx, P), *_bad_side(yc, ly, Q)])
                flags = flags[[0, 2, 1, 3]].int()
            host = torch.empty(4, dtype=torch.int32, pin_memory=True)
            host.copy_(flags, non_blocking=True)
            event = torch.cuda.Event()
            event.record(side)
        # The caller's tensors are read on the side stream: keep their memory
        # from being reused on the caller's stream before the check has run.
        for t in (xc, yc, lx, ly):
            if t is not None:
                t.record_stream(side)
    pending = _PendingCheck(host, event, P, Q)
    if not defer:
        pending.raise_if_bad()
        pending = None
    return lx, ly, pending


def _bad_side(points: Tensor, lengths: Tensor | None, count: int):
    """(non-finite valid coordinate, length outside [0, count]) as 0-d bool
    tensors on the device (mps_pointops/chamfer.py:79-110)."""
    if lengths is None:
        valid = torch.ones(points.shape[:2], dtype=torch.bool, device=points.device)
        bad_len = torch.zeros((), dtype=torch.bool, device=points.device)
    else:
        valid = (torch.arange(count, device=points.device)[None]
                 < lengths.clamp(0, count)[:, None])
        bad_len = ((lengths < 0) | (lengths > count)).any()
    bad_val = (valid & ~torch.isfinite(points).all(dim=-1)).any()
    return bad_val, bad_len


class _Nearest64(torch.autograd.Function):
    """float64 search (both norms) and backward on the double kernels
    (mps_pointops/chamfer.py:161-212, 227-251, 269-293)."""

    @staticmethod
    def forward(ctx, x, y, lx, ly, bidirectional: bool, norm: int):
        B, P, D = x.shape
        Q = y.shape[1]
        dev = x.device
        dist_x = torch.empty((B, P), dtype=torch.float64, device=dev)
        idx_x = torch.empty((B, P), dtype=torch.long, device=dev)
        dist_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.float64, device=dev)
        idx_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.long, device=dev)
        xc, yc = x.contiguous(), y.contiguous()
        with N.on_device(dev):
            N.check(N.lib().mpo_chamfer_nearest_f64(
                N.ptr(xc), N.ptr(yc), N.ptr(lx), N.ptr(ly), B, P, Q, D, norm, int(bidirectional),
                N.ptr(dist_x), N.ptr(idx_x), N.ptr(dist_y), N.ptr(idx_y), N.stream(dev)),
                "chamfer nearest (float64)")
        ctx.save_for_backward(xc, yc, idx_x, idx_y)
        ctx.bidirectional, ctx.norm = bidirectional, norm
        ctx.mark_non_differentiable(idx_x, idx_y)
        ctx.set_materialize_grads(False)
        return dist_x, dist_y, idx_x, idx_y

    @staticmethod
    @once_differentiable
    def backward(ctx, g_dx, g_dy, _gix, _giy):
        x, y, idx_x, idx_y = ctx.saved_tensors
        B, P, D = x.shape
        Q = y.shape[1]
        grad_x = torch.empty_like(x)
        grad_y = torch.empty_like(y)
        gx = None if g_dx is None else g_dx.double().contiguous()
        gy = None if (g_dy is None or not ctx.bidirectional) else g_dy.double().contiguous()
        with N.on_device(x.device):
            N.check(N.lib().mpo_chamfer_backward_f64(
                N.ptr(x), N.ptr(y), B, P, Q, D, ctx.norm, N.ptr(idx_x), N.ptr(gx), N.ptr(idx_y),
                N.ptr(gy), N.ptr(grad_x), N.ptr(grad_y), N.stream(x.device)),
                "chamfer backward (float64)")
        return grad_x, grad_y, None, None, None, None


class _NearestSquared(torch.autograd.Function):
    """Native nearest search (both directions from one call) and native
    scatter backward (mps_pointops/chamfer.py:215-251)."""

    @staticmethod
    def forward(ctx, x, y, lx, ly, bidirectional: bool):
        B, P, D = x.shape
        Q = y.shape[1]
        dev = x.device
        dist_x = torch.empty((B, P), dtype=torch.float32, device=dev)
        idx_x = torch.empty((B, P), dtype=torch.long, device=dev)
        dist_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.float32, device=dev)
        idx_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.long, device=dev)
        xc, yc = x.contiguous(), y.contiguous()
        lib = N.lib()
        with N.on_device(dev):
            ws = N.workspace(lib.mpo_chamfer_workspace_bytes(B, P, Q, D, int(bidirectional)), dev)
            N.check(N.timed("chamfer_nearest", dev, lib.mpo_chamfer_nearest,
                            N.ptr(xc), N.ptr(yc), N.ptr(lx), N.ptr(ly), B, P, Q, D,
                            int(bidirectional), N.ptr(dist_x), N.ptr(idx_x), N.ptr(dist_y),
                            N.ptr(idx_y), N.ptr(ws), 0 if ws is None else ws.numel(),
                            N.stream(dev)), "chamfer nearest")
        ctx.save_for_backward(xc, yc, idx_x, idx_y)
        ctx.bidirectional = bidirectional
        ctx.mark_non_differentiable(idx_x, idx_y)
        ctx.set_materialize_grads(False)
        return dist_x, dist_y, idx_x, idx_y

    @staticmethod
    @once_differentiable
    def backward(ctx, g_dx, g_dy, _gix, _giy):
        x, y, idx_x, idx_y = ctx.saved_tensors
        B, P, D = x.shape
        Q = y.shape[1]
        grad_x = torch.empty_like(x)
        grad_y = torch.empty_like(y)
        gx = None if g_dx is None else g_dx.float().contiguous()
        gy = None if (g_dy is None or not ctx.bidirectional) else g_dy.float().contiguous()
        with N.on_device(x.device):
            N.check(N.lib().mpo_chamfer_backward(
                N.ptr(x), N.ptr(y), B, P, Q, D, N.ptr(idx_x), N.ptr(gx), N.ptr(idx_y), N.ptr(gy),
                N.ptr(grad_x), N.ptr(grad_y), N.stream(x.device)), "chamfer backward")
        return grad_x, grad_y, None, None, None


class _NearestL1(torch.autograd.Function):
    """L1 nearest search in both directions and PyTorch3D's selected-pair
    subgradient (mps_pointops/chamfer.py:254-293)."""

    @staticmethod
    def forward(ctx, x, y, lx, ly, bidirectional: bool):
        B, P, D = x.shape
        Q = y.shape[1]
        dev = x.device
        dist_x = torch.empty((B, P), dtype=torch.float32, device=dev)
        idx_x = torch.empty((B, P), dtype=torch.long, device=dev)
        dist_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.float32, device=dev)
        idx_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.long, device=dev)
        xc, yc = x.contiguous(), y.contiguous()
        with N.on_device(dev):
            N.check(N.lib().mpo_chamfer_nearest_l1(
                N.ptr(xc), N.ptr(yc), N.ptr(lx), N.ptr(ly), B, P, Q, D, int(bidirectional),
                N.ptr(dist_x), N.ptr(idx_x), N.ptr(dist_y), N.ptr(idx_y), N.stream(dev)),
                "chamfer nearest (L1)")
        ctx.save_for_backward(xc, yc, idx_x, idx_y)
        ctx.bidirectional = bidirectional
        ctx.mark_non_differentiable(idx_x, idx_y)
        ctx.set_materialize_grads(False)
        return dist_x, dist_y, idx_x, idx_y

    @staticmethod
    @once_differentiable
    def backward(ctx, g_dx, g_dy, _gix, _giy):
        x, y, idx_x, idx_y = ctx.saved_tensors
        B, P, D = x.shape
        Q = y.shape[1]
        grad_x = torch.empty_like(x)
        grad_y = torch.empty_like(y)
        gx = None if g_dx is None else g_dx.float().contiguous()
        gy = None if (g_dy is None or not ctx.bidirectional) else g_dy.float().contiguous()
        with N.on_device(x.device):
            N.check(N.lib().mpo_chamfer_l1_backward(
                N.ptr(x), N.ptr(y), B, P, Q, D, N.ptr(idx_x), N.ptr(gx), N.ptr(idx_y), N.ptr(gy),
                N.ptr(grad_x), N.ptr(grad_y), N.stream(x.device)), "chamfer backward (L1)")
        return grad_x, grad_y, None, None, None


class _ChamferLoss(torch.autograd.Function):
    """Fused search + reduction for the common case (no weights, no normals,
    point_reduction mean/sum): one native call forward, one backward, instead
    of the search plus a chain of torch reductions (mps_pointops/chamfer.py:
    436-488).  The loss sums run in a fixed order (reproducible)."""

    @staticmethod
    def forward(ctx, x, y, lx, ly, bidirectional: bool, point_mode: int, batch_mode: int):
        B, P, D = x.shape
        Q = y.shape[1]
        dev = x.device
        dist_x = torch.empty((B, P), dtype=torch.float32, device=dev)
        idx_x = torch.empty((B, P), dtype=torch.long, device=dev)
        dist_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.float32, device=dev)
        idx_y = torch.empty((B, Q if bidirectional else 0), dtype=torch.long, device=dev)
        loss = torch.empty((B,) if batch_mode == 0 else (), dtype=torch.float32, device=dev)
        xc, yc = x.contiguous(), y.contiguous()
        lib = N.lib()
        with N.on_device(dev):
            ws = N.workspace(lib.mpo_chamfer_loss_workspace_bytes(B, P, Q, D, int(bidirectional)),
                             dev)
            N.check(N.timed("chamfer_nearest", dev, lib.mpo_chamfer_loss,
                            N.ptr(xc), N.ptr(yc), N.ptr(lx), N.ptr(ly), B, P, Q, D,
                            int(bidirectional), point_mode, batch_mode, N.ptr(dist_x),
                            N.ptr(idx_x), N.ptr(dist_y), N.ptr(idx_y), N.ptr(loss), N.ptr(ws),
                            0 if ws is None else ws.numel(), N.stream(dev)), "chamfer loss")
        ctx.save_for_backward(xc, yc, idx_x, idx_y)
        ctx.lengths = (lx, ly)
        ctx.modes = (bidirectional, point_mode, batch_mode)
        return loss

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        x, y, idx_x, idx_y = ctx.saved_tensors
        lx, ly = ctx.lengths
        bidirectional, point_mode, batch_mode = ctx.modes
        B, P, D = x.shape
        Q = y.shape[1]
        grad_x = torch.empty_like(x)
        grad_y = torch.empty_like(y)
        gl = g.float().contiguous()
        with N.on_device(x.device):
            N.check(N.lib().mpo_chamfer_loss_backward(
                N.ptr(x), N.ptr(y), N.ptr(lx), N.ptr(ly), B, P, Q, D, int(bidirectional),
                point_mode, batch_mode, N.ptr(idx_x), N.ptr(idx_y), N.ptr(gl), N.ptr(grad_x),
                N.ptr(grad_y), N.stream(x.device)), "chamfer loss backward")
        return grad_x, grad_y, None, None, None, None, None


def _full_lengths(points: Tensor, lengths: Tensor | None) -> Tensor:
    if lengths is not None:
        return lengths
    return torch.full((points.shape[0],), points.shape[1], dtype=torch.long, device=points.device)


def _normal_loss(query_normals, ref_normals, index, query_lengths, ref_lengths, abs_cosine):
    """1 - |cos| between a valid query's normal and its nearest reference's
    normal (mps_pointops/chamfer.py:60-76)."""
    valid = torch.arange(index.shape[1], device=index.device)[None] < query_lengths[:, None]
    safe = index.clamp_min(0)
    picked = ref_normals.gather(1, safe.unsqueeze(-1).expand(-1, -1, 3))
    picked = torch.where((ref_lengths > 0)[:, None, None], picked, torch.zeros_like(picked))
    q = torch.where(valid.unsqueeze(-1), query_normals, torch.zeros_like(query_normals))
    picked = torch.where(valid.unsqueeze(-1), picked, torch.zeros_like(picked))
    cosine = F.cosine_similarity(q, picked, dim=2, eps=1e-6)
    loss = 1 - (cosine.abs() if abs_cosine else cosine)
    return torch.where(valid, loss, torch.zeros_like(loss))


def _reduce_points(dist: Tensor, lengths: Tensor | None, mode: PointReduction) -> Tensor:
    """mps_pointops/chamfer.py:325-331."""
    if mode is None:
        return dist
    if mode == "max":
        return dist.max(dim=1).values if dist.shape[1] else dist.new_zeros((dist.shape[0],))
    total = dist.sum(dim=1)
    if mode == "sum":
        return total
    return total / (lengths.clamp(min=1) if lengths is not None else max(dist.shape[1], 1))


def _zero_weight_anchor(points: Tensor, lengths: Tensor | None, weights: Tensor) -> Tensor:
    """Graph-connected (B, B) zeros of PyTorch3D's all-zero-weight branch
    (mps_pointops/chamfer.py:334-339), padded rows excluded."""
    lengths = _full_lengths(points, lengths)
    valid = torch.arange(points.shape[1], device=points.device)[None] < lengths[:, None]
    kept = torch.where(valid.unsqueeze(-1), points, torch.zeros_like(points))
    return (weights[:, None] * kept.sum(dim=(1, 2))[None, :]) * 0


def chamfer_distance(
    x,
    y,
    x_lengths: Tensor | None = None,
    y_lengths: Tensor | None = None,
    x_normals: Tensor | None = None,
    y_normals: Tensor | None = None,
    weights: Tensor | None = None,
    batch_reduction: BatchReduction = "mean",
    point_reduction: PointReduction = "mean",
    norm: int = 2,
    single_directional: bool = False,
    abs_cosine: bool = True,
):
    """Chamfer loss (squared L2, or L1 with ``norm=1``) with PyTorch3D
    reduction conventions (mps_pointops/chamfer.py:342-488).

    ``x`` (B,P,D) and ``y`` (B,Q,D) float32 or float64 CUDA tensors, D >= 1.
    Each valid point is matched to the FIRST nearest valid point of the other
    cloud (squared distance in the input precision, no FMA, lowest index on
    ties); the loss is the
    reduced sum of the matched squared distances in both directions (one with
    ``single_directional``).  Returns ``(loss, normal_loss)``.  Input checks
    synchronise once with the host (twice with weights).
    """
    if norm not in (1, 2):
        raise ValueError("Support for 1 or 2 norm.")
    if batch_reduction not in (None, "mean", "sum"):
        raise ValueError("batch_reduction must be None, 'mean', or 'sum'")
    if point_reduction not in (None, "mean", "sum", "max"):
        raise ValueError("point_reduction must be None, 'mean', 'sum', or 'max'")
    if point_reduction is None and batch_reduction is not None:
        raise ValueError("batch_reduction must be None when point_reduction is None")
    if point_reduction == "max" and (x_normals is not None or y_normals is not None):
        raise ValueError('Normals must be None if point_reduction is "max"')
    x, x_lengths, x_normals = _unpack_cloud(x, x_lengths, x_normals, "x")
    y, y_lengths, y_normals = _unpack_cloud(y, y_lengths, y_normals, "y")
    # When nothing else can raise between the input check and the search
    # (no normals, no weights), the check's result is read after the search
    # is queued, so the device never idles on this host round trip.
    defer = x_normals is None and y_normals is None and weights is None and norm == 2
    lx, ly, pending = _validate_clouds(x, y, x_lengths, y_lengths, defer=defer)
    if x.shape[-1] != 3 and (x_normals is not None or y_normals is not None):
        raise NotImplementedError("normal loss currently requires D == 3")
    _validate_normals(x, x_normals, "x_normals")
    _validate_normals(y, y_normals, "y_normals")
    if point_reduction == "max" and (x_normals is not None or y_normals is not None):
        raise ValueError('Normals must be None if point_reduction is "max"')
    return_normals = x_normals is not None and y_normals is not None
    if weights is not None:
        if weights.shape != (x.shape[0],) or weights.device != x.device or weights.dtype != x.dtype:
            raise ValueError("weights must match the batch size, input device, and input dtype")
        if bool((~torch.isfinite(weights) | (weights < 0)).any().item()):
            raise ValueError("weights must be finite and nonnegative")
        if bool((weights == 0).all().item()):
            return _all_zero_weights(x, y, lx, ly, weights, point_reduction, batch_reduction,
                                     single_directional)
    if (norm == 2 and weights is None and not return_normals and point_reduction in ("mean", "sum")
            and x.dtype == torch.float32):
        loss = _ChamferLoss.apply(x, y, lx, ly, not single_directional,
                                  1 if point_reduction == "mean" else 0,
                                  {None: 0, "sum": 1, "mean": 2}[batch_reduction])
        if pending is not None:
            pending.raise_if_bad()
        return loss, None

    if x.dtype == torch.float64:
        dx, dy, ix, iy = _Nearest64.apply(x, y, lx, ly, not single_directional, norm)
    else:
        search = _NearestL1 if norm == 1 else _NearestSquared
        dx, dy, ix, iy = search.apply(x, y, lx, ly, not single_directional)
    if pending is not None:
        pending.raise_if_bad()
    nx = ny = None
    if return_normals:
        flx, fly = _full_lengths(x, lx), _full_lengths(y, ly)
        nx = _normal_loss(x_normals, y_normals, ix, flx, fly, abs_cosine)
    if weights is not None:
        dx = dx * weights[:, None]
        nx = nx * weights[:, None] if nx is not None else None
    rx = _reduce_points(dx, lx, point_reduction)
    rnx = _reduce_points(nx, lx, point_reduction) if nx is not None else None
    if single_directional:
        loss, normal_loss = rx, rnx
    else:
        if return_normals:
            ny = _normal_loss(y_normals, x_normals, iy, fly, flx, abs_cosine)
        if weights is not None:
            dy = dy * weights[:, None]
            ny = ny * weights[:, None] if ny is not None else None
        ry = _reduce_points(dy, ly, point_reduction)
        rny = _reduce_points(ny, ly, point_reduction) if ny is not None else None
        if point_reduction is None:
            loss = (rx, ry)
        elif point_reduction == "max":
            loss = torch.maximum(rx, ry)
        else:
            loss = rx + ry
        if rnx is not None and rny is not None:
            normal_loss = (rnx, rny) if point_reduction is None else rnx + rny
        else:
            normal_loss = None

    if batch_reduction is not None:
        loss = loss.sum()
        if normal_loss is not None:
            normal_loss = normal_loss.sum()
        if batch_reduction == "mean":
            if weights is None:
                denominator = max(x.shape[0], 1)
            else:
                total = weights.sum()
                denominator = torch.where(total > 0, total, torch.ones_like(total))
            loss = loss / denominator
            if normal_loss is not None:
                normal_loss = normal_loss / denominator
    return loss, normal_loss


def _all_zero_weights(x, y, lx, ly, weights, point_reduction, batch_reduction,
                      single_directional):
    """PyTorch3D's all-zero-weight result shapes (mps_pointops/chamfer.py:397-424)."""
    zero_x = _zero_weight_anchor(x, lx, weights)
    if single_directional:
        zero_loss, zero_normals = zero_x, zero_x
    else:
        zero_y = _zero_weight_anchor(y, ly, weights)
        if point_reduction == "max":
            zero_loss, zero_normals = torch.maximum(zero_x, zero_y), None
        elif point_reduction is None:
            zero_loss, zero_normals = (zero_x, zero_y), (zero_x, zero_y)
        else:
            zero_loss = zero_normals = zero_x + zero_y
    if batch_reduction is not None:
        zero_loss = zero_loss.sum()
        if zero_normals is not None:
            zero_normals = zero_normals.sum()
    return zero_loss, zero_normals
