"""PointNet++ set-abstraction grouping on the B200 kernels.

``gather_operation`` and ``grouping_operation`` are drop-ins for the
pointnet2_ops functions that the reference serves with torch ``gather``
(gamzerA/mps-pointops mps_pointops/compat.py:62-73): same shapes, values and
gradients, computed for float32 CUDA tensors by ``mpo_group_points`` (one
launch, no int32 -> int64 index cast, no expanded index tensor) and its
scatter-add backward.  Other dtypes and devices keep the reference's torch
``gather``, which is its own implementation of these two functions.

``sample_and_gather`` fuses the sampling step (pointnet2_ops FPS and the
gather of the sampled coordinates) into the FPS launch.
``query_and_group`` fuses the set-abstraction grouping that the reference
composes from four calls (tests/test_pointnet2_e2e.py:40-44: ball query,
grouping of the coordinates minus the centre, grouping of the features,
concatenation) into one ``mpo_query_and_group`` call that writes the
(B, 3 + C, npoint, nsample) result once.  ``QueryAndGroup`` and ``GroupAll``
are the pointnet2_ops modules built on it.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from . import _native as N
from ._ball_query_cuda import _checked_radius_and_k


class _PendingBoundsCheck:
    """torch ``gather`` rejects an index outside [0, N).  Here the bounds check
    runs on the device next to the gather (``mpo_index_check``) and its flag is
    copied to pinned memory; the kernel reads 0 for such an index, so the
    launch stays memory-safe.  The host does not wait for the flag: like a
    device-side check of a CUDA gather, a bad index is reported as soon as the
    flag has arrived -- at the end of this or a later grouping call, or at
    :func:`check_indices`.  Indices made by this package's FPS and pointnet2
    ball query are in range by construction and are not checked."""

    def __init__(self, idx: Tensor, size: int):
        self.size = size
        self.slot = None
        if not idx.numel():
            return
        pool = _flag_pool(idx.device)
        self.slot = pool.take()
        self.pool = pool
        flag = pool.device[self.slot:self.slot + 1]
        N.check(N.lib().mpo_index_check(N.ptr(idx), 1 if idx.dtype == torch.int64 else 0,
                                        idx.numel(), size, N.ptr(flag), N.stream(idx.device)),
                "index check")
        pool.host[self.slot:self.slot + 1].copy_(flag, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(idx.device))

    def done(self) -> bool:
        return self.slot is None or self.event.query()

    def bad(self) -> bool:
        """Wait for the flag, release its slot, and return whether it is set."""
        if self.slot is None:
            return False
        self.event.synchronize()
        result = bool(int(self.pool.host[self.slot]))
        self.pool.give(self.slot)
        self.slot = None
        return result


class _FlagPool:
    """Device flags and their pinned host copies for the pending checks of one
    device, allocated once (a pinned allocation per call would cost more than
    the gather)."""

    SLOTS = 256

    def __init__(self, device: torch.device):
        self.device = torch.empty(self.SLOTS, dtype=torch.int32, device=device)
        self.host = torch.empty(self.SLOTS, dtype=torch.int32, pin_memory=True)
        self.free = list(range(self.SLOTS))

    def take(self) -> int:
        if not self.free:
            check_indices(block=True)  # every slot is pending: resolve them
        return self.free.pop()

    def give(self, slot: int) -> None:
        self.free.append(slot)


_pools: dict = {}


def _flag_pool(device: torch.device) -> _FlagPool:
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _pools:
        _pools[key] = _FlagPool(torch.device("cuda", key))
    return _pools[key]


_pending: list[_PendingBoundsCheck] = []


def check_indices(block: bool = True) -> None:
    """Report an out-of-range index given to an earlier gather_operation or
    grouping_operation call: raises ``RuntimeError`` for the first such call
    whose check has finished (all of them with ``block=True``)."""
    global _pending
    keep = []
    for i, chk in enumerate(_pending):
        if not block and not chk.done():
            keep.append(chk)
            continue
        if chk.bad():
            # The remaining checks stay pending; each releases its slot when read.
            _pending = keep + _pending[i + 1:]
            raise RuntimeError(f"index out of bounds for dimension 2 with size {chk.size}")
    _pending = keep


def _native_index(idx: Tensor) -> Tensor:
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.long()
    return idx.contiguous()


def _known_in_range(idx: Tensor, size: int) -> bool:
    # Indices made by this package's FPS and pointnet2 ball query for a cloud
    # of at least `size` points are in range by construction.
    bound = getattr(idx, "_mpo_index_bound", None)
    return bound is not None and bound <= size


class _GroupPoints(torch.autograd.Function):
    """out[b, c, p, s] = features[b, c, idx[b, p, s]] with its scatter-add backward."""

    @staticmethod
    def forward(ctx, features: Tensor, idx: Tensor, checked: bool) -> Tensor:
        B, C, Np = features.shape
        _, P, S = idx.shape
        feats = features.contiguous()
        out = torch.empty((B, C, P, S), dtype=features.dtype, device=features.device)
        with N.on_device(features.device):
            if not checked:
                _pending.append(_PendingBoundsCheck(idx, Np))
            lib = N.lib()
            ws_bytes = int(lib.mpo_group_points_workspace_bytes(B, C, Np, P, S))
            ws = N.workspace(ws_bytes, features.device)
            N.check(lib.mpo_group_points(N.ptr(feats), N.ptr(idx), int(idx.dtype == torch.int64),
                                         B, C, Np, P, S, N.ptr(out), N.ptr(ws), ws_bytes,
                                         N.stream(features.device)), "grouping_operation")
        check_indices(block=False)
        ctx.save_for_backward(idx)
        ctx.points = Np
        return out

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        (idx,) = ctx.saved_tensors
        B, C, P, S = grad_out.shape
        g = grad_out.contiguous()
        grad = torch.empty((B, C, ctx.points), dtype=g.dtype, device=g.device)
        with N.on_device(g.device):
            lib = N.lib()
            ws_bytes = int(lib.mpo_group_points_workspace_bytes(B, C, ctx.points, P, S))
            ws = N.workspace(ws_bytes, g.device)
            N.check(lib.mpo_group_points_backward(N.ptr(g), N.ptr(idx),
                                                  int(idx.dtype == torch.int64), B, C,
                                                  ctx.points, P, S, N.ptr(grad), N.ptr(ws),
                                                  ws_bytes, N.stream(g.device)),
                    "grouping_operation backward")
        return grad, None, None


def _native_ok(features: Tensor, idx: Tensor) -> bool:
    return (features.device.type == "cuda" and features.dtype == torch.float32
            and idx.device == features.device and not idx.is_floating_point()
            and features.shape[0] <= 65535)


def gather_operation(features: Tensor, idx: Tensor) -> Tensor:
    """Like ``pointnet2_utils.gather_operation`` (mps_pointops/compat.py:62-65):
    (B, C, N), (B, npoint) -> (B, C, npoint), out[b, c, p] = features[b, c, idx[b, p]]."""
    B, C, _ = features.shape
    if not _native_ok(features, idx):
        return features.gather(2, idx.long().unsqueeze(1).expand(B, C, -1))
    N.require_cuda(features, "gather_operation")
    checked = _known_in_range(idx, features.shape[2])
    return _GroupPoints.apply(features, _native_index(idx).unsqueeze(-1), checked).squeeze(-1)


def grouping_operation(features: Tensor, idx: Tensor) -> Tensor:
    """Like ``pointnet2_utils.grouping_operation`` (mps_pointops/compat.py:68-73):
    (B, C, N), (B, npoint, nsample) -> (B, C, npoint, nsample)."""
    B, C, _ = features.shape
    _, npoint, nsample = idx.shape
    if not _native_ok(features, idx):
        flat = idx.long().reshape(B, 1, npoint * nsample).expand(B, C, -1)
        return features.gather(2, flat).reshape(B, C, npoint, nsample)
    N.require_cuda(features, "grouping_operation")
    checked = _known_in_range(idx, features.shape[2])
    return _GroupPoints.apply(features, _native_index(idx), checked)


class _SampleAndGather(torch.autograd.Function):
    """pointnet2_ops FPS (start 0, near-origin points skipped, int32) and the
    gather of the sampled points, in one launch; the gradient of the gathered
    points scatters back to xyz."""

    @staticmethod
    def forward(ctx, xyz: Tensor, npoint: int):
        B, Np, _ = xyz.shape
        pts = xyz.contiguous()
        idx = torch.empty((B, npoint), dtype=torch.int32, device=xyz.device)
        new_xyz = torch.empty((B, npoint, 3), dtype=xyz.dtype, device=xyz.device)
        if idx.numel():
            lib = N.lib()
            with N.on_device(xyz.device):
                ws = N.workspace(lib.mpo_fps_workspace_bytes(B, Np, npoint, 0), xyz.device)
                N.check(lib.mpo_fps_gather(N.ptr(pts), B, Np, npoint, 0, 1, 1, 0, N.ptr(idx),
                                           N.ptr(new_xyz), None, N.ptr(ws),
                                           0 if ws is None else ws.numel(),
                                           N.stream(xyz.device)), "furthest_point_sample")
        ctx.save_for_backward(idx)
        ctx.points = Np
        ctx.mark_non_differentiable(idx)
        return idx, new_xyz

    @staticmethod
    def backward(ctx, _grad_idx, grad_new: Tensor):
        (idx,) = ctx.saved_tensors
        B, P = idx.shape
        g = grad_new.contiguous()
        grad = torch.empty((B, ctx.points, 3), dtype=g.dtype, device=g.device)
        with N.on_device(g.device):
            N.check(N.lib().mpo_gather_points_backward(N.ptr(g), N.ptr(idx), B, ctx.points, P,
                                                       N.ptr(grad), N.stream(g.device)),
                    "sample_and_gather backward")
        return grad, None


def sample_and_gather(xyz: Tensor, npoint: int) -> tuple[Tensor, Tensor]:
    """Fused set-abstraction sampling: ``(idx, new_xyz)`` with
    ``idx = compat.furthest_point_sample(xyz, npoint)`` (int32) and
    ``new_xyz = gather_operation(xyz^T, idx)^T`` (B, npoint, 3) -- the
    sampling step of tests/test_pointnet2_e2e.py:37-39 in one launch; the FPS
    kernel writes each sample's coordinates as it picks it.  Gradients of
    new_xyz flow back to xyz."""
    if xyz.dim() != 3 or xyz.shape[-1] != 3:
        raise ValueError(f"xyz must have shape (B, N, 3), got {tuple(xyz.shape)}")
    if npoint < 0:
        raise ValueError(f"npoint must be >= 0, got {npoint}")
    if npoint > 0 and xyz.shape[1] == 0:
        raise ValueError("cannot sample from an empty point cloud")
    N.require_cuda(xyz, "sample_and_gather")
    if xyz.dtype != torch.float32:
        raise TypeError(f"xyz must be float32 on CUDA, got {xyz.dtype}")
    return _SampleAndGather.apply(xyz, npoint)


class _QueryAndGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xyz: Tensor, new_xyz: Tensor, features: Tensor | None, radius_sq: float,
                nsample: int, use_xyz: bool):
        B, Np, _ = xyz.shape
        P = new_xyz.shape[1]
        C = 0 if features is None else features.shape[1]
        a, q = xyz.contiguous(), new_xyz.contiguous()
        f = None if features is None else features.contiguous()
        idx = torch.empty((B, P, nsample), dtype=torch.int32, device=xyz.device)
        out = torch.empty((B, (3 if use_xyz else 0) + C, P, nsample), dtype=xyz.dtype,
                          device=xyz.device)
        with N.on_device(xyz.device):
            lib = N.lib()
            ws_bytes = int(lib.mpo_query_and_group_workspace_bytes(B, Np, P, nsample, C))
            ws = N.workspace(ws_bytes, xyz.device)
            N.check(lib.mpo_query_and_group(N.ptr(a), N.ptr(q), N.ptr(f), B, Np, P, nsample, C,
                                            radius_sq, int(use_xyz), N.ptr(idx), N.ptr(out),
                                            N.ptr(ws), ws_bytes, N.stream(xyz.device)),
                    "query_and_group")
        ctx.save_for_backward(idx)
        ctx.sizes = (B, Np, P, nsample, C, use_xyz, features is not None)
        ctx.mark_non_differentiable(idx)
        return out, idx

    @staticmethod
    def backward(ctx, grad_out: Tensor, _grad_idx):
        (idx,) = ctx.saved_tensors
        B, Np, P, S, C, use_xyz, has_features = ctx.sizes
        g = grad_out.contiguous()
        dev = g.device
        want_xyz, want_new, want_feat = ctx.needs_input_grad[:3]
        gx = torch.empty((B, Np, 3), dtype=g.dtype, device=dev) if want_xyz else None
        gq = torch.empty((B, P, 3), dtype=g.dtype, device=dev) if want_new else None
        gf = (torch.empty((B, C, Np), dtype=g.dtype, device=dev)
              if (want_feat and has_features) else None)
        with N.on_device(dev):
            lib = N.lib()
            ws_bytes = int(lib.mpo_query_and_group_workspace_bytes(B, Np, P, S, C)) if gf is not None else 0
            ws = N.workspace(ws_bytes, dev)
            N.check(lib.mpo_query_and_group_backward(N.ptr(g), N.ptr(idx), B, Np, P, S, C,
                                                     int(use_xyz), N.ptr(gx), N.ptr(gq),
                                                     N.ptr(gf), N.ptr(ws), ws_bytes, N.stream(dev)),
                    "query_and_group backward")
        return gx, gq, gf, None, None, None


def query_and_group(xyz: Tensor, new_xyz: Tensor, features: Tensor | None, radius: float,
                    nsample: int, use_xyz: bool = True) -> tuple[Tensor, Tensor]:
    """Fused PointNet++ grouping: ``(new_features, idx)``.

    Equals ``idx = compat.ball_query(radius, nsample, xyz, new_xyz)``, then
    ``grouping_operation(xyz^T, idx) - new_xyz^T[..., None]`` concatenated
    along channels with ``grouping_operation(features, idx)`` (the
    composition of tests/test_pointnet2_e2e.py:40-44), for float32 CUDA
    tensors, with gradients for xyz, new_xyz and features.

    Args:
        xyz: (B, N, 3) points.  new_xyz: (B, npoint, 3) centres.
        features: (B, C, N) or None.  radius, nsample: the ball query.
        use_xyz: put the centred coordinates in front of the features.
    Returns:
        (B, 3 * use_xyz + C, npoint, nsample) float32 and the (B, npoint,
        nsample) int32 neighbour indices.
    """
    _, radius_sq = _checked_radius_and_k(radius, nsample)
    if xyz.dim() != 3 or new_xyz.dim() != 3 or xyz.shape[-1] != 3 or new_xyz.shape[-1] != 3:
        raise ValueError("xyz and new_xyz must have shapes (B, N, 3) and (B, npoint, 3)")
    if xyz.shape[0] != new_xyz.shape[0] or xyz.device != new_xyz.device:
        raise ValueError("xyz and new_xyz must have the same batch size and device")
    if features is None and not use_xyz:
        raise ValueError("Cannot have not features and not use xyz as a feature!")
    if features is not None:
        if (features.dim() != 3 or features.shape[0] != xyz.shape[0]
                or features.shape[2] != xyz.shape[1] or features.device != xyz.device):
            raise ValueError("features must have shape (B, C, N) on the device of xyz")
    N.require_cuda(xyz, "query_and_group")
    for t in (xyz, new_xyz) + (() if features is None else (features,)):
        if t.dtype != torch.float32:
            raise TypeError(f"query_and_group takes float32 tensors, got {t.dtype}")
    if xyz.shape[0] > 65535:
        raise ValueError("batch must be at most 65535")
    return _QueryAndGroup.apply(xyz, new_xyz, features, radius_sq, nsample, bool(use_xyz))


class QueryAndGroup(nn.Module):
    """``pointnet2_ops.pointnet2_utils.QueryAndGroup``: groups the points of a
    ball around each centre; forward(xyz, new_xyz, features=None) ->
    (B, 3 + C, npoint, nsample) (coordinates relative to the centre first
    when ``use_xyz``), on the fused kernel."""

    def __init__(self, radius: float, nsample: int, use_xyz: bool = True):
        super().__init__()
        self.radius, self.nsample, self.use_xyz = radius, nsample, use_xyz

    def forward(self, xyz: Tensor, new_xyz: Tensor, features: Tensor | None = None) -> Tensor:
        if features is None and not self.use_xyz:
            raise ValueError("Cannot have not features and not use xyz as a feature!")
        out, _ = query_and_group(xyz, new_xyz, features, self.radius, self.nsample,
                                 self.use_xyz)
        return out


class GroupAll(nn.Module):
    """``pointnet2_ops.pointnet2_utils.GroupAll``: one group holding every
    point; forward(xyz, new_xyz, features=None) -> (B, 3 + C, 1, N)."""

    def __init__(self, use_xyz: bool = True):
        super().__init__()
        self.use_xyz = use_xyz

    def forward(self, xyz: Tensor, new_xyz: Tensor, features: Tensor | None = None) -> Tensor:
        grouped_xyz = xyz.transpose(1, 2).unsqueeze(2)
        if features is None:
            return grouped_xyz
        grouped_features = features.unsqueeze(2)
        if self.use_xyz:
            return torch.cat([grouped_xyz, grouped_features], dim=1)
        return grouped_features


__all__ = ["GroupAll", "QueryAndGroup", "check_indices", "gather_operation",
           "grouping_operation", "query_and_group", "sample_and_gather"]
