"""Autograd wrappers of the native row gathers and the flat interpolation
(``mpo_gather_rows``, ``mpo_flat_interpolate`` and their backwards).

They serve the neighbour gather of the PyTorch3D ball-query adapter
(mps_pointops/pytorch3d.py:26-38), Pointcept's ``grouping``
(pointcept.py:168-203) and Pointcept's ``interpolation``
(pointcept.py:219-243): ``-1`` slots give zero rows, gradients are
scatter-added back to the gathered rows (and subtracted from the centres of
relative coordinates).
"""

from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import _native as N


def _gather(src: Tensor, idx: Tensor, out: Tensor, stride: int, offset: int,
            centers: Tensor | None = None, K: int = 1) -> None:
    B, n, W = src.shape
    R = idx.shape[1]
    N.check(N.lib().mpo_gather_rows(
        N.ptr(src), B, n, W, N.ptr(idx), int(idx.dtype == torch.int32), R, N.ptr(centers), K,
        N.ptr(out), stride, offset, N.stream(src.device)), "gather rows")


def _gather_backward(grad: Tensor, stride: int, offset: int, B: int, n: int, W: int,
                     idx: Tensor, K: int, grad_src: Tensor | None,
                     grad_centers: Tensor | None) -> None:
    R = idx.shape[1]
    N.check(N.lib().mpo_gather_rows_backward(
        N.ptr(grad), stride, offset, B, n, W, N.ptr(idx), int(idx.dtype == torch.int32), R, K,
        N.ptr(grad_src), N.ptr(grad_centers), N.stream(grad.device)), "gather rows backward")


class GatherRows(torch.autograd.Function):
    """points (B, P, W), indices (B, Q, K) -> (B, Q, K, W), zero rows for
    indices outside [0, P); gradient to ``points``."""

    @staticmethod
    def forward(ctx, points: Tensor, indices: Tensor) -> Tensor:
        B, P, W = points.shape
        _, Q, K = indices.shape
        src = points.contiguous()
        idx = indices.reshape(B, Q * K).contiguous()
        out = torch.empty((B, Q, K, W), dtype=points.dtype, device=points.device)
        with N.on_device(points.device):
            _gather(src, idx, out, W, 0)
        ctx.save_for_backward(idx)
        ctx.shape = (B, P, W)
        ctx.mark_non_differentiable(indices)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad: Tensor):
        (idx,) = ctx.saved_tensors
        B, P, W = ctx.shape
        grad_points = torch.zeros((B, P, W), dtype=grad.dtype, device=grad.device)
        with N.on_device(grad.device):
            _gather_backward(grad.contiguous(), W, 0, B, P, W, idx, 1, grad_points, None)
        return grad_points, None


class GroupRows(torch.autograd.Function):
    """Pointcept grouping: feat (N, C), xyz (N, 3), centres (M, 3), idx (M, K)
    -> (M, K, C), or (M, K, 3 + C) with the relative coordinates
    xyz[idx] - centre first; ``-1`` slots are zero rows."""

    @staticmethod
    def forward(ctx, feat: Tensor, xyz: Tensor, centres: Tensor, idx: Tensor,
                with_xyz: bool) -> Tensor:
        n, C = feat.shape
        M, K = idx.shape
        W = C + (3 if with_xyz else 0)
        flat_idx = idx.reshape(1, M * K).contiguous()
        out = torch.empty((M, K, W), dtype=feat.dtype, device=feat.device)
        with N.on_device(feat.device):
            if with_xyz:
                _gather(xyz.contiguous().unsqueeze(0), flat_idx, out, W, 0,
                        centers=centres.contiguous(), K=K)
            _gather(feat.contiguous().unsqueeze(0), flat_idx, out, W, W - C)
        ctx.save_for_backward(flat_idx)
        ctx.dims = (n, C, M, K, with_xyz)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad: Tensor):
        (flat_idx,) = ctx.saved_tensors
        n, C, M, K, with_xyz = ctx.dims
        W = C + (3 if with_xyz else 0)
        g = grad.contiguous()
        dev = grad.device
        grad_feat = grad_xyz = grad_centres = None
        with N.on_device(dev):
            if ctx.needs_input_grad[0]:
                grad_feat = torch.zeros((n, C), dtype=grad.dtype, device=dev)
                _gather_backward(g, W, W - C, 1, n, C, flat_idx, 1, grad_feat, None)
            if with_xyz and (ctx.needs_input_grad[1] or ctx.needs_input_grad[2]):
                grad_xyz = torch.zeros((n, 3), dtype=grad.dtype, device=dev)
                grad_centres = torch.zeros((M, 3), dtype=grad.dtype, device=dev)
                _gather_backward(g, W, 0, 1, n, 3, flat_idx, K, grad_xyz, grad_centres)
        return grad_feat, grad_xyz, grad_centres, None, None


class FlatInterpolate(torch.autograd.Function):
    """Pointcept inverse-distance interpolation: feat (N, C), idx (M, k) int32,
    dist (M, k) -> (M, C); gradient to ``feat`` only (the weights are fixed)."""

    @staticmethod
    def forward(ctx, feat: Tensor, idx: Tensor, dist: Tensor) -> Tensor:
        n, C = feat.shape
        M, k = idx.shape
        f = feat.contiguous()
        i = idx.to(torch.int32).contiguous()
        d = dist.contiguous()
        out = torch.empty((M, C), dtype=feat.dtype, device=feat.device)
        with N.on_device(feat.device):
            N.check(N.lib().mpo_flat_interpolate(N.ptr(f), n, C, N.ptr(i), N.ptr(d), M, k,
                                                 N.ptr(out), N.stream(feat.device)),
                    "interpolation")
        ctx.save_for_backward(i, d)
        ctx.dims = (n, C)
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad: Tensor):
        i, d = ctx.saved_tensors
        n, C = ctx.dims
        M, k = i.shape
        grad_feat = torch.empty((n, C), dtype=grad.dtype, device=grad.device)
        with N.on_device(grad.device):
            N.check(N.lib().mpo_flat_interpolate_backward(
                N.ptr(grad.contiguous()), N.ptr(i), N.ptr(d), M, k, n, C, N.ptr(grad_feat),
                N.stream(grad.device)), "interpolation backward")
        return grad_feat, None, None
