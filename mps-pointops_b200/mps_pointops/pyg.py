"""The point-search operators of pyg-lib (used by PyG 2.8) on the B200 kernels.

Counterpart of ``mps_pointops.pyg`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/pyg.py:1-181), which adds MPS kernels to pyg-lib's operator
schemas.  pyg-lib ships its own CUDA kernels, so :func:`register_cuda` keeps
them unless ``override=True``; the call surfaces ``_fps_cuda``, ``_knn_cuda``
and ``_radius_cuda`` follow pyg-lib's argument order and defaults and can be
called directly.  pyg-lib's ``grid_cluster`` is not part of this build.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _native as N
from . import flat

_UINT_MAX = (1 << 32) - 1
_CUDA_LIBRARY: torch.library.Library | None = None


def _ptrs(x: Tensor, y: Tensor, ptr_x: Tensor | None, ptr_y: Tensor | None,
          *, feature_space: bool = False) -> tuple[Tensor, Tensor]:
    """pyg.py:57-69: an unbatched x is the full reference set, even when y has
    a batch pointer (pyg-lib then ignores ptr_y)."""
    flat._search_inputs(x, y, feature_space=feature_space)
    if ptr_x is None:
        ptr_x = torch.tensor([0, len(x)], dtype=torch.long, device=x.device)
        ptr_y = torch.tensor([0, len(y)], dtype=torch.long, device=y.device)
    elif ptr_y is None:
        raise ValueError("ptr_y is required when ptr_x is given")
    return ptr_x, ptr_y


def _check_inputs(x: Tensor, y: Tensor, ptr_x: Tensor, ptr_y: Tensor, *,
                  feature_space: bool = False) -> tuple[int, int]:
    """The offset checks of mps_pointops/_flat_search_mps.py:41-63, with CUDA in
    place of MPS.  The search kernels check the offsets again on the device."""
    if (x.ndim != 2 or y.ndim != 2 or x.shape[1] < 1
            or x.shape[1] != y.shape[1] or (not feature_space and x.shape[1] != 3)):
        if feature_space:
            raise ValueError("x and y must have shapes (N, D) and (M, D) with D >= 1")
        raise ValueError("x and y must have shapes (N, 3) and (M, 3)")
    if x.device.type != "cuda" or y.device != x.device:
        raise ValueError("x and y must be on the same CUDA device")
    if ptr_x.ndim != 1 or ptr_y.ndim != 1 or ptr_x.shape != ptr_y.shape or not ptr_x.numel():
        raise ValueError("ptr_x and ptr_y must have the same nonempty 1-D shape")
    for name, ptr, count in (("ptr_x", ptr_x, x.shape[0]), ("ptr_y", ptr_y, y.shape[0])):
        if ptr.dtype != torch.int64 or ptr.device != x.device:
            raise ValueError(f"{name} must be an int64 tensor on {x.device}")
        lengths = ptr[1:] - ptr[:-1]
        first, last, bad = torch.stack((
            ptr[0], ptr[-1], torch.any((lengths < 0) | (lengths > _UINT_MAX)).long())).tolist()
        if int(first) != 0 or int(last) != count:
            raise ValueError(f"{name} must start at 0 and end at {count}")
        if bad:
            raise ValueError(f"{name} must be nondecreasing with per-batch size <= 2**32-1")
    return int(ptr_x.numel() - 1), int(y.shape[0])


def _knn_cuda(x: Tensor, y: Tensor, ptr_x: Tensor | None = None, ptr_y: Tensor | None = None,
              k: int = 1, cosine: bool = False, num_workers: int = 1) -> Tensor:
    """pyg-lib's query-major ``[query, reference]`` kNN edges (pyg.py:72-97)."""
    ptr_x, ptr_y = _ptrs(x, y, ptr_x, ptr_y, feature_space=True)
    _check_inputs(x, y, ptr_x, ptr_y, feature_space=True)
    k = flat._nonnegative_int(k, "k")
    flat._nonnegative_int(num_workers, "num_workers")
    if cosine:
        raise NotImplementedError("cosine kNN is not supported for CUDA point clouds")
    if x.dtype != torch.float32:
        raise TypeError("x and y must be float32 for kNN on CUDA")
    if k == 0 or len(x) == 0 or len(y) == 0:
        return torch.empty((2, 0), dtype=torch.long, device=x.device)
    width = min(k, len(x))
    flat._check_cuda_knn_width(width)
    N.require_cuda(x, "pyg knn")
    return flat._edges(flat.knn_indices(x, y, ptr_x, ptr_y, width, check=False))


def _radius_cuda(x: Tensor, y: Tensor, ptr_x: Tensor | None = None,
                 ptr_y: Tensor | None = None, r: float = 1.0, max_num_neighbors: int = 32,
                 num_workers: int = 1, ignore_same_index: bool = False) -> Tensor:
    """The first neighbours in x order, optionally omitting the x row with
    the query's own global index (pyg.py:100-126)."""
    ptr_x, ptr_y = _ptrs(x, y, ptr_x, ptr_y)
    _check_inputs(x, y, ptr_x, ptr_y)
    limit = flat._nonnegative_int(max_num_neighbors, "max_num_neighbors")
    flat._nonnegative_int(num_workers, "num_workers")
    if x.dtype not in (torch.float16, torch.float32):
        raise TypeError("x and y must be float16 or float32 for radius on CUDA")
    if limit == 0 or len(x) == 0 or len(y) == 0:
        return torch.empty((2, 0), dtype=torch.long, device=x.device)
    width = min(limit, len(x))
    N.require_cuda(x, "pyg radius")
    return flat._edges(flat.radius_indices(x, y, ptr_x, ptr_y, r, width,
                                           ignore_same_index=ignore_same_index, check=False))


def _fps_cuda(src: Tensor, ptr: Tensor, ratio: float = 0.5, random_start: bool = True) -> Tensor:
    """pyg-lib's pointer-shaped FPS call surface (pyg.py:129-131)."""
    return flat.fps(src, ratio=ratio, random_start=random_start, ptr=ptr)


def register_cuda(*, override: bool = False) -> list[str]:
    """Register these kernels as CUDA implementations of ``pyg::fps``,
    ``pyg::knn`` and ``pyg::radius`` (the role of register_mps, pyg.py:144-181).

    Requires pyg-lib 0.6 or newer, whose operator schemas these functions
    implement.  An operator that already has a CUDA kernel (pyg-lib's own) is
    left unchanged unless ``override=True``.  Returns the operator names
    registered by this call; later calls register nothing.
    """
    global _CUDA_LIBRARY
    if _CUDA_LIBRARY is not None:
        return []
    try:
        import pyg_lib
    except ImportError as exc:
        raise ImportError(
            "PyG 2.8 integration requires pyg-lib>=0.6 with a wheel matching "
            "your PyTorch version"
        ) from exc

    implementations = {"fps": _fps_cuda, "knn": _knn_cuda, "radius": _radius_cuda}
    for name in implementations:
        if not hasattr(pyg_lib.ops, name) or not hasattr(torch.ops.pyg, name):
            raise RuntimeError(f"pyg-lib does not provide pyg::{name}; pyg-lib>=0.6 is required")

    library = torch.library.Library("pyg", "IMPL", "CUDA")
    registered = []
    for name, implementation in implementations.items():
        if override or not torch._C._dispatch_has_kernel_for_dispatch_key(f"pyg::{name}", "CUDA"):
            library.impl(name, implementation)
            registered.append(name)
    _CUDA_LIBRARY = library  # registrations live as long as the Library object
    return registered


__all__ = ["register_cuda"]
