"""Flat point-cloud operators with the ``torch_cluster`` index convention.

Drop-in for ``mps_pointops.flat`` of gamzerA/mps-pointops v1.0.0
(mps_pointops/flat.py:1-428): ``fps``, ``knn``, ``radius``, ``knn_graph`` and
``radius_graph`` with the same signatures, defaults, validation order,
exception types and messages.  ``x`` holds reference points, ``y`` query
points; batch vectors are sorted and indices in the results refer to the
original flat tensors.  Where the reference sends MPS tensors to its flat
Metal kernels (mps_pointops/_flat_fps_mps.py, _flat_search_mps.py), this
module sends CUDA tensors to the sm_100a kernels of libmpo_b200.so
(``mpo_flat_fps``, ``mpo_flat_knn``, ``mpo_flat_radius``).  Requests whose
result is empty are answered before any device work, as in the reference;
every other request on a non-CUDA tensor raises ``RuntimeError``.

Device rules (the reference's GPU rules, with CUDA in place of MPS):
  * FPS and kNN take float32 points; radius takes float16 or float32, and
    float16 points are widened to float32 before the search (the widening of
    flat_search.metal:164-167, exact).
  * FPS sample counts use the GPU rule of torch_cluster: the batch sizes are
    converted to the ratio's dtype before the product (flat.py:150-158).
  * kNN serves an effective k = min(k, len(x)) of at most 256.
Arithmetic follows the reference's CPU path (flat.py:256-288): squared
distances ((d0*d0 + d1*d1) + d2*d2) with each operation rounded on its own,
kNN in ascending (squared distance, index) order with every non-finite
distance dropped, radius ``d2 < fl32(r * r)`` with ``r * r`` in double.
"""

from __future__ import annotations

import math
import struct
from typing import Sequence

import torch
from torch import Tensor

from . import _native as N
from ._ball_query_cuda import _checked_radius_and_k

_CUDA_KNN_MAX_K = 256


def _points(value: Tensor, name: str) -> None:
    if not isinstance(value, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if value.ndim != 2 or value.shape[1] != 3:
        raise ValueError(f"{name} must have shape (N, 3), got {tuple(value.shape)}")
    if not value.is_floating_point():
        raise TypeError(f"{name} must have a floating-point dtype")


def _features(value: Tensor, name: str) -> None:
    if not isinstance(value, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if value.ndim != 2 or value.shape[1] < 1:
        raise ValueError(f"{name} must have shape (N, D) with D >= 1, got {tuple(value.shape)}")
    if not value.is_floating_point():
        raise TypeError(f"{name} must have a floating-point dtype")


def _batch_size(value: int | None) -> int | None:
    if value is None:
        return None
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise ValueError("batch_size must be a non-negative integer")
    return value


def _check_batch_host(batch: Tensor | None, count: int, device: torch.device, name: str) -> None:
    """The checks of flat.py:49-64 that need no device data."""
    if batch is None:
        return
    if not isinstance(batch, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor or None")
    if batch.ndim != 1 or batch.numel() != count:
        raise ValueError(f"{name} must have shape ({count},)")
    if batch.device != device:
        raise ValueError(f"{name} must be on {device}")
    if batch.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"{name} must have an integer dtype (int32 or int64)")


def _batch_facts(batch: Tensor) -> list[Tensor]:
    # (first id negative, ids decrease somewhere, last id) of a nonempty batch
    return [(batch[0] < 0).long(), (batch[1:] < batch[:-1]).any().long(), batch[-1].long()]


def _batch_sizes(batches: list[tuple[Tensor | None, int, torch.device, str]]) -> list[int]:
    """Validate sorted batch vectors (flat.py:49-64) in the reference's order and
    return their batch counts, reading the device facts of all of them in one
    device-to-host transfer (the reference reads them with separate .item()
    calls).  A host-side error of a later vector is raised only after the
    earlier vectors' device facts have been checked, as in the reference."""
    facts: list[Tensor] = []
    owners = []
    host_error = None
    for batch, count, device, name in batches:
        try:
            _check_batch_host(batch, count, device, name)
        except (TypeError, ValueError) as exc:
            host_error = exc
            break
        if batch is not None and count:
            facts.extend(_batch_facts(batch))
            owners.append(name)
    values = torch.stack(facts).tolist() if facts else []
    sizes = {}
    for i, name in enumerate(owners):
        first_negative, unsorted, last = values[3 * i:3 * i + 3]
        if first_negative or unsorted:
            raise ValueError(f"{name} must be sorted with non-negative batch IDs")
        sizes[name] = int(last) + 1
    if host_error is not None:
        raise host_error
    return [sizes.get(name, 0) for _, _, _, name in batches]


def _check_batch(batch: Tensor | None, count: int, device: torch.device, name: str) -> int:
    """Validate a sorted batch vector; return its batch count (flat.py:49-64)."""
    return _batch_sizes([(batch, count, device, name)])[0]


def _ptr_from_batch(batch: Tensor | None, count: int, device: torch.device, size: int) -> Tensor:
    """Segment offsets of a sorted batch vector (flat.py:67-76)."""
    if batch is None:
        # A missing batch vector means one point cloud, even if it is empty.
        return torch.tensor([0, count], dtype=torch.long, device=device)
    if size == 0:
        return torch.zeros(1, dtype=torch.long, device=device)
    boundaries = torch.arange(size + 1, dtype=torch.long, device=device)
    return torch.searchsorted(batch.contiguous().long(), boundaries).long()


def _pair_ptrs(x: Tensor, y: Tensor, batch_x: Tensor | None, batch_y: Tensor | None,
               batch_size: int | None) -> tuple[Tensor, Tensor]:
    """flat.py:79-97: both offset arrays over the same number of batch slots."""
    explicit_size = _batch_size(batch_size)
    size_x, size_y = _batch_sizes([(batch_x, len(x), x.device, "batch_x"),
                                   (batch_y, len(y), y.device, "batch_y")])
    size = max(1, size_x, size_y, explicit_size or 0)
    if size > 1 and (batch_x is None or batch_y is None):
        raise ValueError("batch_x and batch_y are both required for multiple batches")
    if explicit_size is not None and explicit_size < max(size_x, size_y):
        raise ValueError("batch_size is smaller than the largest batch ID")
    return (
        _ptr_from_batch(batch_x, len(x), x.device, size),
        _ptr_from_batch(batch_y, len(y), y.device, size),
    )


def _fps_ptr(x: Tensor, batch: Tensor | None, batch_size: int | None,
             ptr: Tensor | Sequence[int] | None) -> Tensor:
    """flat.py:100-122: ``ptr`` wins over ``batch``."""
    if ptr is not None:
        if isinstance(ptr, Tensor):
            if ptr.device != x.device or ptr.dtype not in (torch.int32, torch.int64):
                raise ValueError("ptr must be an integer tensor on the same device as x")
            result = ptr.long()
        elif isinstance(ptr, (list, tuple)):
            result = torch.tensor(ptr, dtype=torch.long, device=x.device)
        else:
            raise TypeError("ptr must be a tensor, a sequence of integers, or None")
        if result.ndim != 1 or len(result) == 0:
            raise ValueError("ptr must be a non-empty one-dimensional offset array")
        first, last, decreasing = torch.stack((
            result[0], result[-1], (result[1:] < result[:-1]).any().long())).tolist()
        if int(first) != 0 or int(last) != len(x):
            raise ValueError("ptr must start at 0 and end at len(x)")
        if decreasing:
            raise ValueError("ptr must be non-decreasing")
        return result.contiguous()
    explicit_size = _batch_size(batch_size)
    inferred_size = _check_batch(batch, len(x), x.device, "batch")
    if explicit_size is not None and explicit_size < inferred_size:
        raise ValueError("batch_size is smaller than the largest batch ID")
    size = (max(1, inferred_size, explicit_size or 0) if batch is None
            else max(inferred_size, explicit_size or 0))
    return _ptr_from_batch(batch, len(x), x.device, size)


def _ratio(value: float | Tensor | None, dtype: torch.dtype) -> Tensor:
    """The CPU scalar tensor torch_cluster would use as the ratio (flat.py:125-147).

    A Python ratio becomes a tensor of the points' dtype; a tensor ratio keeps
    its dtype and shape, which decide the precision of the sample counts.
    """
    if value is None:
        value = 0.5
    if isinstance(value, Tensor):
        if value.numel() != 1 or value.ndim > 1:
            raise ValueError("ratio tensor must be scalar or a length-one vector")
        result = value.detach().to("cpu")
    elif isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError("ratio must be a number or scalar tensor")
    else:
        result = torch.tensor(float(value), dtype=dtype)
    if not math.isfinite(float(result)) or float(result) < 0:
        raise ValueError("ratio must be finite and non-negative")
    return result


def _sample_counts(lengths: list[int], ratio: Tensor, *, gpu: bool) -> list[int]:
    """torch_cluster's degree conversion and ceiling (flat.py:150-158).

    Its CPU path converts the batch sizes to float32; its GPU path to the
    ratio's dtype.  Torch scalar promotion then depends on whether a tensor
    ratio is 0-D or of shape [1].
    """
    sizes = torch.tensor(lengths, dtype=ratio.dtype if gpu else torch.float32)
    return torch.ceil(sizes * ratio).to(torch.long).tolist()


def _raise_status(status: Tensor, what: str) -> None:
    code = int(status.item())
    if code == 0:
        return
    if what == "fps" and code == 2:
        raise ValueError("invalid ptr, out_ptr, or starts for the input point clouds")
    if what == "fps" and code == 1:
        raise RuntimeError("mps_pointops: flat FPS cross-CTA exchange timed out")
    raise ValueError(f"{what}: the batch offsets must run from 0 to the point counts without "
                     "decreasing")


def fps(
    x: Tensor,
    batch: Tensor | None = None,
    ratio: float | Tensor | None = None,
    random_start: bool = True,
    batch_size: int | None = None,
    ptr: Tensor | Sequence[int] | None = None,
) -> Tensor:
    """Sample global point indices with the torch_cluster count rule (flat.py:161-217).

    Each cloud yields ``ceil(len * ratio)`` samples (``ratio=None`` means 0.5)
    by farthest point sampling from a random point (``random_start``) or its
    first point; a request longer than the cloud repeats its local index 0
    once every point is taken.  ``ptr`` takes precedence over ``batch``.
    Returns int64 global indices on ``x.device``.
    """
    _points(x, "x")
    if x.device.type == "cuda" and x.dtype != torch.float32:
        raise TypeError("x must be float32 on CUDA")
    sample_ratio = _ratio(ratio, x.dtype)
    offsets = _fps_ptr(x, batch, batch_size, ptr)
    offset_values = offsets.cpu().tolist()
    lengths = [hi - lo for lo, hi in zip(offset_values, offset_values[1:])]
    counts = _sample_counts(lengths, sample_ratio, gpu=x.device.type != "cpu")
    output_offsets = [0]
    for count in counts:
        output_offsets.append(output_offsets[-1] + count)
    if output_offsets[-1] == 0:
        return torch.empty(0, dtype=torch.long, device=x.device)

    if random_start:
        length_tensor = torch.tensor(lengths, dtype=torch.long, device=x.device)
        starts = (torch.rand(len(lengths), device=x.device) * length_tensor).long()
        starts = torch.minimum(starts, (length_tensor - 1).clamp_min(0))
    else:
        starts = torch.zeros(len(lengths), dtype=torch.long, device=x.device)

    N.require_cuda(x, "flat.fps")
    total = output_offsets[-1]
    max_len = max(lengths)
    device = x.device
    out = torch.empty(total, dtype=torch.long, device=device)
    out_ptr = torch.tensor(output_offsets, dtype=torch.long, device=device)
    status = torch.empty(1, dtype=torch.int32, device=device)
    points = x.contiguous()
    starts = starts.contiguous()  # held until the launch is queued
    with N.on_device(device):
        lib = N.lib()
        ws_bytes = int(lib.mpo_flat_fps_workspace_bytes(len(lengths), max_len))
        ws = N.workspace(ws_bytes, device)
        N.check(lib.mpo_flat_fps(N.ptr(points), N.ptr(offsets), N.ptr(out_ptr),
                                 N.ptr(starts), len(lengths), len(x), total, max_len,
                                 N.ptr(out), N.ptr(status), N.ptr(ws), ws_bytes,
                                 N.stream(device)), "flat fps")
    if max_len > 8192:
        # Only the cooperative CTA-group path (clouds above 8192 points) can
        # fail at run time (a bounded exchange wait); the offsets, counts and
        # starts built above are valid by construction.
        _raise_status(status, "fps")
    return out


def _search_inputs(x: Tensor, y: Tensor, *, feature_space: bool = False) -> None:
    validate = _features if feature_space else _points
    validate(x, "x")
    validate(y, "y")
    if x.shape[1] != y.shape[1]:
        raise ValueError(f"x and y feature dimensions differ: {x.shape[1]} and {y.shape[1]}")
    if x.device != y.device:
        raise ValueError(f"x and y must be on the same device, got {x.device} and {y.device}")
    if x.dtype != y.dtype:
        raise TypeError(f"x and y must have the same dtype, got {x.dtype} and {y.dtype}")


def _nonnegative_int(value: int, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise ValueError(f"{name} must be a non-negative integer")
    return value


def _check_cuda_knn_width(width: int) -> None:
    """Reject requests the flat kNN kernels cannot serve (flat.py:238-244)."""
    if width > _CUDA_KNN_MAX_K:
        raise ValueError(f"effective k must be at most {_CUDA_KNN_MAX_K} on CUDA, got {width}")


def _edges(indices: Tensor) -> Tensor:
    """(ny, width) padded global indices -> [query, reference] edges (flat.py:247-253)."""
    if indices.numel() == 0:
        return torch.empty((2, 0), dtype=torch.long, device=indices.device)
    valid = indices >= 0
    queries = torch.arange(indices.shape[0], device=indices.device, dtype=torch.long)
    queries = queries[:, None].expand_as(indices)[valid]
    return torch.stack((queries, indices[valid]), dim=0)


def _radius_sq(r: float) -> float:
    """fl32(r * r) with r * r in double: the threshold torch_cluster compares
    against (mps_pointops/_flat_search_mps.py:66-76)."""
    try:
        return struct.unpack("f", struct.pack("f", r * r))[0]
    except OverflowError:
        return math.inf


def _longest(ptr: Tensor) -> int:
    if ptr.numel() < 2:
        return 0
    return int((ptr[1:] - ptr[:-1]).max().item())


def knn_indices(x: Tensor, y: Tensor, ptr_x: Tensor, ptr_y: Tensor, k: int, *,
                check: bool = True) -> Tensor:
    """(len(y), k) global x indices per query in (squared distance, index)
    order, -1 padded: the flat kNN kernel call (_flat_search_mps.py:79-108).
    ``check=False`` skips reading the device-side offset check (for offsets
    already validated on the host; the kernels stay memory-safe either way)."""
    out = torch.empty((y.shape[0], k), dtype=torch.int64, device=x.device)
    if y.shape[0] == 0 or k == 0:
        return out
    status = torch.empty(1, dtype=torch.int32, device=x.device)
    xc, yc = x.contiguous(), y.contiguous()
    px, py = ptr_x.contiguous(), ptr_y.contiguous()
    # The longest reference cloud only picks the D = 3 kernel (above 2**18
    # references per cloud); the total row count bounds it for free.
    longest = xc.shape[0]
    if xc.shape[1] == 3 and k <= 32 and longest > (1 << 18):
        longest = _longest(px)
    with N.on_device(x.device):
        N.check(N.lib().mpo_flat_knn(N.ptr(xc), N.ptr(yc), N.ptr(px), N.ptr(py), px.numel() - 1,
                                     xc.shape[0], yc.shape[0], xc.shape[1], k, longest,
                                     N.ptr(out), N.ptr(status), N.stream(x.device)), "flat knn")
    if check:
        _raise_status(status, "knn")
    return out


def radius_indices(x: Tensor, y: Tensor, ptr_x: Tensor, ptr_y: Tensor, r: float,
                   max_num_neighbors: int, ignore_same_index: bool = False, *,
                   check: bool = True) -> Tensor:
    """(len(y), max_num_neighbors) first global x indices in input order with
    squared distance < fl32(r * r), -1 padded (_flat_search_mps.py:111-147).
    ``ignore_same_index`` drops the x row whose global index equals the
    query's before the cap (pyg-lib's radius)."""
    # The reference's GPU path validates r like its ball query: it must round
    # to float32, and a positive r to a normal float32 of at least 2**-112.
    radius_f32, _ = _checked_radius_and_k(r, max_num_neighbors)
    out = torch.empty((y.shape[0], max_num_neighbors), dtype=torch.int64, device=x.device)
    if y.shape[0] == 0 or max_num_neighbors == 0:
        return out
    if radius_f32 == 0.0:
        return out.fill_(-1)
    status = torch.empty(1, dtype=torch.int32, device=x.device)
    xc, yc = x.float().contiguous(), y.float().contiguous()
    px, py = ptr_x.contiguous(), ptr_y.contiguous()
    with N.on_device(x.device):
        N.check(N.lib().mpo_flat_radius(N.ptr(xc), N.ptr(yc), N.ptr(px), N.ptr(py), px.numel() - 1,
                                        xc.shape[0], yc.shape[0], _radius_sq(float(r)),
                                        max_num_neighbors, int(bool(ignore_same_index)),
                                        N.ptr(out), N.ptr(status), N.stream(x.device)),
                "flat radius")
    if check:
        _raise_status(status, "radius")
    return out


def knn(
    x: Tensor,
    y: Tensor,
    k: int,
    batch_x: Tensor | None = None,
    batch_y: Tensor | None = None,
    cosine: bool = False,
    num_workers: int = 1,
    batch_size: int | None = None,
) -> Tensor:
    """Global ``[query, reference]`` edges to the nearest points (flat.py:291-329).

    ``batch_size`` sets the number of batch slots, including empty ones.  x and
    y are coordinate or feature vectors with D >= 1; the effective neighbour
    count ``min(k, len(x))`` must be at most 256 on CUDA.  ``cosine=True`` is
    not implemented; ``num_workers`` is accepted for call-site compatibility.
    """
    _search_inputs(x, y, feature_space=True)
    k = _nonnegative_int(k, "k")
    if cosine:
        raise NotImplementedError("cosine kNN is not supported")
    _nonnegative_int(num_workers, "num_workers")
    if x.device.type == "cuda" and x.dtype != torch.float32:
        raise TypeError("x and y must be float32 for kNN on CUDA")
    if k == 0 or len(x) == 0 or len(y) == 0:
        return torch.empty((2, 0), dtype=torch.long, device=x.device)
    ptr_x, ptr_y = _pair_ptrs(x, y, batch_x, batch_y, batch_size)
    width = min(k, len(x))
    N.require_cuda(x, "flat.knn")
    _check_cuda_knn_width(width)
    return _edges(knn_indices(x, y, ptr_x, ptr_y, width, check=False))


def radius(
    x: Tensor,
    y: Tensor,
    r: float,
    batch_x: Tensor | None = None,
    batch_y: Tensor | None = None,
    max_num_neighbors: int = 32,
    num_workers: int = 1,
    batch_size: int | None = None,
    ignore_same_index: bool = False,
) -> Tensor:
    """Global ``[query, reference]`` edges with squared distance ``< r²``
    (flat.py:332-373): neighbours in reference input order, at most
    ``max_num_neighbors`` per query.  ``ignore_same_index=True`` is not
    implemented here (the PyG operator surface in :mod:`mps_pointops.pyg`
    offers it); ``num_workers`` is accepted for call-site compatibility.
    """
    _search_inputs(x, y)
    limit = _nonnegative_int(max_num_neighbors, "max_num_neighbors")
    _nonnegative_int(num_workers, "num_workers")
    if ignore_same_index:
        raise NotImplementedError("ignore_same_index=True is not supported")
    if isinstance(r, bool) or not isinstance(r, (int, float)):
        raise ValueError("r must be a finite non-negative number")
    r = float(r)
    if not math.isfinite(r) or r < 0:
        raise ValueError("r must be a finite non-negative number")
    if x.device.type == "cuda" and x.dtype not in (torch.float16, torch.float32):
        raise TypeError("x and y must be float16 or float32 for radius on CUDA")
    if limit == 0 or len(x) == 0 or len(y) == 0:
        return torch.empty((2, 0), dtype=torch.long, device=x.device)
    ptr_x, ptr_y = _pair_ptrs(x, y, batch_x, batch_y, batch_size)
    width = min(limit, len(x))
    N.require_cuda(x, "flat.radius")
    return _edges(radius_indices(x, y, ptr_x, ptr_y, r, width, check=False))


def _graph_edges(edges: Tensor, loop: bool, flow: str) -> Tensor:
    if flow not in ("source_to_target", "target_to_source"):
        raise ValueError("flow must be 'source_to_target' or 'target_to_source'")
    if flow == "source_to_target":
        edges = edges.flip(0)
    if not loop:
        edges = edges[:, edges[0] != edges[1]]
    return edges


def knn_graph(
    x: Tensor,
    k: int,
    batch: Tensor | None = None,
    loop: bool = False,
    flow: str = "source_to_target",
    cosine: bool = False,
    num_workers: int = 1,
    batch_size: int | None = None,
) -> Tensor:
    """kNN graph with ``torch_cluster`` 1.6.3 edge orientation (flat.py:386-404)."""
    k = _nonnegative_int(k, "k")
    if flow not in ("source_to_target", "target_to_source"):
        raise ValueError("flow must be 'source_to_target' or 'target_to_source'")
    edges = knn(
        x, x, k if loop else k + 1, batch, batch,
        cosine=cosine, num_workers=num_workers, batch_size=batch_size,
    )
    return _graph_edges(edges, loop, flow)


def radius_graph(
    x: Tensor,
    r: float,
    batch: Tensor | None = None,
    loop: bool = False,
    max_num_neighbors: int = 32,
    flow: str = "source_to_target",
    num_workers: int = 1,
    batch_size: int | None = None,
) -> Tensor:
    """Radius graph with ``torch_cluster`` 1.6.3 edge orientation (flat.py:407-425)."""
    limit = _nonnegative_int(max_num_neighbors, "max_num_neighbors")
    if flow not in ("source_to_target", "target_to_source"):
        raise ValueError("flow must be 'source_to_target' or 'target_to_source'")
    edges = radius(
        x, x, r, batch, batch, limit if loop else limit + 1,
        num_workers=num_workers, batch_size=batch_size,
    )
    return _graph_edges(edges, loop, flow)


__all__ = ["fps", "knn", "radius", "knn_graph", "radius_graph"]
