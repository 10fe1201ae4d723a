"""Multi-GPU partitioning of the point-cloud ops (one process per GPU).

The reference is single-device; this module adds the data-parallel layout of
the batched workloads.  Independent clouds (or, for one very large cloud,
contiguous query ranges against a replicated reference cloud) are split
contiguously over the ranks of a ``torch.distributed`` process group; every
rank runs the single-GPU kernels on its shard.  The only cross-rank traffic is

* ``all_gather_shards``: an ``all_gather_into_tensor`` of per-shard outputs
  (indices, distances) when every rank needs the full result, and
* ``chamfer_distance_sharded``: one ``all_reduce(SUM)`` of the Chamfer loss
  partials -- the gradients of a cloud depend only on that cloud, so no
  gradient exchange is needed.

Both go through NCCL over NVLink on GPUs and work with ``gloo`` on the CPU.
For the 4-byte loss all-reduce of a data-parallel step, ``PeerLossReducer``
replaces NCCL with the library's own kernel over peer memory (one NVLink
store per rank pair and a bounded poll), which has a fraction of the
latency of a collective launch.
The functions take the local op as a parameter (``local_fn``) so the
partitioning logic can be exercised without a GPU.
"""

from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) slice of ``total`` items owned by ``rank``; the first
    ``total % world`` ranks get one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _world(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def all_gather_shards(local: torch.Tensor, total: int, dim: int = 0, group=None) -> torch.Tensor:
    """Concatenate every rank's shard of a tensor split along ``dim`` by
    :func:`shard_range` into the full tensor on every rank."""
    rank, world = _world(group)
    sizes = [shard_range(total, r, world) for r in range(world)]
    longest = max(hi - lo for lo, hi in sizes)
    moved = local.movedim(dim, 0).contiguous()
    pad = longest - moved.shape[0]
    if pad:
        moved = torch.cat([moved, moved.new_zeros((pad, *moved.shape[1:]))])
    out = moved.new_empty((world * longest, *moved.shape[1:]))
    dist.all_gather_into_tensor(out, moved, group=group)
    parts = [out[r * longest: r * longest + (hi - lo)] for r, (lo, hi) in enumerate(sizes)]
    return torch.cat(parts).movedim(0, dim)


class PendingLoss:
    """The global Chamfer loss of :func:`chamfer_distance_sharded` with
    ``overlap=True``: its all-reduce runs on the communication stream while the
    caller goes on (backward, next step); :meth:`value` waits for it (the
    current stream waits on the collective, the host does not)."""

    def __init__(self, total: torch.Tensor, work):
        self._total, self._work = total, work

    def value(self) -> torch.Tensor:
        if self._work is not None:
            self._work.wait()
            self._work = None
        return self._total


class _StreamWork:
    """The wait handle of a reduction enqueued on a side stream: waiting makes
    the caller's current stream wait for it (the host does not block)."""

    def __init__(self, stream: torch.cuda.Stream):
        self._stream = stream

    def wait(self):
        torch.cuda.current_stream(self._stream.device).wait_stream(self._stream)


class PeerLossReducer:
    """All-reduce (sum) of one float per rank through the ranks' peer memory,
    for the global loss of a data-parallel Chamfer step on the GPUs of one
    node (``mpo_allreduce_sum_f32_p2p``).

    Construction is collective: every rank of ``group`` creates its exchange
    array, the CUDA IPC handles are all-gathered, and each rank maps the
    others' arrays.  :meth:`reduce` enqueues one 32-thread kernel on a side
    stream that stores this rank's value into every rank's array over NVLink
    and waits (bounded by ``timeout_s``) for all of theirs; the result is the
    values summed in rank order, the same bits on every rank.  Every rank must
    call :meth:`reduce` the same number of times, in the same order.
    :meth:`check` raises if a wait ran out; :meth:`close` (collective) frees
    the mappings.
    """

    def __init__(self, group=None, timeout_s: float = 10.0):
        from . import _native as N
        self._N = N
        self._lib = N.lib()
        self.rank, self.world = _world(group)
        self._group = group
        self.device = torch.device("cuda", torch.cuda.current_device())
        limit = 32
        if self.world > limit:
            raise ValueError(f"PeerLossReducer: at most {limit} ranks, got {self.world}")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        N.check(self._lib.mpo_p2p_slots_create(ctypes.byref(own), handle), "mpo_p2p_slots_create")
        self._own = own.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._mapped: list[int] = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            N.check(self._lib.mpo_p2p_slots_open(buf, ctypes.byref(p)), "mpo_p2p_slots_open")
            self._mapped.append(p.value)
            ptrs.append(p.value)
        self._slots = (ctypes.c_void_p * self.world)(*ptrs)
        self._seq = 0
        self._timeout_ns = int(timeout_s * 1e9)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._stream = torch.cuda.Stream(self.device)

    def reduce(self, value: torch.Tensor, scale: float = 1.0) -> "PendingLoss":
        """Sum of fl(value[0] * scale) over the ranks (float32, one element),
        as a :class:`PendingLoss`."""
        if value.dtype != torch.float32 or value.numel() != 1 or value.device != self.device:
            raise ValueError("PeerLossReducer.reduce: value must be one float32 element on "
                             f"{self.device}")
        if self._slots is None:
            raise RuntimeError("PeerLossReducer: closed")
        value = value.detach().contiguous()
        self._seq = self._seq % 0xFFFFFFFF + 1
        out = torch.empty(1, dtype=torch.float32, device=self.device)
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        self._N.check(self._lib.mpo_allreduce_sum_f32_p2p(
            self._N.ptr(value), ctypes.c_float(scale), self._N.ptr(out), self._slots, self.world,
            self.rank, self._seq, self._timeout_ns, self._N.ptr(self._status),
            ctypes.c_void_p(self._stream.cuda_stream)), "mpo_allreduce_sum_f32_p2p")
        value.record_stream(self._stream)
        out.record_stream(self._stream)
        return PendingLoss(out.view(()), _StreamWork(self._stream))

    def check(self) -> None:
        """Raise if any reduction so far gave up waiting (synchronises)."""
        st = int(self._status.item())
        if st:
            raise RuntimeError(f"PeerLossReducer: no value from rank {st - 1} within "
                               f"{self._timeout_ns / 1e9:g} s (loss reported as NaN)")

    def close(self) -> None:
        """Collective: unmap the other ranks' arrays and free this rank's."""
        if self._slots is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._group)
        for p in self._mapped:
            self._N.check(self._lib.mpo_p2p_slots_close(ctypes.c_void_p(p)), "mpo_p2p_slots_close")
        self._mapped = []
        dist.barrier(group=self._group)
        self._N.check(self._lib.mpo_p2p_slots_destroy(ctypes.c_void_p(self._own)),
                      "mpo_p2p_slots_destroy")
        self._slots = None


def chamfer_distance_sharded(x_local: torch.Tensor, y_local: torch.Tensor, batch_total: int,
                             group=None, local_fn: Callable | None = None,
                             overlap: bool = False, reducer: PeerLossReducer | None = None):
    """Mean/mean squared-L2 Chamfer loss over a batch split across ranks.

    ``x_local`` / ``y_local`` hold this rank's clouds (its :func:`shard_range`
    slice of ``batch_total``).  Returns the global loss (identical on every
    rank); its backward yields exactly this rank's slice of the single-GPU
    gradient, because loss = (1/B) * sum over clouds of the per-cloud loss.

    With ``overlap`` it returns ``(local, pending)`` instead: ``local`` is this
    rank's term (1/B) * sum of its per-cloud losses, whose backward gives the
    same gradients, and ``pending`` (:class:`PendingLoss`) the global loss,
    all-reduced asynchronously -- the collective then never stalls the
    compute stream between forward and backward.  ``reducer`` (with
    ``overlap``) sums the partials with a :class:`PeerLossReducer` instead of
    NCCL.
    """
    if local_fn is None:
        from .chamfer import chamfer_distance as local_fn
    partial, _ = local_fn(x_local, y_local, batch_reduction="sum")
    scale = 1.0 / max(batch_total, 1)
    if overlap and reducer is not None:
        return partial * scale, reducer.reduce(partial, scale)
    if overlap:
        local = partial * scale
        total = local.detach().clone()
        work = dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group, async_op=True)
        return local, PendingLoss(total, work)
    total = partial.detach().clone()
    dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return partial * scale + (total - partial.detach()) * scale


def knn_query_sharded(query: torch.Tensor, ref: torch.Tensor, k: int, group=None,
                      gather: bool = True, local_fn: Callable | None = None):
    """kNN of a large query set against a replicated reference cloud: rank r
    searches its contiguous query slice; with ``gather`` the (dist, idx)
    shards are all-gathered along the query axis."""
    if local_fn is None:
        from .ops import knn as local_fn
    rank, world = _world(group)
    lo, hi = shard_range(query.shape[1], rank, world)
    d, i = local_fn(query[:, lo:hi], ref, k)
    if not gather:
        return d, i
    return (all_gather_shards(d, query.shape[1], dim=1, group=group),
            all_gather_shards(i, query.shape[1], dim=1, group=group))


def ball_query_sharded(query: torch.Tensor, ref: torch.Tensor, radius: float, K: int, group=None,
                       gather: bool = True, local_fn: Callable | None = None):
    """Ball query of a large query set against a replicated reference cloud,
    partitioned like :func:`knn_query_sharded`."""
    if local_fn is None:
        from .ops import ball_query as local_fn
    rank, world = _world(group)
    lo, hi = shard_range(query.shape[1], rank, world)
    d, i = local_fn(query[:, lo:hi], ref, radius, K)
    if not gather:
        return d, i
    return (all_gather_shards(d, query.shape[1], dim=1, group=group),
            all_gather_shards(i, query.shape[1], dim=1, group=group))


def batch_sharded(fn: Callable, *tensors: torch.Tensor, batch_total: int, group=None,
                  gather: bool = True, **kwargs):
    """Run ``fn`` on this rank's slice of independent clouds (dim 0) and
    optionally all-gather every tensor output along dim 0."""
    rank, world = _world(group)
    lo, hi = shard_range(batch_total, rank, world)
    out = fn(*(t[lo:hi] for t in tensors), **kwargs)
    if not gather:
        return out
    if isinstance(out, torch.Tensor):
        return all_gather_shards(out, batch_total, 0, group)
    return tuple(all_gather_shards(o, batch_total, 0, group) for o in out)
