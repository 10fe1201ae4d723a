"""The peer-memory loss all-reduce kernel (mpo_allreduce_sum_f32_p2p) on ONE
GPU.  Kernels of different ranks wait on one another, so they never run as
separate launches on one GPU here; instead each test plays one rank whose
"peers" are plain local arrays: the other ranks' words are written into this
rank's array beforehand (as their stores would have), and the test reads the
words this rank stored into the peers' arrays.  The bounded wait is checked
with a word that nothing ever writes (20 ms limit).  The multi-rank path
over CUDA IPC runs in tests/test_dist_nccl_gpu.py when two GPUs are visible."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from mps_pointops import _native as N

pytestmark = pytest.mark.gpu

MAX_RANKS = 32
SHORT_NS = 20_000_000


def word(seq: int, v: float) -> int:
    bits = int(np.array([v], dtype=np.float32).view(np.uint32)[0])
    w = (seq << 32) | bits
    return w - (1 << 64) if w >= 1 << 63 else w      # as int64


def arrays(n, dev):
    return [torch.zeros(2 * MAX_RANKS, dtype=torch.int64, device=dev) for _ in range(n)]


def run(value, scale, slots, rank, seq, dev, timeout_ns=2_000_000_000, status=None):
    out = torch.full((1,), -7.0, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev) if status is None else status
    v = torch.tensor([value], dtype=torch.float32, device=dev)
    ptrs = (ctypes.c_void_p * len(slots))(*[s.data_ptr() for s in slots])
    N.check(N.lib().mpo_allreduce_sum_f32_p2p(N.ptr(v), ctypes.c_float(scale), N.ptr(out), ptrs,
                                              len(slots), rank, seq, timeout_ns, N.ptr(status),
                                              N.stream(dev)), "allreduce")
    torch.cuda.synchronize()
    return out.item(), int(status.item())


def test_single_rank(cuda_device):
    (a,) = arrays(1, cuda_device)
    got, st = run(3.5, 0.25, [a], 0, 1, cuda_device)
    assert st == 0 and got == 0.875
    assert int(a[MAX_RANKS + 0]) == word(1, 0.875)      # seq 1 -> bank 1


def test_rank_order_sum_and_stores(cuda_device):
    """Rank 2 of 4: ranks 0, 1, 3 already stored 1e8, 1, 1 into its array; its
    own value is -4e8 * 0.25 = -1e8.  The sum in rank order is
    ((1e8 + 1) - 1e8) + 1 = 1 (1e8 + 1 rounds to 1e8); any order that adds
    -1e8 before 1e8 + 1 gives 2."""
    seq, rank = 6, 2
    slots = arrays(4, cuda_device)
    own = slots[rank]
    bank = (seq & 1) * MAX_RANKS
    for r, v in ((0, 1e8), (1, 1.0), (3, 1.0)):
        own[bank + r] = word(seq, v)
    got, st = run(-4e8, 0.25, slots, rank, seq, cuda_device)
    assert st == 0 and got == 1.0
    for r in range(4):
        assert int(slots[r][bank + rank]) == word(seq, -1e8)
        assert int(slots[r][(1 - (seq & 1)) * MAX_RANKS + rank]) == 0   # other bank untouched


def test_missing_rank_times_out(cuda_device):
    slots = arrays(3, cuda_device)
    seq = 9
    bank = (seq & 1) * MAX_RANKS
    slots[0][bank + 2] = word(seq, 5.0)                   # rank 1 never stores
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    got, st = run(1.0, 1.0, slots, 0, seq, cuda_device, SHORT_NS, status)
    assert math.isnan(got) and st == 2                    # 1 + the missing rank
    # The status is sticky; a later complete reduction still computes.
    slots[0][(10 & 1) * MAX_RANKS + 1] = word(10, 2.0)
    slots[0][(10 & 1) * MAX_RANKS + 2] = word(10, 4.0)
    got, st = run(1.0, 1.0, slots, 0, 10, cuda_device, SHORT_NS, status)
    assert got == 7.0 and st == 2


def test_stale_word_is_not_taken(cuda_device):
    """A word of reduction seq - 2 (same bank) must not satisfy reduction seq."""
    slots = arrays(2, cuda_device)
    slots[0][(5 & 1) * MAX_RANKS + 1] = word(3, 123.0)
    got, st = run(1.0, 1.0, slots, 0, 5, cuda_device, SHORT_NS)
    assert math.isnan(got) and st == 2
    slots[0][(5 & 1) * MAX_RANKS + 1] = word(5, 123.0)
    got, st = run(1.0, 1.0, slots, 0, 5, cuda_device, SHORT_NS)
    assert got == 124.0 and st == 0


def test_create_and_destroy_exchange_array(cuda_device):
    lib = N.lib()
    slots = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    N.check(lib.mpo_p2p_slots_create(ctypes.byref(slots), handle), "create")
    assert slots.value and any(handle)
    assert lib.mpo_p2p_slots_bytes() == 2 * MAX_RANKS * 8
    N.check(lib.mpo_p2p_slots_destroy(slots), "destroy")
