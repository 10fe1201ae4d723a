"""The allocation-free FPS entry point, mpo_fps_noalloc, on the GPU.

It is meant for callers that cannot allocate device memory themselves -- a
plugin whose host application passes it nothing but the input and output
buffers, or a loop that is not allowed to allocate once running -- so it keeps
the cross-CTA scratch of the large-cloud path in a fixed array inside the
library instead of a caller workspace.  This test calls it through the C ABI
twice in a row (the second call must not see the first call's scratch) and
requires exactly the indices of the workspace-taking entry point, mpo_fps
(index outputs: tolerance 0).  It sits in its own file, collected last, and
passes both alone and after the rest of the suite.
"""

from __future__ import annotations

import pytest
import torch

from mps_pointops import _native as N

pytestmark = pytest.mark.gpu

GROUP = 2  # MPO_FPS_GROUP: the path that uses the scratch


def _cloud(b, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, n, 3, generator=g)


def _with_workspace(xyz, npoint, start, strategy):
    lib = N.lib()
    B, n, _ = xyz.shape
    out = torch.full((B, npoint), -5, dtype=torch.long, device=xyz.device)
    ws = torch.zeros(max(1, lib.mpo_fps_workspace_bytes(B, n, npoint, strategy)),
                     dtype=torch.uint8, device=xyz.device)
    N.check(lib.mpo_fps(N.ptr(xyz), B, n, npoint, start, 0, 0, strategy, N.ptr(out), None,
                        N.ptr(ws), ws.numel(), N.stream(xyz.device)), "mpo_fps")
    return out


def _no_alloc(xyz, npoint, start, strategy):
    lib = N.lib()
    B, n, _ = xyz.shape
    out = torch.full((B, npoint), -7, dtype=torch.long, device=xyz.device)
    status = torch.full((1,), 9, dtype=torch.int32, device=xyz.device)
    N.check(lib.mpo_fps_noalloc(N.ptr(xyz), B, n, npoint, start, 0, 0, strategy, N.ptr(out),
                                N.ptr(status), N.stream(xyz.device)), "mpo_fps_noalloc")
    return out, status


def test_no_alloc_fps_matches_workspace_entry_point_twice(cuda_device):
    first = _cloud(3, 20000, seed=1).to(cuda_device)     # 3 CTAs per cloud
    second = _cloud(2, 9000, seed=2).to(cuda_device)     # different B, N and start
    for xyz, npoint, start in ((first, 300, 5), (second, 257, 4444)):
        want = _with_workspace(xyz, npoint, start, GROUP)
        got, status = _no_alloc(xyz, npoint, start, GROUP)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert torch.equal(got, want)
    # auto strategy on a large cloud also takes the scratch path
    big = _cloud(1, 70000, seed=3).to(cuda_device)
    got, status = _no_alloc(big, 64, 0, 0)
    torch.cuda.synchronize()
    assert status.item() == 0 and torch.equal(got, _with_workspace(big, 64, 0, 0))


def test_no_alloc_fps_large_batch_reuses_scratch(cuda_device):
    """200 clouds of 20000 points: 3 CTAs per cloud, several cooperative waves
    that reuse the same fixed scratch one after another."""
    xyz = _cloud(200, 20000, seed=4).to(cuda_device)
    want = _with_workspace(xyz, 16, 7, GROUP)
    got, status = _no_alloc(xyz, 16, 7, GROUP)
    torch.cuda.synchronize()
    assert status.item() == 0 and torch.equal(got, want)
