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


def _with_workspace(xyz, npoint, start, strategy, skip=0, int32=0):
    lib = N.lib()
    B, n, _ = xyz.shape
    dtype = torch.int32 if int32 else torch.long
    out = torch.full((B, npoint), -5, dtype=dtype, device=xyz.device)
    ws = torch.zeros(max(1, lib.mpo_fps_workspace_bytes(B, n, npoint, strategy)),
                     dtype=torch.uint8, device=xyz.device)
    N.check(lib.mpo_fps(N.ptr(xyz), B, n, npoint, start, skip, int32, strategy, N.ptr(out), None,
                        N.ptr(ws), ws.numel(), N.stream(xyz.device)), "mpo_fps")
    return out


def _no_alloc(xyz, npoint, start, strategy, skip=0, int32=0):
    lib = N.lib()
    B, n, _ = xyz.shape
    dtype = torch.int32 if int32 else torch.long
    out = torch.full((B, npoint), -7, dtype=dtype, device=xyz.device)
    status = torch.full((1,), 9, dtype=torch.int32, device=xyz.device)
    N.check(lib.mpo_fps_noalloc(N.ptr(xyz), B, n, npoint, start, skip, int32, strategy,
                                N.ptr(out), N.ptr(status), N.stream(xyz.device)),
            "mpo_fps_noalloc")
    return out, status


@pytest.mark.parametrize("strategy", [0, 1])   # MPO_FPS_AUTO, MPO_FPS_SINGLE
def test_no_alloc_one_cta_path_matches_workspace_entry_point(cuda_device, strategy):
    """Clouds of up to 8192 points run one CTA per cloud and need no scratch;
    the allocation-free entry keeps its own one-CTA kernel there, so it is
    compared with mpo_fps at several sizes, with skip_near_origin and the
    int32 output, twice in a row."""
    for n, b, npoint, start in ((1, 1, 1, 0), (33, 3, 33, 5), (4097, 2, 1024, 7),
                                (8192, 4, 2048, 8191), (2000, 9, 600, 0)):
        xyz = _cloud(b, n, seed=n).to(cuda_device)
        xyz[:, : max(1, n // 10)] *= 1e-3          # some points near the origin
        for skip, int32 in ((0, 0), (1, 1), (1, 0), (0, 1)):
            for _ in range(2):
                want = _with_workspace(xyz, npoint, start, strategy, skip, int32)
                got, status = _no_alloc(xyz, npoint, start, strategy, skip, int32)
                torch.cuda.synchronize()
                assert status.item() == 0
                assert torch.equal(got, want), (n, b, skip, int32)


def test_no_alloc_shared_memory_tier(cuda_device):
    """1.5 M points: every SM takes part and each CTA keeps the points beyond
    8192 in shared memory (no workspace needed); 4 M points would need the
    workspace tier, which this entry point rejects."""
    xyz = _cloud(1, 1_500_000, seed=5).to(cuda_device)
    for _ in range(2):
        got, status = _no_alloc(xyz, 300, 11, 0)
        torch.cuda.synchronize()
        assert status.item() == 0 and torch.equal(got, _with_workspace(xyz, 300, 11, 0))
    lib = N.lib()
    big = torch.zeros(1, 4_000_000, 3, device=cuda_device)
    out = torch.empty(1, 4, dtype=torch.long, device=cuda_device)
    rc = lib.mpo_fps_noalloc(N.ptr(big), 1, 4_000_000, 4, 0, 0, 0, 0, N.ptr(out), None,
                             N.stream(cuda_device))
    assert rc == 1 and b"need workspace" in lib.mpo_last_error()


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
