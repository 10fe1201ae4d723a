"""FPS on B200 vs the reference's CPU path (golden fixtures) and the oracle.

Indices must be bit-exact (mps_pointops/reference.py:27-58 contract); cases
follow gamzerA/mps-pointops tests/test_fps.py and tests/test_compat.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mps_pointops
from conftest import golden
from mps_pointops import compat
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def cloud(b, n, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, n, 3, generator=g)


@pytest.mark.parametrize("strategy", ["auto", "multigroup"])
def test_golden_cases(cuda_device, strategy):
    for name, c in golden("fps").items():
        npoint, start, skip = (int(v) for v in c["meta"])
        xyz = torch.from_numpy(c["xyz"]).to(cuda_device)
        if strategy == "multigroup" and xyz.shape[0] > 1:
            continue
        got = mps_pointops.furthest_point_sample(xyz, npoint, start, bool(skip), strategy=strategy)
        assert got.dtype == torch.long
        np.testing.assert_array_equal(got.cpu().numpy(), c["idx"], err_msg=f"{name}/{strategy}")


def test_compat_int32_skip_near_origin(cuda_device):
    c = golden("fps")["skip_near_origin"]
    got = compat.furthest_point_sample(torch.from_numpy(c["xyz"]).to(cuda_device), 2000)
    assert got.dtype == torch.int32
    np.testing.assert_array_equal(got.cpu().numpy(), c["idx"].astype(np.int32))
    picked = set(got[0].tolist())
    assert picked.isdisjoint(range(1, 41)) and 41 in picked
    zeros = compat.furthest_point_sample(torch.zeros(1, 50, 3, device=cuda_device), 5)
    assert zeros.tolist() == [[0, 0, 0, 0, 0]]


@pytest.mark.parametrize("n", [1, 2, 31, 32, 33, 1023, 1024, 1025, 2049, 4096, 5000, 8192, 8193,
                               20000])
def test_sizes_match_oracle(cuda_device, n):
    xyz = cloud(2, n, seed=n)
    npoint = min(n, 300)
    want = O.furthest_point_sample(xyz.numpy(), npoint, n // 3, False)
    got = mps_pointops.furthest_point_sample(xyz.to(cuda_device), npoint, n // 3)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("n", [2, 33, 4097, 8193, 100_000])
def test_group_path_matches_single(cuda_device, n):
    xyz = cloud(1, n, seed=19).to(cuda_device)
    auto = mps_pointops.furthest_point_sample(xyz, 128, start_idx=1, strategy="auto")
    group = mps_pointops.furthest_point_sample(xyz, 128, start_idx=1, strategy="multigroup")
    assert torch.equal(auto, group)
    want = O.furthest_point_sample(xyz.cpu().numpy(), 128, 1, False)
    np.testing.assert_array_equal(group.cpu().numpy(), want)


def _sphere(n, seed):
    """BASELINE config 3's distribution: unit sphere, N(0, 0.01) radial jitter."""
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(1, n, 3, generator=g)
    p = p / p.norm(dim=-1, keepdim=True)
    return p * (1 + 0.01 * torch.randn(1, n, 1, generator=g))


def _large_case(name):
    import hashlib
    c = golden("fps_large")[name]
    n, npoint, seed = (int(v) for v in c["meta"])
    xyz = _sphere(n, seed)
    digest = np.frombuffer(hashlib.sha256(xyz.numpy().tobytes()).digest(), dtype=np.uint8)
    assert np.array_equal(digest, c["sha256"]), "torch's generator no longer rebuilds this input"
    return xyz, npoint, c["idx"].astype(np.int64)


def test_config3_full_run_matches_reference(cuda_device):
    """BASELINE config 3 end to end: 65,536 samples from 2^20 points, against
    reference.furthest_point_sample's own output (tests/golden/fps_large.npz).
    The 8-bit step sequence of the cross-CTA exchange wraps 256 times."""
    xyz, npoint, want = _large_case("config3")
    got = mps_pointops.furthest_point_sample(xyz.to(cuda_device), npoint)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    # the first 256 steps also against the C oracle
    np.testing.assert_array_equal(want[:, :256], O.furthest_point_sample(xyz.numpy(), 256, 0,
                                                                         False))


@pytest.mark.parametrize("name", ["n1p5m", "n4m"])
def test_beyond_8192_points_per_sm_matches_reference(cuda_device, name):
    """1.5 M points (registers + shared-memory tier) and 4 M points (registers
    + shared memory + workspace tier): 1024 samples against the reference's
    CPU path and the C oracle."""
    xyz, npoint, want = _large_case(name)
    got = mps_pointops.furthest_point_sample(xyz.to(cuda_device), npoint)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    np.testing.assert_array_equal(want, O.furthest_point_sample(xyz.numpy(), npoint, 0, False))


def test_overflow_tiers_edge_cases(cuda_device):
    """Tier boundaries, skip_near_origin, a NaN in the workspace tier, ties on
    a lattice, a non-zero start and several clouds: all against the oracle."""
    g = torch.Generator().manual_seed(31)
    n = 3_600_000                       # beyond registers + shared memory on 148 SMs
    xyz = torch.randint(0, 40, (1, n, 3), generator=g).float()      # many exact ties
    xyz[0, 5:20000] *= 1e-3 / 40                                   # near the origin
    _check(xyz, 200, 12345, True, cuda_device)
    xyz2 = torch.randn(1, n, 3, generator=g)
    xyz2[0, n - 17, 1] = float("nan")                              # in the last CTA's tail
    _check(xyz2, 64, 0, False, cuda_device)
    two = torch.randn(2, 1_300_000, 3, generator=g)                # two clouds, one wave each
    _check(two, 128, 77, False, cuda_device)


def test_group_status_word_reports_success(cuda_device):
    from mps_pointops import _native as N
    xyz = cloud(1, 20000, seed=3).to(cuda_device)
    out = torch.empty(1, 64, dtype=torch.long, device=cuda_device)
    status = torch.full((1,), 7, dtype=torch.int32, device=cuda_device)
    lib = N.lib()
    ws = torch.empty(lib.mpo_fps_workspace_bytes(1, 20000, 64, 2), dtype=torch.uint8,
                     device=cuda_device)
    N.check(lib.mpo_fps(N.ptr(xyz), 1, 20000, 64, 0, 0, 0, 2, N.ptr(out), N.ptr(status),
                        N.ptr(ws), ws.numel(), N.stream(cuda_device)), "fps")
    torch.cuda.synchronize()
    assert status.item() == 0
    np.testing.assert_array_equal(out.cpu().numpy(),
                                  O.furthest_point_sample(xyz.cpu().numpy(), 64, 0, False))


def test_noncontiguous_and_empty(cuda_device):
    xyz = cloud(1, 4000)[:, ::2]
    got = mps_pointops.furthest_point_sample(xyz.to(cuda_device), 100)
    np.testing.assert_array_equal(got.cpu().numpy(),
                                  O.furthest_point_sample(xyz.numpy(), 100, 0, False))
    x = torch.randn(3, 50, 3, device=cuda_device)
    assert mps_pointops.furthest_point_sample(x, 0).shape == (3, 0)
    assert mps_pointops.furthest_point_sample(x[:0], 5).shape == (0, 5)
    with pytest.raises(TypeError):
        mps_pointops.furthest_point_sample(x.half(), 4)
    with pytest.raises(ValueError, match="batch size 1"):
        mps_pointops.furthest_point_sample(x, 8, strategy="multigroup")


def test_nan_points_follow_torch_argmax(cuda_device):
    xyz = cloud(1, 300, seed=5)
    xyz[0, 17, 1] = float("nan")
    want = O.furthest_point_sample(xyz.numpy(), 20, 0, False)
    got = mps_pointops.furthest_point_sample(xyz.to(cuda_device), 20)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


# ---- one-CTA path (fps_cta_kernel: contiguous points per thread) on long runs,
# ties, duplicates, skip-near-origin, non-finite and overflowing clouds ------------------
def _check(xyz, npoint, start=0, skip=False, device=None):
    want = O.furthest_point_sample(xyz.numpy(), npoint, start, skip)
    got = mps_pointops.furthest_point_sample(xyz.to(device), npoint, start, skip)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("n", [2048, 4097, 6000, 8192])
def test_cta_uniform_cube_all_samples(cuda_device, n):
    """Config 1's distribution, sampled to a quarter and to every point."""
    g = torch.Generator().manual_seed(n)
    xyz = torch.rand(2, n, 3, generator=g)
    _check(xyz, n // 4, 0, False, cuda_device)
    _check(xyz[:1], n, n - 1, False, cuda_device)


def test_cta_lattice_ties(cuda_device):
    """Integer lattice: min_d2 ties everywhere; the first index must win."""
    g = torch.Generator().manual_seed(8)
    xyz = torch.randint(0, 6, (2, 6144, 3), generator=g).float()
    _check(xyz, 1024, 5, False, cuda_device)
    _check(xyz, 6144, 0, False, cuda_device)


def test_cta_duplicates_and_degenerate_extent(cuda_device):
    xyz = torch.zeros(1, 5000, 3)
    _check(xyz, 100, 7, False, cuda_device)
    line = torch.zeros(1, 4500, 3)
    line[0, :, 1] = torch.arange(4500, dtype=torch.float32) % 97
    _check(line, 300, 0, False, cuda_device)


def test_cta_skip_near_origin_and_clusters(cuda_device):
    g = torch.Generator().manual_seed(21)
    centres = torch.rand(12, 3, generator=g) * 20 - 10
    labels = torch.randint(0, 12, (1, 5000), generator=g)
    xyz = centres[labels] + 0.3 * torch.randn(1, 5000, 3, generator=g)
    xyz[0, 100:400] = 0.01 * torch.randn(300, 3, generator=g)   # many near the origin
    _check(xyz, 1500, 0, True, cuda_device)
    _check(xyz, 1500, 250, False, cuda_device)


def test_cta_nonfinite_and_overflowing_clouds(cuda_device):
    g = torch.Generator().manual_seed(22)
    xyz = torch.randn(1, 5000, 3, generator=g)
    xyz[0, 1234, 2] = float("nan")
    _check(xyz, 200, 0, False, cuda_device)
    xyz = torch.randn(1, 5000, 3, generator=g)
    xyz[0, 77, 0] = float("inf")
    _check(xyz, 200, 0, False, cuda_device)
    big = torch.randn(1, 4200, 3, generator=g) * 3e19   # squared distances overflow to inf
    _check(big, 150, 3, False, cuda_device)


def test_cta_fps_gather_and_int32(cuda_device):
    g = torch.Generator().manual_seed(23)
    xyz = torch.rand(3, 6000, 3, generator=g)
    want = O.furthest_point_sample(xyz.numpy(), 1024, 0, True).astype(np.int32)
    got = compat.furthest_point_sample(xyz.to(cuda_device), 1024)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
