"""kNN (xyz and feature space) and three_nn on B200 vs the reference's exact
oracles (tests/test_knn.py:15-23, tests/test_feature_knn.py:16-35 of
gamzerA/mps-pointops) and the C oracle.  Indices and squared distances are
bit-exact; Euclidean distances are IEEE sqrt of those (compared exactly to the
oracle, rtol 1e-6 to fixtures made with torch's CPU sqrt)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mps_pointops
from conftest import golden
from mps_pointops import _native as N
from mps_pointops import compat
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def cloud(b, n, seed=0, d=3):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, n, d, generator=g)


def check(query, ref, k, device):
    want_d, want_i = O.knn(query.numpy(), ref.numpy(), k)
    d, i = mps_pointops.knn(query.to(device), ref.to(device), k)
    assert d.dtype == torch.float32 and i.dtype == torch.long
    assert d.shape == i.shape == (query.shape[0], query.shape[1], k)
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)


def test_golden_xyz(cuda_device):
    for name, c in golden("knn").items():
        d, i = mps_pointops.knn(torch.from_numpy(c["query"]).to(cuda_device),
                                torch.from_numpy(c["ref"]).to(cuda_device), int(c["k"]))
        np.testing.assert_array_equal(i.cpu().numpy(), c["idx"], err_msg=name)
        np.testing.assert_allclose(d.cpu().numpy(), c["dist"], rtol=1e-6, atol=0, err_msg=name)


def test_golden_feature(cuda_device):
    for name, c in golden("feature_knn").items():
        d, i = mps_pointops.knn(torch.from_numpy(c["query"]).to(cuda_device),
                                torch.from_numpy(c["ref"]).to(cuda_device), int(c["k"]))
        np.testing.assert_array_equal(i.cpu().numpy(), c["idx"], err_msg=name)
        np.testing.assert_allclose(d.cpu().numpy(), c["dist"], rtol=3e-6, atol=2e-6, err_msg=name)


@pytest.mark.parametrize("n", [1, 31, 33, 1000, 1025, 5000])
@pytest.mark.parametrize("k", [1, 3, 5, 16, 32, 33, 128, 256])
def test_xyz_matches_oracle(cuda_device, n, k):
    if k > n:
        pytest.skip("k > n")
    ref = cloud(2, n, seed=n)
    check(ref[:, :70] + 0.01, ref, k, cuda_device)


@pytest.mark.parametrize("m", [1, 7, 9, 100, 257, 3000])
def test_query_counts(cuda_device, m):
    check(cloud(2, m, seed=1), cloud(2, 2000), 16, cuda_device)


@pytest.mark.parametrize("d", [1, 2, 4, 5, 64, 128])
@pytest.mark.parametrize("k", [1, 5, 20, 33])
def test_feature_matches_oracle(cuda_device, d, k):
    q = cloud(2, 40, seed=d, d=d)
    r = cloud(2, 700, seed=d + 1, d=d)
    r[:, 20] = r[:, 3]
    q[:, 0] = r[:, 3]
    check(q, r, k, cuda_device)


def test_dgcnn_shape_slice(cuda_device):
    """BASELINE config 4 distribution (unit-norm D=64 features), k=20, self included."""
    g = torch.Generator().manual_seed(5)
    f = torch.nn.functional.normalize(torch.randn(2, 1024, 64, generator=g), dim=-1)
    check(f, f, 20, cuda_device)
    d, i = mps_pointops.knn(f.to(cuda_device), f.to(cuda_device), 20)
    assert torch.equal(i[..., 0].cpu(), torch.arange(1024).expand(2, -1))


def test_sqdist_output_is_exact(cuda_device):
    q, r = cloud(1, 300, seed=2), cloud(1, 5000, seed=3)
    dist = torch.empty(1, 300, 24, device=cuda_device)
    idx = torch.empty(1, 300, 24, dtype=torch.long, device=cuda_device)
    sd = torch.empty(1, 300, 24, device=cuda_device)
    qc, rc = q.to(cuda_device), r.to(cuda_device)
    N.check(N.lib().mpo_knn(N.ptr(qc), N.ptr(rc), 1, 300, 5000, 3, 24, N.ptr(dist), N.ptr(idx),
                            N.ptr(sd), None, 0, N.stream(cuda_device)), "knn")
    want = O.knn_sqdist(q.numpy(), r.numpy(), idx.cpu().numpy())
    np.testing.assert_array_equal(sd.cpu().numpy(), want)


@pytest.mark.parametrize("descending", [False, True])
def test_sorted_reference(cuda_device, descending):
    ref = cloud(1, 20000)
    ref = ref[:, ref[0, :, 0].argsort(descending=descending)]
    check(cloud(1, 64, seed=1), ref, 128, cuda_device)
    check(cloud(1, 64, seed=1), ref, 16, cuda_device)


def test_ties_break_by_smaller_index(cuda_device):
    ref = torch.zeros(1, 300, 3)
    ref[0, ::3] = 1.0
    for k in (7, 32, 150, 256):
        check(torch.zeros(1, 2, 3), ref, k, cuda_device)


def test_nonfinite_candidates(cuda_device):
    x = torch.zeros((1, 3, 64))
    x[0, 0, 0], x[0, 1, 0], x[0, 2, 0] = 1.0, 1e30, 2.0
    y = torch.zeros((1, 2, 64))
    y[0, 1, 0] = float("nan")
    dist, idx = mps_pointops.knn(y.to(cuda_device), x.to(cuda_device), 3)
    assert idx.cpu().tolist() == [[[0, 2, -1], [-1, -1, -1]]]  # tests/test_feature_knn.py:130-133
    assert dist[0, 0, :2].cpu().tolist() == [1.0, 2.0]
    assert torch.isinf(dist[:, :, 2]).all().item()
    ref = cloud(1, 50, seed=9)
    ref[0, 4, 2] = float("nan")
    ref[0, 9, 0] = float("inf")
    check(cloud(1, 5, seed=8), ref, 50, cuda_device)


def test_empty_and_errors(cuda_device):
    ref = torch.randn(2, 50, 3, device=cuda_device)
    d, i = mps_pointops.knn(ref[:, :0], ref, 5)
    assert d.shape == i.shape == (2, 0, 5)
    d, i = mps_pointops.knn(ref, ref, 0)
    assert d.shape == i.shape == (2, 50, 0)
    big = torch.randn(1, 300, 3, device=cuda_device)
    with pytest.raises(ValueError, match="at most 256"):
        mps_pointops.knn(big, big, 257)
    with pytest.raises(TypeError):
        mps_pointops.knn(big.half(), big.half(), 4)
    with pytest.raises(ValueError):
        mps_pointops.knn(big, big.cpu(), 4)


@pytest.mark.parametrize("transpose_mode", [True, False])
def test_knn_cuda_module_layouts(cuda_device, transpose_mode):  # tests/test_compat.py:148-160
    ref = cloud(2, 3000).to(cuda_device)
    query = cloud(2, 100, seed=1).to(cuda_device)
    want_d, want_i = mps_pointops.knn(query, ref, 16)
    module = compat.KNN(16, transpose_mode=transpose_mode)
    if transpose_mode:
        d, i = module(ref, query)
    else:
        d, i = module(ref.transpose(1, 2), query.transpose(1, 2))
        d, i = d.transpose(1, 2), i.transpose(1, 2)
    assert torch.equal(i, want_i) and torch.equal(d, want_d)


@pytest.mark.parametrize("k", [1, 16, 32])
def test_large_reference_thread_path(cuda_device, k):
    """Reference clouds above 2^18 points take the thread-per-query kernel."""
    ref = cloud(1, 300_000, seed=21)
    check(cloud(1, 40, seed=22), ref, k, cuda_device)


def test_three_nn_large_known_cloud(cuda_device):
    from mps_pointops.pointnet2 import three_nn
    known = cloud(1, 300_000, seed=23)
    unknown = cloud(1, 50, seed=24)
    want_d, want_i = O.three_nn(unknown.numpy(), known.numpy())
    d, i = three_nn(unknown.to(cuda_device), known.to(cuda_device))
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)


# ---- k <= 3: knn3t_kernel (thread per query, branchless sorted triple) -----------------
@pytest.mark.parametrize("k", [1, 2, 3])
@pytest.mark.parametrize("n", [3, 7, 8, 9, 127, 1023, 1024, 1025, 4097, 70000])
def test_k_at_most_3_matches_oracle(cuda_device, n, k):
    """Every split count and tile edge of knn3t_kernel, uniform and lattice
    (exact ties) clouds, against the exact (SD, index) oracle."""
    g = torch.Generator().manual_seed(n * 7 + k)
    for ref in (torch.randn(2, n, 3, generator=g),
                torch.randint(0, 4, (2, n, 3), generator=g).float()):
        query = torch.randn(2, 1500 if n < 10000 else 300, 3, generator=g)
        check(query, ref, k, cuda_device)


def test_k_at_most_3_nonfinite(cuda_device):
    """NaN references are dropped and +inf ones ranked (D = 3 kNN), also when
    they come first in a split and when fewer finite points than k exist."""
    g = torch.Generator().manual_seed(5)
    ref = torch.randn(1, 3000, 3, generator=g)
    ref[0, :5, 0] = float("nan")
    ref[0, 5:9, 1] = float("inf")
    ref[0, 1500:1510, 2] = float("nan")
    q = torch.randn(1, 400, 3, generator=g)
    for k in (1, 2, 3):
        check(q, ref, k, cuda_device)
    tiny = torch.tensor([[[float("nan"), 0, 0], [float("inf"), 0, 0], [1.0, 2, 3],
                          [float("inf"), 1, 1]]])
    for k in (1, 2, 3):
        check(torch.zeros(1, 3, 3), tiny, k, cuda_device)


def test_three_nn_thread_kernel_matches_oracle(cuda_device):
    """three_nn on every split count (NaN ranked last), config 1 shapes."""
    from mps_pointops import three_nn
    g = torch.Generator().manual_seed(11)
    for b, n, m in ((8, 4096, 1024), (2, 5000, 3), (1, 300, 70000), (3, 1, 2049)):
        unknown = torch.rand(b, n, 3, generator=g)
        known = torch.rand(b, m, 3, generator=g)
        if m > 10:
            known[0, 7, 1] = float("nan")
            known[-1, m // 2] = float("inf")
        wd, wi = O.three_nn(unknown.numpy(), known.numpy())
        d, i = three_nn(unknown.to(cuda_device), known.to(cuda_device))
        np.testing.assert_array_equal(i.cpu().numpy(), wi)
        np.testing.assert_array_equal(d.cpu().numpy(), wd)
