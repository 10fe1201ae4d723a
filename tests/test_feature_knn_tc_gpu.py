"""Feature-space kNN through the tensor-core candidate path (tcgen05 tf32
scores, exact fp32 re-rank) vs the exact (SD, index) oracle of
tests/test_feature_knn.py:16-35 of gamzerA/mps-pointops.  The path serves
16 <= D <= 96, k <= 32, N >= 2048; results must be bit-exact like the
exact kernels': indices, squared distances and IEEE sqrt distances."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import mps_pointops
from mps_pointops import _native as N
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def feats(b, n, d, seed, normalize=False, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    f = torch.randn(b, n, d, generator=g) * scale
    return torch.nn.functional.normalize(f, dim=-1) if normalize else f


def check(query, ref, k, device):
    assert N.lib().mpo_knn_workspace_bytes(query.shape[0], query.shape[1], ref.shape[1],
                                           query.shape[2], k) > 0, "tensor path not selected"
    want_d, want_i = O.knn(query.numpy(), ref.numpy(), k)
    d, i = mps_pointops.knn(query.to(device), ref.to(device), k)
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)


def test_dgcnn_config4_slice(cuda_device):
    """BASELINE config 4 distribution: unit-norm D=64, k=20, self included."""
    f = feats(2, 4096, 64, seed=5, normalize=True)
    check(f, f, 20, cuda_device)
    _, i = mps_pointops.knn(f.to(cuda_device), f.to(cuda_device), 20)
    assert torch.equal(i[..., 0].cpu(), torch.arange(4096).expand(2, -1))


@pytest.mark.parametrize("d", [16, 20, 33, 64, 72, 96])
@pytest.mark.parametrize("k", [1, 8, 20, 32])
def test_dims_and_k(cuda_device, d, k):
    # M not a multiple of the 128-query CTA tile, N not a multiple of the
    # 128-reference tile; D not a multiple of 16.
    q = feats(2, 300, d, seed=d)
    r = feats(2, 2500, d, seed=d + 1)
    check(q, r, k, cuda_device)


@pytest.mark.parametrize("m", [1, 129])
def test_one_query_and_one_tile_plus_one(cuda_device, m):
    # A single query (one mostly-padding 128-row tile) and one query past a
    # whole tile, against exactly 2048 references (the smallest tensor-path
    # cloud, 16 full reference tiles).
    q = feats(2, m, 32, seed=70 + m)
    r = feats(2, 2048, 32, seed=71 + m)
    check(q, r, 7, cuda_device)


@pytest.mark.parametrize("d", [24, 64])
def test_more_queries_than_references(cuda_device, d):
    # The pack grid spans the longer operand: here the query tiles (24 of
    # 128 rows) outnumber the reference tiles (17).
    q = feats(3, 3000, d, seed=60 + d)
    r = feats(3, 2100, d, seed=61 + d)
    check(q, r, 20, cuda_device)


@pytest.mark.parametrize("d", [16, 20, 33, 64, 96])
def test_self_knn_one_pack(cuda_device, d):
    """knn(f, f, k) on ONE device tensor: the references' packed tiles and
    norms also serve as the queries' (one pack pass instead of two); N not a
    multiple of 128, D = 33 with scalar row loads."""
    f = feats(2, 2500, d, seed=40 + d)
    fc = f.to(cuda_device)
    want_d, want_i = O.knn(f.numpy(), f.numpy(), 20)
    dd, ii = mps_pointops.knn(fc, fc, 20)
    np.testing.assert_array_equal(ii.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dd.cpu().numpy(), want_d)


def test_scaled_and_offset_features(cuda_device):
    # Large norms relative to the distances: the error bound scales with them.
    q = feats(1, 300, 32, seed=7, scale=1000.0) + 5000.0
    r = feats(1, 3000, 32, seed=8, scale=1000.0) + 5000.0
    check(q, r, 16, cuda_device)


def test_wide_features_use_exact_path(cuda_device):
    q, r = feats(1, 64, 128, seed=16), feats(1, 2100, 128, seed=17)
    assert N.lib().mpo_knn_workspace_bytes(1, 64, 2100, 128, 8) == 0
    want_d, want_i = O.knn(q.numpy(), r.numpy(), 8)
    d, i = mps_pointops.knn(q.to(cuda_device), r.to(cuda_device), 8)
    np.testing.assert_array_equal(i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(d.cpu().numpy(), want_d)


def test_ties_and_duplicates(cuda_device):
    r = feats(1, 2048, 24, seed=9)
    r[0, 1000:1100] = r[0, 10]          # 101 identical references
    r[0, 1500] = r[0, 7]
    q = torch.cat([r[:, :50], feats(1, 50, 24, seed=10)], dim=1)
    check(q, r, 20, cuda_device)


def test_overflowing_candidate_lists(cuda_device):
    # Integer features: many exactly equal distances, far more than the
    # candidate capacity, so rows fall back to the exact scan.
    g = torch.Generator().manual_seed(11)
    r = torch.randint(0, 2, (2, 2304, 16), generator=g).float()
    q = torch.randint(0, 2, (2, 200, 16), generator=g).float()
    check(q, r, 32, cuda_device)


def test_nonfinite_inputs(cuda_device):
    r = feats(2, 2048, 32, seed=12)
    q = feats(2, 64, 32, seed=13)
    r[0, 5, 3] = float("nan")
    r[0, 6, 0] = float("inf")
    q[1, 2, 1] = float("nan")         # this query has no admissible candidate
    r[1, 9, 9] = -float("inf")
    check(q, r, 10, cuda_device)
    _, i = mps_pointops.knn(q.to(cuda_device), r.to(cuda_device), 10)
    assert (i[1, 2] == -1).all()


def test_sqdist_output(cuda_device):
    q, r = feats(1, 257, 64, seed=14), feats(1, 4096, 64, seed=15)
    k = 12
    B, M, D = q.shape
    Nn = r.shape[1]
    dist = torch.empty(B, M, k, device=cuda_device)
    idx = torch.empty(B, M, k, dtype=torch.long, device=cuda_device)
    sd = torch.empty(B, M, k, device=cuda_device)
    qc, rc = q.to(cuda_device), r.to(cuda_device)
    lib = N.lib()
    ws_bytes = int(lib.mpo_knn_workspace_bytes(B, M, Nn, D, k))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    N.check(lib.mpo_knn(N.ptr(qc), N.ptr(rc), B, M, Nn, D, k, N.ptr(dist), N.ptr(idx),
                        N.ptr(sd), N.ptr(ws), ws_bytes, N.stream(cuda_device)), "knn")
    want = O.knn_sqdist(q.numpy(), r.numpy(), idx.cpu().numpy())
    np.testing.assert_array_equal(sd.cpu().numpy(), want)
    # Too small a workspace is an error, not a silent fallback.
    st = lib.mpo_knn(N.ptr(qc), N.ptr(rc), B, M, Nn, D, k, N.ptr(dist), N.ptr(idx), None,
                     N.ptr(ws), ws_bytes - 1, N.stream(cuda_device))
    assert st == 4 and "workspace" in N.last_error()


@pytest.mark.parametrize("d", [32, 64])
def test_unaligned_rows(cuda_device, d):
    # Contiguous views whose base sits 4 bytes past a 16-byte boundary: the
    # kernels must use scalar row loads (vector loads would be misaligned).
    q = feats(2, 300, d, seed=20)
    r = feats(2, 2500, d, seed=21)
    qb = torch.zeros(q.numel() + 1, device=cuda_device)
    rb = torch.zeros(r.numel() + 3, device=cuda_device)
    qv = qb[1:].view(q.shape)
    rv = rb[3:].view(r.shape)
    qv.copy_(q.to(cuda_device))
    rv.copy_(r.to(cuda_device))
    assert qv.is_contiguous() and qv.data_ptr() % 16 == 4 and rv.data_ptr() % 16 == 12
    want_d, want_i = O.knn(q.numpy(), r.numpy(), 20)
    dd, ii = mps_pointops.knn(qv, rv, 20)
    np.testing.assert_array_equal(ii.cpu().numpy(), want_i)
    np.testing.assert_array_equal(dd.cpu().numpy(), want_d)


def test_unaligned_workspace_is_rejected(cuda_device):
    q, r = feats(1, 64, 64, seed=22), feats(1, 2048, 64, seed=23)
    k = 8
    B, M, D = q.shape
    Nn = r.shape[1]
    dist = torch.empty(B, M, k, device=cuda_device)
    idx = torch.empty(B, M, k, dtype=torch.long, device=cuda_device)
    qc, rc = q.to(cuda_device), r.to(cuda_device)
    lib = N.lib()
    ws_bytes = int(lib.mpo_knn_workspace_bytes(B, M, Nn, D, k))
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=cuda_device)
    st = lib.mpo_knn(N.ptr(qc), N.ptr(rc), B, M, Nn, D, k, N.ptr(dist), N.ptr(idx), None,
                     ctypes.c_void_p(ws.data_ptr() + 16), ws_bytes, N.stream(cuda_device))
    assert st == 1 and "256-byte aligned" in N.last_error()
