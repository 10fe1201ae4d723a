"""Flat (torch_cluster-style) API on the B200 kernels vs the CPU oracle and
the reference's golden vectors (gamzerA/mps-pointops mps_pointops/flat.py,
tests/test_flat.py, tests/test_flat_graph.py, tests/test_pyg28.py).
Indices are compared bit-exactly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import _native as N
from mps_pointops import compat, flat, pyg
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def ptr_of(lengths):
    p = [0]
    for n in lengths:
        p.append(p[-1] + n)
    return p


def ragged(lengths, d, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(sum(lengths), d, generator=g) * scale


def knn_case(x, y, lx, ly, k, dev):
    px, py = ptr_of(lx), ptr_of(ly)
    want = O.flat_knn_indices(x.numpy(), y.numpy(), px, py, k)
    got = flat.knn_indices(x.to(dev), y.to(dev), torch.tensor(px, device=dev),
                           torch.tensor(py, device=dev), k)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def radius_case(x, y, lx, ly, r, m, dev, ignore_same=False):
    px, py = ptr_of(lx), ptr_of(ly)
    want = O.flat_radius_indices(x.float().numpy(), y.float().numpy(), px, py, r, m, ignore_same)
    got = flat.radius_indices(x.to(dev), y.to(dev), torch.tensor(px, device=dev),
                              torch.tensor(py, device=dev), r, m, ignore_same_index=ignore_same)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


# ------------------------------------------------------------------ golden vectors
def test_golden_flat_search(cuda_device):
    n = 0
    for name, c in golden("flat").items():
        if "ptr_x" not in c:
            continue
        width, radius = int(c["meta"][0]), float(c["meta"][1])
        x, y = torch.from_numpy(c["x"]).to(cuda_device), torch.from_numpy(c["y"]).to(cuda_device)
        px = torch.from_numpy(c["ptr_x"]).to(cuda_device)
        py = torch.from_numpy(c["ptr_y"]).to(cuda_device)
        if radius < 0:
            got = flat.knn_indices(x, y, px, py, width)
        else:
            got = flat.radius_indices(x, y, px, py, radius, width)
        np.testing.assert_array_equal(got.cpu().numpy(), c["idx"], err_msg=name)
        n += 1
    assert n >= 16


def test_golden_edges_public_calls(cuda_device):
    c = golden("flat")["edges"]
    x, bx = torch.from_numpy(c["x"]).to(cuda_device), torch.from_numpy(c["batch_x"]).to(cuda_device)
    y, by = torch.from_numpy(c["y"]).to(cuda_device), torch.from_numpy(c["batch_y"]).to(cuda_device)
    eq = np.testing.assert_array_equal
    eq(flat.knn(x, y, 4, bx, by).cpu().numpy(), c["knn"])
    eq(flat.radius(x, y, 0.8, bx, by, max_num_neighbors=6).cpu().numpy(), c["radius"])
    eq(flat.knn_graph(x, 3, bx).cpu().numpy(), c["knn_graph"])
    eq(flat.knn_graph(x, 3, bx, loop=True, flow="target_to_source").cpu().numpy(),
       c["knn_graph_loop_t2s"])
    eq(flat.radius_graph(x, 0.9, bx, max_num_neighbors=5).cpu().numpy(), c["radius_graph"])
    eq(flat.radius_graph(x, 0.9, bx, loop=True, max_num_neighbors=5).cpu().numpy(),
       c["radius_graph_loop"])


def test_golden_fps(cuda_device):
    c = golden("flat")["fps_over"]
    x = torch.from_numpy(c["x"]).to(cuda_device)
    got = flat.fps(x, ptr=[0, 4, 10], ratio=1.7, random_start=False)
    np.testing.assert_array_equal(got.cpu().numpy(), c["idx"])
    c = golden("flat")["fps_dup"]
    got = flat.fps(torch.from_numpy(c["x"]).to(cuda_device), ratio=1.0, random_start=False)
    np.testing.assert_array_equal(got.cpu().numpy(), c["idx"])


# ------------------------------------------------------------------ reference tests
def bipartite(dev):
    """tests/test_flat.py:10-17."""
    x = torch.tensor([[0., 0, 0], [2., 0, 0], [5., 0, 0], [10., 0, 0], [12., 0, 0]], device=dev)
    y = torch.tensor([[1., 0, 0], [0., 0, 0], [11., 0, 0], [15., 0, 0]], device=dev)
    bx = torch.tensor([0, 0, 0, 2, 2], dtype=torch.long, device=dev)
    by = torch.tensor([0, 1, 2, 2], dtype=torch.long, device=dev)
    return x, y, bx, by


def test_reference_known_answers(cuda_device):
    x, y, bx, by = bipartite(cuda_device)
    # tests/test_flat.py:20-24
    assert flat.fps(x, bx, ratio=0.5, random_start=False).tolist() == [0, 2, 3]
    assert flat.fps(x, ptr=[0, 3, 3, 5], ratio=0.5, random_start=False).tolist() == [0, 2, 3]
    assert flat.fps(x, bx, ratio=0, random_start=False).shape == (0,)
    assert flat.fps(x, ratio=1.1, random_start=False).shape == (6,)
    # :49-54
    edge = flat.knn(x, y, 2, bx, by)
    assert edge.dtype == torch.long and edge.device == x.device
    assert edge.tolist() == [[0, 0, 2, 2, 3, 3], [0, 1, 3, 4, 4, 3]]
    assert flat.knn(x, y, 5, bx, by).shape == (2, 7)
    # :69-77
    assert flat.radius(x, y, 1.1, bx, by, max_num_neighbors=2).tolist() == [
        [0, 0, 2, 2], [0, 1, 3, 4]]
    assert flat.radius(x[:2], x[:1], 1.0).tolist() == [[0], [0]]
    assert flat.radius(x, y, 100.0, bx, by, max_num_neighbors=1).tolist() == [
        [0, 2, 3], [0, 3, 3]]
    # :27-33
    x3 = torch.tensor([[0., 0, 0], [1., 0, 0], [4., 0, 0]], device=cuda_device)
    assert flat.fps(x3, random_start=False).tolist() == [0, 2]
    torch.manual_seed(42)
    sample = flat.fps(x3, ratio=1 / 3, random_start=True)
    assert sample.dtype == torch.long and sample.shape == (1,) and 0 <= sample.item() < 3


def test_knn_excludes_nonfinite_coordinates(cuda_device):  # tests/test_flat.py:58-66
    x = torch.tensor([[0.0, 0.0, 0.0], [float("nan"), 0.0, 0.0], [float("inf"), 0.0, 0.0]],
                     device=cuda_device)
    y = torch.tensor([[0.0, 0.0, 0.0], [float("nan"), 0.0, 0.0]], device=cuda_device)
    assert flat.knn(x, y, 3).cpu().tolist() == [[0], [0]]


@pytest.mark.parametrize("dimensions", [3, 64])
def test_large_effective_k_is_explicit_error(cuda_device, dimensions):  # :128-142
    x = torch.arange(300, dtype=torch.float32)[:, None].expand(-1, dimensions).contiguous()
    x = x.to(cuda_device)
    y = x[:1]
    with pytest.raises(ValueError, match="effective k must be at most 256 on CUDA"):
        flat.knn(x, y, 257)
    with pytest.raises(ValueError, match="effective k must be at most 256 on CUDA"):
        flat.knn_graph(x, 256, loop=False)
    with pytest.raises(ValueError, match="effective k must be at most 256 on CUDA"):
        pyg._knn_cuda(x, y, k=257)
    assert flat.knn(x[:256], y, 300).shape == (2, 256)
    assert pyg._knn_cuda(x[:256], y, k=300).shape == (2, 256)


@pytest.mark.parametrize("n, ratio, expected", [
    (25, 0.6, 16), (45, 0.6, 28), (50, 0.3, 16), (90, 0.3, 28), (10, 0.5, 5), (7, 0.5, 4),
    (9, 1.0, 9)])
def test_fps_sample_counts(cuda_device, n, ratio, expected):  # :172-174
    x = torch.rand(n, 3, device=cuda_device)
    assert len(flat.fps(x, ratio=ratio, random_start=False)) == expected


def test_fps_float64_tensor_ratio_uses_gpu_rule(cuda_device):  # :188-199
    x = torch.rand(25, 3, device=cuda_device)
    assert len(flat.fps(x, ratio=torch.tensor(0.6, dtype=torch.float64),
                        random_start=False)) == 15
    assert len(flat.fps(x, ratio=torch.tensor([0.6], dtype=torch.float64),
                        random_start=False)) == 15


def test_radius_threshold_is_double_product_rounded_to_float32(cuda_device):  # :207-224
    r = 0.21
    r32 = torch.tensor(r, dtype=torch.float32)
    x = torch.tensor([[float(r32), 0.0, 0.0]], device=cuda_device)
    y = torch.zeros(1, 3, device=cuda_device)
    assert flat.radius(x, y, r).tolist() == [[0], [0]]
    r = 0.1
    r32 = torch.tensor(r, dtype=torch.float32)
    x = torch.tensor([[float(r32), 0.0, 0.0]], device=cuda_device)
    assert flat.radius(x, y, r).shape == (2, 0)


def test_cuda_dtype_rules(cuda_device):
    x = torch.rand(10, 3, device=cuda_device, dtype=torch.float64)
    with pytest.raises(TypeError, match="float32 on CUDA"):
        flat.fps(x)
    with pytest.raises(TypeError, match="float32 for kNN on CUDA"):
        flat.knn(x, x, 2)
    with pytest.raises(TypeError, match="float16 or float32 for radius on CUDA"):
        flat.radius(x, x, 0.5)


# ------------------------------------------------------------------ pyg surface
def test_pyg_surface_known_answers(cuda_device):  # tests/test_pyg28.py:27-106
    x = torch.tensor([[0.0, 0, 0], [1.0, 0, 0], [10.0, 0, 0], [11.0, 0, 0]], device=cuda_device)
    y = torch.tensor([[0.1, 0, 0], [10.1, 0, 0]], device=cuda_device)
    ptr_x = torch.tensor([0, 2, 4], device=cuda_device)
    ptr_y = torch.tensor([0, 1, 2], device=cuda_device)
    expected = [[0, 0, 1, 1], [0, 1, 2, 3]]
    assert pyg._fps_cuda(x, ptr_x, 0.5, False).tolist() == [0, 2]
    assert pyg._knn_cuda(x, y, ptr_x, ptr_y, 2).tolist() == expected
    assert pyg._radius_cuda(x, y, ptr_x, ptr_y, 1.0).tolist() == expected
    xs = torch.tensor([[0.0, 0, 0], [0.1, 0, 0], [0.2, 0, 0]], device=cuda_device)
    assert pyg._radius_cuda(xs, xs[:1], None, None, 1.0, 1, 1, True).tolist() == [[0], [1]]
    x2 = torch.tensor([[0.0, 0, 0], [2.0, 0, 0]], device=cuda_device)
    y2 = torch.tensor([[0.1, 0, 0]], device=cuda_device)
    assert pyg._knn_cuda(x2, y2).tolist() == [[0], [0]]
    assert pyg._radius_cuda(x2, y2).tolist() == [[0], [0]]
    xf = torch.zeros((4, 64), device=cuda_device)
    xf[:, 0] = torch.tensor([0.0, 1.0, 10.0, 11.0], device=cuda_device)
    yf = xf[[0, 2]] + 0.1
    assert pyg._knn_cuda(xf, yf, ptr_x, ptr_y, 2).tolist() == expected
    xq = torch.tensor([[0.0, 0, 0], [10.0, 0, 0]], device=cuda_device)
    py2 = torch.tensor([0, 1, 2], dtype=torch.long, device=cuda_device)
    assert pyg._knn_cuda(xq, xq.clone(), None, py2, 1).tolist() == [[0, 1], [0, 1]]
    assert pyg._radius_cuda(xq, xq.clone(), None, py2, 1.0, 2).tolist() == [[0, 1], [0, 1]]


def test_torch_cluster_shim(cuda_device):
    import sys
    saved = sys.modules.pop("torch_cluster", None)
    try:
        compat.install(force=True)
        import torch_cluster
        x, y, bx, by = bipartite(cuda_device)
        assert torch_cluster.knn(x, y, 2, bx, by).tolist() == [
            [0, 0, 2, 2, 3, 3], [0, 1, 3, 4, 4, 3]]
    finally:
        sys.modules.pop("torch_cluster", None)
        if saved is not None:
            sys.modules["torch_cluster"] = saved


# ------------------------------------------------------------------ oracle parity, wider
LX = [0, 1, 7, 33, 100, 257, 0, 64, 2048, 5000, 31]
LY = [5, 3, 0, 40, 17, 90, 2, 64, 700, 1300, 0]


@pytest.mark.parametrize("k", [1, 3, 8, 16, 20, 32, 33, 64, 256])
def test_knn3_ragged(cuda_device, k):
    knn_case(ragged(LX, 3, 1), ragged(LY, 3, 2), LX, LY, k, cuda_device)


@pytest.mark.parametrize("d,k", [(1, 4), (2, 8), (5, 16), (16, 20), (64, 20), (100, 32),
                                 (24, 40), (64, 128)])
def test_knn_features_ragged(cuda_device, d, k):
    knn_case(ragged(LX, d, 3 + d), ragged(LY, d, 4 + d), LX, LY, k, cuda_device)


def test_knn3_large_segment(cuda_device):
    # A segment above 2**18 references takes the packed thread-per-query kernel.
    lx, ly = [300_000, 3000, 0], [1500, 400, 7]
    x, y = ragged(lx, 3, 5), ragged(ly, 3, 6)
    for k in (1, 16, 32):
        knn_case(x, y, lx, ly, k, cuda_device)


def test_knn_ties_and_nonfinite(cuda_device):
    g = torch.Generator().manual_seed(7)
    x = torch.randint(0, 3, (sum(LX), 3), generator=g).float()
    y = torch.randint(0, 3, (sum(LY), 3), generator=g).float()
    x[10, 0] = float("nan")
    x[20, 1] = float("inf")
    x[3000, 2] = -float("inf")
    y[4, 0] = float("nan")
    y[900, 1] = float("inf")
    for k in (5, 32, 50):
        knn_case(x, y, LX, LY, k, cuda_device)
    xf = torch.randint(0, 2, (sum(LX), 16), generator=g).float()
    yf = torch.randint(0, 2, (sum(LY), 16), generator=g).float()
    xf[7, 3] = float("nan")
    knn_case(xf, yf, LX, LY, 20, cuda_device)


@pytest.mark.parametrize("r,m", [(0.3, 8), (0.8, 32), (2.0, 64), (10.0, 300), (1e-30, 4)])
def test_radius_ragged(cuda_device, r, m):
    radius_case(ragged(LX, 3, 8), ragged(LY, 3, 9), LX, LY, r, m, cuda_device)


def test_radius_ignore_same_index_and_half(cuda_device):
    x = ragged(LX, 3, 10)
    radius_case(x, x, LX, LX, 0.7, 16, cuda_device, ignore_same=True)
    xh, yh = ragged(LX, 3, 11).half(), ragged(LY, 3, 12).half()
    radius_case(xh, yh, LX, LY, 0.6, 20, cuda_device)


def test_radius_nonfinite_and_zero(cuda_device):
    x, y = ragged(LX, 3, 13), ragged(LY, 3, 14)
    x[10, 0] = float("nan")
    x[3000, 1] = float("inf")
    y[4, 2] = float("nan")
    radius_case(x, y, LX, LY, 1.5, 16, cuda_device)
    radius_case(x, y, LX, LY, 0.0, 16, cuda_device)


@pytest.mark.parametrize("lengths", [[1, 2, 30, 0, 257, 1000, 4], [9000, 0, 100, 20000, 8192],
                                     [1500, 0, 300, 8192, 4097, 2]])
def test_fps_ragged_against_oracle(cuda_device, lengths):
    x = ragged(lengths, 3, 15)
    ptr = ptr_of(lengths)
    for ratio, random_start in ((0.37, False), (0.05, True), (1.3, False)):
        got = flat.fps(x.to(cuda_device), ptr=ptr, ratio=ratio, random_start=random_start)
        counts = O.flat_sample_counts(lengths, ratio)
        outp = ptr_of(counts)
        got = got.cpu().numpy()
        assert len(got) == outp[-1]
        # The start of each cloud is its first sample; the oracle continues from it.
        starts = [int(got[outp[b]]) - ptr[b] if counts[b] else 0 for b in range(len(lengths))]
        if not random_start:
            assert all(s == 0 for s in starts)
        want = O.flat_fps(x.numpy(), ptr, counts, starts)
        np.testing.assert_array_equal(got, want)


def test_invalid_offsets_are_reported(cuda_device):
    x = ragged([10, 10], 3, 16).to(cuda_device)
    good = torch.tensor([0, 10, 20], device=cuda_device)
    bad = torch.tensor([0, 12, 20], device=cuda_device)  # x offsets past the y rows
    with pytest.raises(ValueError, match="batch offsets"):
        flat.knn_indices(x, x, torch.tensor([0, 25, 20], device=cuda_device), good, 3)
    with pytest.raises(ValueError, match="batch offsets"):
        flat.radius_indices(x, x, good, torch.tensor([0, 5, 3], device=cuda_device), 0.5, 3)
    # Offsets that are valid but differ between x and y are a legal ragged batch.
    flat.knn_indices(x, x, bad, good, 3)
    # The C ABI's own FPS checks: a start outside its cloud sets status 2.
    out = torch.empty(4, dtype=torch.long, device=cuda_device)
    status = torch.empty(1, dtype=torch.int32, device=cuda_device)
    ptr = torch.tensor([0, 10, 20], device=cuda_device)
    out_ptr = torch.tensor([0, 2, 4], device=cuda_device)
    starts = torch.tensor([0, 10], device=cuda_device)
    N.check(N.lib().mpo_flat_fps(N.ptr(x), N.ptr(ptr), N.ptr(out_ptr), N.ptr(starts), 2, 20, 4,
                                 10, N.ptr(out), N.ptr(status), None, 0,
                                 N.stream(cuda_device)), "flat fps")
    assert int(status.item()) == 2
