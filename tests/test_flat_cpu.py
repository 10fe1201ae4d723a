"""Flat (torch_cluster-style) API on the host: the oracle pinned to the
reference's golden vectors and known answers, and the host-side behaviour of
mps_pointops.flat / mps_pointops.pyg that needs no GPU -- validation order,
exception types and messages (gamzerA/mps-pointops tests/test_flat.py,
tests/test_flat_graph.py, tests/test_pyg28.py), early empty results, the
sample-count rules, and the loud refusal of CPU tensors."""

from __future__ import annotations

import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from conftest import PKG_ROOT, ROOT, golden
from mps_pointops import flat, pyg
from oracle import oracle as O


# ------------------------------------------------------------------ oracle pins
def test_oracle_matches_reference_flat_search():
    """tests/golden/flat.npz: mps_pointops/flat.py:264-288 on ragged batches
    with empty clouds, non-finite coordinates, exact ties and D in {1..64}."""
    cases = golden("flat")
    n = 0
    for name, c in cases.items():
        if "ptr_x" not in c:
            continue
        width, radius = int(c["meta"][0]), float(c["meta"][1])
        if radius < 0:
            got = O.flat_knn_indices(c["x"], c["y"], c["ptr_x"], c["ptr_y"], width)
        else:
            got = O.flat_radius_indices(c["x"], c["y"], c["ptr_x"], c["ptr_y"], radius, width)
        np.testing.assert_array_equal(got, c["idx"], err_msg=name)
        n += 1
    assert n >= 16


def test_oracle_matches_reference_flat_fps():
    c = golden("flat")["fps_starts"]
    got = O.flat_fps(c["x"], c["ptr"], c["counts"], c["starts"])
    np.testing.assert_array_equal(got, c["idx"])
    c = golden("flat")["fps_over"]          # ratio 1.7: requests beyond the cloud repeat 0
    counts = O.flat_sample_counts([4, 6], 1.7)
    np.testing.assert_array_equal(O.flat_fps(c["x"], [0, 4, 10], counts, [0, 0]), c["idx"])
    c = golden("flat")["fps_dup"]
    np.testing.assert_array_equal(O.flat_fps(c["x"], [0, 6], [6], [0]), c["idx"])


def test_oracle_sample_counts_match_reference_gpu_rule():
    cases = golden("flat")
    lengths = list(range(300))
    for ratio in (0.05, 0.3, 1 / 3, 0.6, 0.95):
        c = cases[f"counts_{ratio:.4f}"]
        assert O.flat_sample_counts(lengths, ratio) == c["gpu"].tolist()
        # torch_cluster's CPU rule converts sizes to float32 as well for a
        # float32 ratio, so the two agree here.
        assert c["cpu"].tolist() == c["gpu"].tolist()


def test_oracle_edges_match_reference_public_calls():
    c = golden("flat")["edges"]
    bx, by = c["batch_x"], c["batch_y"]
    px = np.searchsorted(bx, np.arange(5)).astype(np.int64)
    py = np.searchsorted(by, np.arange(5)).astype(np.int64)
    np.testing.assert_array_equal(
        O.flat_edges(O.flat_knn_indices(c["x"], c["y"], px, py, 4)), c["knn"])
    np.testing.assert_array_equal(
        O.flat_edges(O.flat_radius_indices(c["x"], c["y"], px, py, 0.8, 6)), c["radius"])


def bipartite():
    """tests/test_flat.py:10-17."""
    x = np.array([[0., 0, 0], [2, 0, 0], [5, 0, 0], [10, 0, 0], [12, 0, 0]], np.float32)
    y = np.array([[1., 0, 0], [0, 0, 0], [11, 0, 0], [15, 0, 0]], np.float32)
    return x, y, [0, 3, 3, 5], [0, 1, 2, 4]


def test_oracle_known_answers_from_reference_tests():
    x, y, px, py = bipartite()
    # tests/test_flat.py:49-54, 69-77, 20-24
    assert O.flat_edges(O.flat_knn_indices(x, y, px, py, 2)).tolist() == [
        [0, 0, 2, 2, 3, 3], [0, 1, 3, 4, 4, 3]]
    assert O.flat_edges(O.flat_knn_indices(x, y, px, py, 5)).shape == (2, 7)
    assert O.flat_edges(O.flat_radius_indices(x, y, px, py, 1.1, 2)).tolist() == [
        [0, 0, 2, 2], [0, 1, 3, 4]]
    assert O.flat_edges(O.flat_radius_indices(x[:2], x[:1], [0, 2], [0, 1], 1.0, 2)).tolist() \
        == [[0], [0]]
    assert O.flat_edges(O.flat_radius_indices(x, y, px, py, 100.0, 1)).tolist() == [
        [0, 2, 3], [0, 3, 3]]
    assert O.flat_fps(x, px, O.flat_sample_counts([3, 0, 2], 0.5), [0, 0, 0]).tolist() == [0, 2, 3]
    # tests/test_flat.py:58-66: non-finite coordinates never match.
    xn = np.array([[0., 0, 0], [np.nan, 0, 0], [np.inf, 0, 0]], np.float32)
    yn = np.array([[0., 0, 0], [np.nan, 0, 0]], np.float32)
    assert O.flat_edges(O.flat_knn_indices(xn, yn, [0, 3], [0, 2], 3)).tolist() == [[0], [0]]
    # tests/test_pyg28.py:53-58: ignore_same_index drops x row 0 before the cap.
    xs = np.array([[0., 0, 0], [0.1, 0, 0], [0.2, 0, 0]], np.float32)
    assert O.flat_edges(O.flat_radius_indices(xs, xs[:1], [0, 3], [0, 1], 1.0, 1,
                                              ignore_same_index=True)).tolist() == [[0], [1]]


def test_radius_threshold_known_answers():
    # tests/test_flat.py:208-224: fl32(r * r) in double vs fl32(r)^2.
    r32 = float(np.float32(0.21))
    x = np.array([[r32, 0, 0]], np.float32)
    y = np.zeros((1, 3), np.float32)
    assert O.flat_radius_indices(x, y, [0, 1], [0, 1], 0.21, 1).tolist() == [[0]]
    r32 = float(np.float32(0.1))
    x = np.array([[r32, 0, 0]], np.float32)
    assert O.flat_radius_indices(x, y, [0, 1], [0, 1], 0.1, 1).tolist() == [[-1]]
    assert flat._radius_sq(0.21) == O.torch_cluster_radius_sq(0.21)
    assert flat._radius_sq(1e30) == float("inf")


# ------------------------------------------------------------------ host API
def tbipartite():
    x, y, _, _ = bipartite()
    return (torch.from_numpy(x), torch.from_numpy(y), torch.tensor([0, 0, 0, 2, 2]),
            torch.tensor([0, 1, 2, 2]))


def test_cpu_tensors_fail_loudly():
    x, y, bx, by = tbipartite()
    for call in (lambda: flat.fps(x, bx, ratio=0.5, random_start=False),
                 lambda: flat.knn(x, y, 2, bx, by),
                 lambda: flat.radius(x, y, 1.1, bx, by),
                 lambda: flat.knn_graph(x, 2, bx),
                 lambda: flat.radius_graph(x, 1.5, bx)):
        with pytest.raises(RuntimeError, match="CUDA tensors only"):
            call()


def test_empty_results_need_no_device():  # tests/test_flat.py:20-46, 81-92
    x, y, bx, _ = tbipartite()
    assert flat.fps(x, bx, ratio=0, random_start=False).shape == (0,)
    assert flat.fps(torch.empty(0, 3)).shape == (0,)
    for method in ("knn", "radius"):
        xe, ye = torch.empty(0, 3), torch.zeros(2, 3)
        r = flat.knn(xe, ye, 4) if method == "knn" else flat.radius(xe, ye, 1)
        assert r.shape == (2, 0) and r.dtype == torch.long
        by = torch.tensor([0, 1])
        r = (flat.knn(xe, ye, 4, batch_y=by) if method == "knn"
             else flat.radius(xe, ye, 1, batch_y=by))
        assert r.shape == (2, 0)
    assert flat.knn(x, y, 0).shape == (2, 0)
    assert flat.radius(x, y, 1.0, max_num_neighbors=0).shape == (2, 0)


def test_fps_validation():  # tests/test_flat.py:36-46
    x, _, _, _ = tbipartite()
    with pytest.raises(ValueError, match="sorted"):
        flat.fps(x, torch.tensor([0, 1, 0, 2, 2]))
    with pytest.raises(ValueError, match="ptr"):
        flat.fps(x, ptr=[0, 4, 3, 5])
    with pytest.raises(ValueError, match="ptr must start at 0"):
        flat.fps(x, ptr=[0, 4])
    with pytest.raises(ValueError, match="ratio"):
        flat.fps(x, ratio=-0.1)
    with pytest.raises(ValueError, match="ratio tensor"):
        flat.fps(x, ratio=torch.tensor([0.5, 0.5]))
    with pytest.raises(TypeError, match="ratio must be a number"):
        flat.fps(x, ratio="half")
    with pytest.raises(ValueError, match="batch_size is smaller"):
        flat.fps(x, torch.tensor([0, 0, 0, 2, 2]), batch_size=1)
    with pytest.raises(ValueError, match=r"shape \(N, 3\)"):
        flat.fps(torch.zeros(4, 2))
    with pytest.raises(TypeError, match="floating-point"):
        flat.fps(torch.zeros(4, 3, dtype=torch.long))


def test_search_validation():  # tests/test_flat.py:95-104
    x, y, bx, by = tbipartite()
    with pytest.raises(NotImplementedError, match="cosine"):
        flat.knn(x, y, 2, cosine=True)
    with pytest.raises(NotImplementedError, match="ignore_same_index"):
        flat.radius(x, y, 1, ignore_same_index=True)
    with pytest.raises(ValueError, match="both required"):
        flat.knn(x, y, 1, batch_x=bx)
    with pytest.raises(ValueError, match="sorted"):
        flat.radius(x, y, 1, batch_x=bx, batch_y=by.flip(0))
    with pytest.raises(ValueError, match="feature dimensions differ"):
        flat.knn(x, torch.zeros(3, 4), 1)
    with pytest.raises(TypeError, match="same dtype"):
        flat.knn(x, y.double(), 1)
    with pytest.raises(ValueError, match="k must be a non-negative integer"):
        flat.knn(x, y, -1)
    with pytest.raises(ValueError, match="r must be a finite non-negative number"):
        flat.radius(x, y, float("nan"))
    with pytest.raises(ValueError, match="max_num_neighbors"):
        flat.radius(x, y, 1.0, max_num_neighbors=True)
    with pytest.raises(ValueError, match="flow must be"):
        flat.knn_graph(x, 2, flow="up")
    with pytest.raises(ValueError, match=r"batch_x must have shape \(5,\)"):
        flat.knn(x, y, 1, bx[:4], by)
    with pytest.raises(TypeError, match="integer dtype"):
        flat.knn(x, y, 1, bx.float(), by)


def test_sample_count_rules():
    # tests/test_flat.py:172-199: torch_cluster's float32 product rounds up.
    for n, ratio, want in ((25, 0.6, 16), (45, 0.6, 28), (50, 0.3, 16), (90, 0.3, 28),
                           (10, 0.5, 5), (7, 0.5, 4), (9, 1.0, 9)):
        r = flat._ratio(ratio, torch.float32)
        assert flat._sample_counts([n], r, gpu=True) == [want]
        assert flat._sample_counts([n], r, gpu=False) == [want]
    # A float64 0-D ratio: CPU keeps float32 sizes, the GPU rule uses float64.
    scalar = flat._ratio(torch.tensor(0.6, dtype=torch.float64), torch.float32)
    vector = flat._ratio(torch.tensor([0.6], dtype=torch.float64), torch.float32)
    assert flat._sample_counts([25], scalar, gpu=False) == [16]
    assert flat._sample_counts([25], scalar, gpu=True) == [15]
    assert flat._sample_counts([25], vector, gpu=True) == [15]
    assert flat._sample_counts([25], vector, gpu=False) == [15]


def test_pyg_surface_validation():
    x, y, _, _ = tbipartite()
    with pytest.raises(ValueError, match="ptr_y is required"):
        pyg._knn_cuda(x, y, torch.tensor([0, 5]), None, 1)
    with pytest.raises(ValueError, match="same CUDA device"):
        pyg._knn_cuda(x, y, None, None, 1)
    with pytest.raises(ImportError, match="pyg-lib"):
        pyg.register_cuda()


def test_register_cuda_with_pyg_lib_schemas(tmp_path):
    """register_cuda against stand-in pyg-lib schemas (a child process, so the
    operator registrations do not leak into this test session)."""
    script = textwrap.dedent(f"""
        import sys, types
        sys.path[:0] = [{str(ROOT)!r}, {str(PKG_ROOT)!r}]
        import torch
        lib = torch.library.Library("pyg", "DEF")
        lib.define("fps(Tensor src, Tensor ptr, float ratio=0.5, bool random_start=True) -> Tensor")
        lib.define("knn(Tensor x, Tensor y, Tensor? ptr_x=None, Tensor? ptr_y=None, int k=1, "
                   "bool cosine=False, int num_workers=1) -> Tensor")
        lib.define("radius(Tensor x, Tensor y, Tensor? ptr_x=None, Tensor? ptr_y=None, "
                   "float r=1.0, int max_num_neighbors=32, int num_workers=1, "
                   "bool ignore_same_index=False) -> Tensor")
        fake = types.ModuleType("pyg_lib")
        fake.ops = types.SimpleNamespace(fps=1, knn=1, radius=1)
        sys.modules["pyg_lib"] = fake
        from mps_pointops import pyg
        names = pyg.register_cuda()
        assert sorted(names) == ["fps", "knn", "radius"], names
        assert pyg.register_cuda() == []
        for n in names:
            assert torch._C._dispatch_has_kernel_for_dispatch_key("pyg::" + n, "CUDA")
        print("ok")
    """)
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
