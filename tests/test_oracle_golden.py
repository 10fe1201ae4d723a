"""Pin the CPU oracle (oracle/) to the reference's golden vectors.

Every fixture in tests/golden/ was produced by the reference's own code
(tests/golden/make_golden.py).  Indices must match exactly; float outputs are
bit-exact where the reference computes them with the same single-rounded
float32 operations, and within a stated tolerance where it does not (the
Chamfer loss and gradients, whose sums the reference evaluates in a
different order).

Euclidean distances that the reference produced through torch's CPU ``sqrt``
(three_nn) are compared with ``rtol=1e-6``: torch's vectorised CPU square
root is not correctly rounded on every host (about 0.6% of float32 results
are one ulp away from IEEE ``sqrt`` on an AVX-512 machine), while the
squared distances and every index are compared exactly.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import oracle as O


def test_fps_matches_reference_cpu_path():
    for name, c in golden("fps").items():
        npoint, start, skip = (int(v) for v in c["meta"])
        got = O.furthest_point_sample(c["xyz"], npoint, start, bool(skip))
        np.testing.assert_array_equal(got, c["idx"], err_msg=name)


def test_knn_matches_reference_exact_oracles():
    for name, c in golden("knn").items():
        d, i = O.knn(c["query"], c["ref"], int(c["k"]))
        np.testing.assert_array_equal(i, c["idx"], err_msg=name)
        np.testing.assert_array_equal(d, c["dist"], err_msg=name)
    for name, c in golden("feature_knn").items():
        d, i = O.knn(c["query"], c["ref"], int(c["k"]))
        np.testing.assert_array_equal(i, c["idx"], err_msg=name)
        np.testing.assert_array_equal(d, c["dist"], err_msg=name)


def test_ball_query_matches_reference_cpu_path():
    for name, c in golden("ball_query").items():
        d2, i = O.ball_query(c["query"], c["ref"], float(c["radius"]), int(c["K"]))
        np.testing.assert_array_equal(i, c["idx"], err_msg=name)
        np.testing.assert_array_equal(d2.view(np.int32), c["dist2"].view(np.int32), err_msg=name)


def test_compat_padding_known_answer():
    xyz = np.array([[[5.0, 0, 0], [0.1, 0, 0], [9, 9, 9], [0.2, 0, 0]]], np.float32)
    new_xyz = np.array([[[0.0, 0, 0], [50.0, 50, 50]]], np.float32)
    got = O.ball_query_pointnet2(0.5, 4, xyz, new_xyz)
    np.testing.assert_array_equal(got, golden("compat_pad")["idx"])
    assert got.tolist() == [[[1, 3, 1, 1], [0, 0, 0, 0]]]  # tests/test_compat.py:140-145


def test_radius_squared_known_answer():
    # tests/test_ball_query_mps.py:248-261: fl32(fl32(0.1)^2) has bits 0x3c23d70b.
    assert np.float32(O.radius_squared(0.1)).view(np.uint32) == 0x3C23D70B


def test_config1_pipeline_matches_reference():
    c = golden("config1")
    idx = O.furthest_point_sample(c["xyz"], 1024, 0, True)
    np.testing.assert_array_equal(idx.astype(np.int32), c["fps_idx"])
    centres = np.take_along_axis(c["xyz"], idx[..., None].repeat(3, -1), 1)
    np.testing.assert_array_equal(centres, c["centres"])
    np.testing.assert_array_equal(O.ball_query_pointnet2(0.2, 32, c["xyz"], centres),
                                  c["ball_query_idx"])
    d, i = O.knn(centres, c["xyz"], 16)
    np.testing.assert_array_equal(i, c["knn_idx"])
    np.testing.assert_array_equal(d, c["knn_dist"])
    d, i = O.three_nn(c["xyz"], centres)
    np.testing.assert_array_equal(i, c["three_nn_idx"])
    np.testing.assert_allclose(d, c["three_nn_dist"], rtol=1e-6, atol=0)


def test_three_nn_and_interpolate_match_reference():
    g = golden("pointnet2")
    for name in ("nn_random", "nn_ties"):
        c = g[name]
        d, i = O.three_nn(c["unknown"], c["known"])
        np.testing.assert_array_equal(i, c["idx"], err_msg=name)
        np.testing.assert_allclose(d, c["dist"], rtol=1e-6, atol=0, err_msg=name)
    assert g["nn_ties"]["idx"].tolist() == [[[0, 1, 3], [0, 3, 2]]]  # tests/test_pointnet2.py:35
    c = g["interp_random"]
    out = O.three_interpolate(c["features"], c["indices"], c["weights"])
    np.testing.assert_array_equal(out, c["out"])
    gf = O.three_interpolate_backward(c["grad_out"], c["indices"], c["weights"],
                                      c["features"].shape[-1])
    np.testing.assert_allclose(gf, c["grad_features"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", ["ties_and_duplicates", "seeded_stride"])
def test_propagation_matches_original_pointnet2_cuda(case):
    """docs/parity/pointnet2-cuda.json: the compiled upstream CUDA extension."""
    c = golden("pointnet2_upstream_cuda")[case]
    d, i = O.three_nn(c["unknown"], c["known"])
    np.testing.assert_array_equal(i, c["nearest_indices"])
    np.testing.assert_allclose(d, c["distances"], rtol=2e-6, atol=1e-5)
    out = O.three_interpolate(c["features"], c["interpolate_indices"], c["weights"])
    np.testing.assert_allclose(out, c["interpolated"], rtol=2e-6, atol=1e-5)
    gf = O.three_interpolate_backward(c["gradient"], c["interpolate_indices"], c["weights"],
                                      c["features"].shape[-1])
    np.testing.assert_allclose(gf, c["feature_gradient"], rtol=2e-6, atol=1e-5)
    assert not c["weight_gradient"].any()  # upstream returns an explicit zero weight grad


def test_segmentation_fixture_selections():
    """All 12 FPS / ball-query / three_nn selections of the SSG segmentation fixture."""
    g = golden("pointnet2_segmentation")
    xyz = [g["xyz"]]
    sels = []
    for npoint, radius in [(1024, 0.1), (256, 0.2), (64, 0.4), (16, 0.8)]:
        s = O.furthest_point_sample(xyz[-1], npoint, 0, True)
        new = np.take_along_axis(xyz[-1], s[..., None].repeat(3, -1), 1)
        sels += [s.astype(np.int32), O.ball_query_pointnet2(radius, 32, xyz[-1], new)]
        xyz.append(new)
    for i in range(4):
        sels.append(O.three_nn(xyz[3 - i], xyz[4 - i])[1])
    keys = sorted(k for k in g if k.startswith("selection"))
    assert len(keys) == 12
    for key, got in zip(keys, sels):
        np.testing.assert_array_equal(got, g[key], err_msg=key)


def test_chamfer_matches_reference():
    for name, c in golden("chamfer").items():
        lx, ly = c.get("x_lengths"), c.get("y_lengths")
        loss, gx, gy, (dx, ix), (dy, iy) = O.chamfer_mean_loss_and_grad(c["x"], c["y"], lx, ly)
        P, Q = c["x"].shape[1], c["y"].shape[1]
        vx = np.arange(P)[None] < (lx[:, None] if lx is not None else P)
        vy = np.arange(Q)[None] < (ly[:, None] if ly is not None else Q)
        np.testing.assert_array_equal(np.where(vx, ix, -1), np.where(vx, c["idx_x"], -1), err_msg=name)
        np.testing.assert_array_equal(np.where(vy, iy, -1), np.where(vy, c["idx_y"], -1), err_msg=name)
        np.testing.assert_array_equal(np.where(vx, dx, 0), c["dist_x"], err_msg=name)
        np.testing.assert_array_equal(np.where(vy, dy, 0), c["dist_y"], err_msg=name)
        np.testing.assert_allclose(loss, c["loss"], rtol=1e-5, atol=1e-7, err_msg=name)
        np.testing.assert_allclose(gx, c["grad_x"], rtol=1e-5, atol=1e-7, err_msg=name)
        np.testing.assert_allclose(gy, c["grad_y"], rtol=1e-5, atol=1e-7, err_msg=name)


def _nd_inputs(name):
    import hashlib
    from cases import ND_CASES, nd_cloud_pair
    c = golden("chamfer_nd")[name]
    B, P, Q, D, seed, lens = ND_CASES[name]
    x, y = nd_cloud_pair(B, P, Q, D, seed, lattice=name.endswith("lattice"))
    digest = hashlib.sha256(x.numpy().tobytes() + y.numpy().tobytes()).digest()
    assert np.frombuffer(digest, dtype=np.uint8).tolist() == c["sha256"].tolist()
    lx = None if lens is None else np.array(lens[0], dtype=np.int64)
    ly = None if lens is None else np.array(lens[1], dtype=np.int64)
    return c, x.numpy(), y.numpy(), lx, ly


def test_chamfer_nd_oracle_matches_reference():
    """Feature-space Chamfer (D != 3): the oracle's nearest indices equal the
    reference's for both norms, in both directions."""
    for name in ["d1", "d2_ragged", "d5", "d8_lattice"]:
        c, x, y, lx, ly = _nd_inputs(name)
        vx, vy = nd_valid(x, lx), nd_valid(y, ly)
        for norm in (1, 2):
            _, ix = O.chamfer_nearest(x, y, lx, ly, norm=norm)
            _, iy = O.chamfer_nearest(y, x, ly, lx, norm=norm)
            np.testing.assert_array_equal(ix[vx], c[f"f32_n{norm}_idx_x"][vx], err_msg=name)
            np.testing.assert_array_equal(iy[vy], c[f"f32_n{norm}_idx_y"][vy], err_msg=name)
            assert (ix[~vx] == -1).all() and (iy[~vy] == -1).all()


def nd_valid(points, lengths):
    """Rows below each cloud's length (the reference leaves the others'
    indices unspecified: its loss never reads them)."""
    B, P = points.shape[:2]
    lens = np.full(B, P) if lengths is None else lengths
    return np.arange(P)[None, :] < lens[:, None]
