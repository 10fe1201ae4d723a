"""Generate the golden fixtures in tests/golden/ from the reference package.

Run once, in a container that has the reference checkout, with
``MPO_REFERENCE_PATH`` naming its root (the directory holding the
``mps_pointops`` package)::

    MPO_REFERENCE_PATH=<checkout> python tests/golden/make_golden.py [case ...]

Every output is produced by the reference's OWN code: its CPU path
(``mps_pointops.reference``, ``pointnet2._three_nn_reference``,
``chamfer.chamfer_distance`` ...), the exact kNN oracles in its test files
(``tests/test_knn.py:15-23``, ``tests/test_feature_knn.py:16-35``), its parity
input generators (``tools/pointnet2parity.py:125-170``) and the parity records
it ships (``docs/parity/pointnet2-cuda.json``: the original PointNet++ CUDA
extension; ``docs/parity/pointnet2-segmentation-*.npz``).  The inputs are
stored next to the outputs, so the tests need neither the reference nor a
torch RNG of the same version at run time.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

if "MPO_REFERENCE_PATH" not in os.environ:
    sys.exit("make_golden.py: set MPO_REFERENCE_PATH to the reference checkout's root")
REF = Path(os.environ["MPO_REFERENCE_PATH"])
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REF / "tests"))
sys.path.insert(0, str(REF / "tools"))

from mps_pointops import compat, reference  # noqa: E402  (the reference package)
from mps_pointops import chamfer as ref_chamfer  # noqa: E402
from mps_pointops import pointnet2 as ref_pointnet2  # noqa: E402
import test_feature_knn  # noqa: E402  (reference tests: scalar fp32 oracle)
import test_knn  # noqa: E402  (reference tests: exact lexsort oracle)
import pointnet2parity  # noqa: E402  (reference tools: parity inputs)

sys.path.insert(0, str(OUT))
from cases import ND_CASES, nd_cloud_pair, sphere_cloud  # noqa: E402  (shared with the tests)


def cloud(b, n, seed=0):
    """tests/test_fps.py:9-11, tests/test_knn.py:10-12."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, n, 3, generator=g)


def save(name: str, **arrays) -> None:
    arrays = {k: (v.detach().cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v))
              for k, v in arrays.items()}
    np.savez_compressed(OUT / f"{name}.npz", **arrays)


# ------------------------------------------------------------------ FPS
def fps_cases():
    cases = {}
    for n in [1, 2, 31, 32, 33, 1023, 1024, 1025, 5000]:          # tests/test_fps.py:22-25
        cases[f"n{n}"] = (cloud(1, n), min(n, 256), 0, False)
    cases["batch5"] = (cloud(5, 3000), 128, 0, False)                # :28-31
    cases["start777"] = (cloud(2, 1000), 64, 777, False)            # :34-36
    cases["oversample"] = (cloud(1, 10), 25, 0, False)               # :39-42
    cases["duplicates"] = (torch.tensor([[[0.0, 0, 0], [1, 0, 0], [1, 0, 0], [-1, 0, 0],
                                          [0, 1, 0], [0, 1, 0]]]), 6, 0, False)  # :45-48
    xyz = cloud(1, 2000)                                             # tests/test_compat.py:95-111
    inside = np.float32(np.sqrt(np.float32(1e-3))) * np.float32(0.999)
    outside = np.float32(np.sqrt(np.float32(1e-3))) * np.float32(1.001)
    xyz[0, 1:40] = torch.tensor([inside, 0.0, 0.0]) * torch.rand(
        39, 1, generator=torch.Generator().manual_seed(5))
    xyz[0, 40] = torch.tensor([float(inside), 0.0, 0.0])
    xyz[0, 41] = torch.tensor([float(outside), 0.0, 0.0])
    cases["skip_near_origin"] = (xyz, 2000, 0, True)
    cases["all_near_origin"] = (torch.zeros(1, 50, 3), 5, 0, True)  # tests/test_compat.py:114-118
    pattern = torch.zeros((1, 129, 3))                               # tests/test_fps.py:103-118
    pattern[0, 1::2, 0] = 1
    pattern[0, 2::4, 1] = -1
    for skip in (False, True):
        cases[f"ties_skip{int(skip)}"] = (pattern.clone(), 150, 3, skip)
    for n in [4095, 4096, 4097, 8193]:                               # tests/test_fps.py:88-100
        cases[f"chunk{n}"] = (cloud(1, n, seed=27), min(n + 2, 20), n // 2, False)
    g = torch.Generator().manual_seed(0)
    cases["config1_compat"] = (torch.rand(8, 4096, 3, generator=g), 1024, 0, True)
    out = {}
    for name, (xyz, npoint, start, skip) in cases.items():
        want = reference.furthest_point_sample(xyz, npoint, start, skip)
        out[f"{name}/xyz"] = xyz
        out[f"{name}/meta"] = np.array([npoint, start, int(skip)], dtype=np.int64)
        out[f"{name}/idx"] = want
    save("fps", **out)


# ------------------------------------------------------------------ kNN
def knn_cases():
    out = {}
    for n in [1, 31, 32, 33, 1000, 5000]:                            # tests/test_knn.py:35-42
        for k in [1, 5, 32, 128]:
            if k > n:
                continue
            ref = cloud(1, n)
            out[f"n{n}_k{k}/query"] = ref[:, :50] + 0.01
            out[f"n{n}_k{k}/ref"] = ref
    for m in [1, 7, 8, 9, 100]:                                      # :45-48
        out[f"m{m}/query"] = cloud(1, m, seed=1)
        out[f"m{m}/ref"] = cloud(1, 2000)
    ref = cloud(1, 256)                                              # :51-54 (k = N = 256)
    out["kmax/query"], out["kmax/ref"] = ref[:, :20], ref
    out["batch3/query"], out["batch3/ref"] = cloud(3, 40, seed=1), cloud(3, 3000)  # :57-59
    for desc in (False, True):                                       # :62-67
        ref = cloud(1, 20000)
        ref = ref[:, ref[0, :, 0].argsort(descending=desc)]
        out[f"sorted{int(desc)}/query"], out[f"sorted{int(desc)}/ref"] = cloud(1, 64, seed=1), ref
    ref = torch.zeros(1, 300, 3)                                     # :70-74
    ref[0, ::3] = 1.0
    out["ties/query"], out["ties/ref"] = torch.zeros(1, 2, 3), ref
    ks = {"kmax": 256, "batch3": 32, "sorted0": 128, "sorted1": 128, "ties": 150}
    names = sorted({k.split("/")[0] for k in out})
    for name in names:
        if name.startswith("n"):
            k = int(name.split("_k")[1])
        elif name.startswith("m"):
            k = 16
        else:
            k = ks[name]
        q, r = out[f"{name}/query"], out[f"{name}/ref"]
        d, i = test_knn.exact(q, r, k)                               # the reference's own oracle
        out[f"{name}/k"] = np.array(k)
        out[f"{name}/dist"] = d.astype(np.float32)
        out[f"{name}/idx"] = i.astype(np.int64)
    save("knn", **out)


def feature_knn_cases():
    out = {}
    for dim in [1, 2, 4, 64, 128]:                                   # tests/test_feature_knn.py:38-58
        for k in [1, 5, 33]:
            gen = torch.Generator().manual_seed(107 + dim)
            query = torch.randn((2, 9, dim), generator=gen)
            ref = torch.randn((2, 97, dim), generator=gen)
            ref[:, 20] = ref[:, 3]
            query[:, 0] = ref[:, 3]
            name = f"d{dim}_k{k}"
            dists, idxs = zip(*(test_feature_knn._oracle(query[b], ref[b], k) for b in range(2)))
            out[f"{name}/query"], out[f"{name}/ref"] = query, ref
            out[f"{name}/k"] = np.array(k)
            out[f"{name}/dist"] = np.stack(dists)
            out[f"{name}/idx"] = np.stack(idxs)
    gen = torch.Generator().manual_seed(2026)                        # :61-73
    ref = torch.randn((1, 300, 64), generator=gen)
    query = torch.randn((1, 4, 64), generator=gen)
    ref[0, 1] = ref[0, 0]
    query[0, 0] = ref[0, 0]
    d, i = test_feature_knn._oracle(query[0], ref[0], 256)
    out["k256/query"], out["k256/ref"], out["k256/k"] = query, ref, np.array(256)
    out["k256/dist"], out["k256/idx"] = d[None], i[None]
    save("feature_knn", **out)


# ------------------------------------------------------------------ ball query
def ball_query_cases():
    out = {}

    def add(name, q, r, radius, K):
        d2, idx = reference.ball_query(q, r, radius, K)              # reference.py:83-121
        out[f"{name}/query"], out[f"{name}/ref"] = q, r
        out[f"{name}/radius"], out[f"{name}/K"] = np.array(radius, np.float64), np.array(K)
        out[f"{name}/dist2"], out[f"{name}/idx"] = d2, idx

    torch.manual_seed(9)
    add("random", torch.randn(2, 7, 3), torch.randn(2, 19, 3), 2.0, 5)
    add("first_k", torch.zeros((1, 1, 3)),                           # tests/test_ball_query_mps.py:76-87
        torch.tensor([[[0.8, 0, 0], [0.1, 0, 0], [1.0, 0, 0], [0.2, 0, 0]]]), 1.0, 2)
    positions = [0, 1, 31, 32, 64, 128, 224, 250, 256]              # :90-112
    pts = torch.zeros((1, 257, 3))
    pts[0, :, 0] = torch.arange(257, dtype=torch.float32)
    for k in [1, 7, 31, 33, 65]:
        add(f"sorted_k{k}", pts[:, positions].clone(), pts, 20.5, k)
    one = torch.tensor(1.0)
    add("boundary", torch.zeros((1, 1, 3)), torch.tensor(                # :216-229
        [[[torch.nextafter(one, torch.tensor(0.0)).item(), 0, 0], [1.0, 0, 0],
          [torch.nextafter(one, torch.tensor(float("inf"))).item(), 0, 0]]]), 1.0, 3)
    add("r2_rounding", torch.zeros((1, 1, 3)),                       # :248-261
        torch.tensor([[[0.09999999403953552, 3.112176273134537e-05, 0.0]]]), 0.1, 1)
    nf = torch.full((1, 97, 3), 2.0)                                  # :200-213
    nf[0, [0, 31, 32, 63, 64, 95, 96], :] = 0.0
    nf[0, 31, 0], nf[0, 64, 0] = float("nan"), float("inf")
    add("nonfinite_blocks", torch.zeros((1, 1, 3)), nf, 0.5, 7)
    q = torch.tensor([[[0.0, 0, 0], [float("nan"), 0, 0], [float("inf"), 0, 0],
                       [-float("inf"), 0, 0]]])                       # :465-490
    p = torch.tensor([[[float("nan"), 0, 0], [float("inf"), 0, 0], [-float("inf"), 0, 0],
                       [0.25, 0, 0], [0.5, 0, 0]]])
    add("nonfinite_queries", q, p, 1.0, 3)
    add("tiny_radius", torch.zeros((1, 1, 3)),                       # :385-409
        torch.tensor([[[0.0, 0.0, 0.0], [1e-20, 0.0, 0.0]]]), 1e-30, 2)
    add("huge_radius", torch.zeros((1, 1, 3)),
        torch.tensor([[[1e19, 0.0, 0.0], [5e19, 0.0, 0.0], [2e20, 0.0, 0.0]]]), 1e20, 3)
    add("zero_radius", torch.rand(1, 4, 3, generator=torch.Generator().manual_seed(3)),
        torch.rand(1, 20, 3, generator=torch.Generator().manual_seed(4)), 0.0, 3)
    g = torch.Generator().manual_seed(11)
    add("dense", torch.rand(3, 300, 3, generator=g), torch.rand(3, 2000, 3, generator=g), 0.15, 64)
    save("ball_query", **out)

    # compat padding, BASELINE config 1 (xyz = rand(8,4096,3) seed 0, centres = FPS 1024)
    g = torch.Generator().manual_seed(0)
    xyz = torch.rand(8, 4096, 3, generator=g)
    idx = compat.furthest_point_sample(xyz, 1024)
    centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx).transpose(1, 2).contiguous()
    grouped = compat.ball_query(0.2, 32, xyz, centres)
    knn_d, knn_i = test_knn.exact(centres, xyz, 16)
    tn_d, tn_i = ref_pointnet2._three_nn_reference(xyz, centres)
    save("config1", xyz=xyz, fps_idx=idx, centres=centres, ball_query_idx=grouped,
         knn_dist=knn_d.astype(np.float32), knn_idx=knn_i.astype(np.int64),
         three_nn_dist=tn_d, three_nn_idx=tn_i)
    pad = compat.ball_query(0.5, 4, torch.tensor([[[5.0, 0, 0], [0.1, 0, 0], [9, 9, 9], [0.2, 0, 0]]]),
                            torch.tensor([[[0.0, 0, 0], [50.0, 50, 50]]]))  # tests/test_compat.py:140-145
    save("compat_pad", idx=pad)


# ------------------------------------------------------------------ PointNet++ propagation
def pointnet2_cases():
    out = {}
    rng = np.random.default_rng(59)                                   # tests/test_pointnet2.py:42-58
    unknown = torch.from_numpy(rng.normal(size=(2, 37, 6)).astype("float32"))[..., ::2].contiguous()
    known = torch.from_numpy(rng.normal(size=(2, 113, 6)).astype("float32"))[..., ::2].contiguous()
    d, i = ref_pointnet2._three_nn_reference(unknown, known)
    out.update({"nn_random/unknown": unknown, "nn_random/known": known,
                "nn_random/dist": d, "nn_random/idx": i})
    u = torch.tensor([[[0., 0., 0.], [2., 0., 0.]]])                  # :24-39
    k = torch.tensor([[[1., 0., 0.], [-1., 0., 0.], [0., 2., 0.], [1., 0., 0.]]])
    d, i = ref_pointnet2._three_nn_reference(u, k)
    out.update({"nn_ties/unknown": u, "nn_ties/known": k, "nn_ties/dist": d, "nn_ties/idx": i})
    gen = torch.Generator().manual_seed(109)                          # :115-126
    f = torch.randn(2, 4, 17, generator=gen)
    ind = torch.randint(17, (2, 11, 3), generator=gen, dtype=torch.int32)
    w = torch.randn(2, 11, 3, generator=gen)
    up = torch.randn(2, 4, 11, generator=gen)
    fr = f.clone().requires_grad_()
    o = ref_pointnet2._three_interpolate_reference(fr, ind, w)
    o.backward(up)
    out.update({"interp_random/features": f, "interp_random/indices": ind,
                "interp_random/weights": w, "interp_random/grad_out": up,
                "interp_random/out": o.detach(), "interp_random/grad_features": fr.grad})
    save("pointnet2", **out)

    # Original PointNet++ CUDA extension outputs (docs/parity/pointnet2-cuda.json) with the
    # inputs rebuilt by the reference's own generators (tools/pointnet2parity.py:125-170).
    rec = json.loads((REF / "docs/parity/pointnet2-cuda.json").read_text())
    cpu = torch.device("cpu")
    up = {}
    for name, make in (("ties-and-duplicates", pointnet2parity._small_inputs),
                       ("seeded-stride", pointnet2parity._large_inputs)):
        unknown, known, features, weights, gradient = make(cpu)
        case = rec["cases"][name]
        key = name.replace("-", "_")
        up[f"{key}/unknown"], up[f"{key}/known"] = unknown.detach(), known.detach()
        up[f"{key}/features"], up[f"{key}/weights"] = features.detach(), weights.detach()
        up[f"{key}/gradient"] = gradient
        for field, dtype in (("nearest_indices", np.int32), ("distances", np.float32),
                             ("interpolate_indices", np.int32), ("interpolated", np.float32),
                             ("feature_gradient", np.float32), ("weight_gradient", np.float32)):
            up[f"{key}/{field}"] = np.asarray(case[field], dtype=dtype)
    save("pointnet2_upstream_cuda", **up)

    # PointNet++ SSG segmentation fixture: the xyz of docs/parity/pointnet2-segmentation-
    # synthetic-fixture.npz and the 12 selection arrays the reference recorded on MPS
    # (docs/parity/pointnet2-segmentation-mps-safe.npz); its CPU path reproduces all 12.
    fx = np.load(REF / "docs/parity/pointnet2-segmentation-synthetic-fixture.npz")
    mps = np.load(REF / "docs/parity/pointnet2-segmentation-mps-safe.npz")
    sel = {k.replace("::", "_"): mps[k] for k in mps.files if k.startswith("selection::")}
    save("pointnet2_segmentation", xyz=fx["points"][..., :3].copy(), **sel)


# ------------------------------------------------------------------ Chamfer
def chamfer_cases():
    out = {}

    def add(name, x, y, lx=None, ly=None):
        B = x.shape[0]
        flx = torch.full((B,), x.shape[1], dtype=torch.long) if lx is None else lx
        fly = torch.full((B,), y.shape[1], dtype=torch.long) if ly is None else ly
        ix = ref_chamfer._nearest_indices(x, y, flx, fly)           # chamfer.py:161-212
        iy = ref_chamfer._nearest_indices(y, x, fly, flx)
        dx = ref_chamfer._selected_squared_distance(x, y, ix, flx)  # chamfer.py:297-308
        dy = ref_chamfer._selected_squared_distance(y, x, iy, fly)
        xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
        loss, _ = ref_chamfer.chamfer_distance(xr, yr, lx, ly)
        loss.backward()
        out[f"{name}/x"], out[f"{name}/y"] = x, y
        if lx is not None:
            out[f"{name}/x_lengths"], out[f"{name}/y_lengths"] = lx, ly
        out[f"{name}/idx_x"], out[f"{name}/idx_y"] = ix, iy
        out[f"{name}/dist_x"], out[f"{name}/dist_y"] = dx, dy
        out[f"{name}/loss"] = loss.detach()
        out[f"{name}/grad_x"], out[f"{name}/grad_y"] = xr.grad, yr.grad

    gen = torch.Generator().manual_seed(137)                          # tests/test_chamfer.py:480-511
    add("lengths", torch.randn((3, 13, 3), generator=gen), torch.randn((3, 67, 3), generator=gen),
        torch.tensor([13, 4, 9]), torch.tensor([67, 39, 3]))
    gen = torch.Generator().manual_seed(2026)                         # :431-449
    add("uneven", torch.randn((2, 7, 3), generator=gen), torch.randn((2, 5, 3), generator=gen),
        torch.tensor([7, 3]), torch.tensor([5, 2]))
    q = torch.zeros((2, 9, 3))                                         # :452-477 (finite rows)
    r = torch.full((2, 37, 3), 9.0)
    r[:, 0], r[:, 31], r[:, 36] = torch.tensor([1.0, 0, 0]), torch.tensor([-1.0, 0, 0]), \
        torch.tensor([0.0, 1, 0])
    add("ties", q, r, torch.tensor([8, 7]), torch.tensor([37, 32]))
    add("tie_reverse", torch.tensor([[[0.0, 0, 0], [2.0, 0, 0]]]), torch.tensor([[[1.0, 0, 0]]]))
    g2 = torch.Generator().manual_seed(2)                              # BASELINE config 2 shape, smaller
    x = torch.randn(2, 2048, 3, generator=g2)
    g3 = torch.Generator().manual_seed(3)
    y = x + 0.05 * torch.randn(2, 2048, 3, generator=g3)
    y = torch.stack([y[b, torch.randperm(2048, generator=g3)] for b in range(2)])
    add("config2_small", x, y)
    g4 = torch.Generator().manual_seed(4)
    add("d8", torch.randn(2, 33, 8, generator=g4), torch.randn(2, 45, 8, generator=g4))
    save("chamfer", **out)


def chamfer_nd_cases():
    """Feature-space (D != 3) Chamfer across several tiles of the symmetric
    kernel, and float64 inputs (chamfer.py:101-102), on the reference's CPU
    path: nearest indices of both directions and losses for norm 2 and norm 1,
    gradients where the clouds are small.  Inputs are rebuilt from the seeds
    in ND_CASES (a digest is stored to detect a different generator)."""
    import hashlib
    out = {}
    for name, (B, P, Q, D, seed, lens) in ND_CASES.items():
        x, y = nd_cloud_pair(B, P, Q, D, seed, lattice=name.endswith("lattice"))
        out[f"{name}/sha256"] = np.frombuffer(
            hashlib.sha256(x.numpy().tobytes() + y.numpy().tobytes()).digest(), dtype=np.uint8)
        lx = None if lens is None else torch.tensor(lens[0])
        ly = None if lens is None else torch.tensor(lens[1])
        flx = torch.full((B,), P) if lx is None else lx
        fly = torch.full((B,), Q) if ly is None else ly
        for dtype in (torch.float32, torch.float64):
            xs, ys = x.to(dtype), y.to(dtype)
            tag = f"{name}/{'f64' if dtype == torch.float64 else 'f32'}"
            for norm in (1, 2):
                xr, yr = xs.clone().requires_grad_(), ys.clone().requires_grad_()
                loss, _ = ref_chamfer.chamfer_distance(xr, yr, lx, ly, norm=norm)
                loss.backward()
                out[f"{tag}_n{norm}_idx_x"] = ref_chamfer._nearest_indices(
                    xs, ys, flx, fly, norm=norm).int()
                out[f"{tag}_n{norm}_idx_y"] = ref_chamfer._nearest_indices(
                    ys, xs, fly, flx, norm=norm).int()
                out[f"{tag}_n{norm}_loss"] = loss.detach()
                if dtype == torch.float32 or D <= 8:
                    out[f"{tag}_n{norm}_grad_x"] = xr.grad
                    out[f"{tag}_n{norm}_grad_y"] = yr.grad
    # float64 single-directional with weights and sum reductions
    g = torch.Generator().manual_seed(907)
    x64 = torch.randn(3, 50, 3, generator=g, dtype=torch.float64)
    y64 = torch.randn(3, 41, 3, generator=g, dtype=torch.float64)
    w = torch.tensor([0.5, 2.0, 1.0], dtype=torch.float64)
    xr, yr = x64.clone().requires_grad_(), y64.clone().requires_grad_()
    loss, _ = ref_chamfer.chamfer_distance(xr, yr, weights=w, batch_reduction="sum",
                                           single_directional=True)
    loss.backward()
    out["f64_weighted/x"], out["f64_weighted/y"], out["f64_weighted/weights"] = x64, y64, w
    out["f64_weighted/loss"] = loss.detach()
    out["f64_weighted/grad_x"], out["f64_weighted/grad_y"] = xr.grad, yr.grad
    save("chamfer_nd", **out)


def chamfer_l1_cases():
    """chamfer_distance(norm=1) on the reference's CPU path (chamfer.py:161-212,
    254-293, 342-488): losses and gradients for lengths, weights, normals,
    reductions and single-directional calls."""
    out = {}
    g = torch.Generator().manual_seed(55)
    x, y = torch.randn(3, 40, 3, generator=g), torch.randn(3, 31, 3, generator=g)
    lx, ly = torch.tensor([40, 17, 5]), torch.tensor([31, 9, 30])
    xn = torch.nn.functional.normalize(torch.randn(3, 40, 3, generator=g), dim=-1)
    yn = torch.nn.functional.normalize(torch.randn(3, 31, 3, generator=g), dim=-1)
    w = torch.tensor([0.5, 2.0, 1.0])
    cases = {
        "plain": dict(),
        "lengths": dict(x_lengths=lx, y_lengths=ly),
        "weights_sum": dict(x_lengths=lx, y_lengths=ly, weights=w, batch_reduction="sum"),
        "normals": dict(x_lengths=lx, y_lengths=ly, x_normals=xn, y_normals=yn),
        "single_max": dict(single_directional=True, point_reduction="max", batch_reduction=None),
        "d5": dict(),
    }
    for name, kw in cases.items():
        xs, ys = (torch.randn(2, 23, 5, generator=g), torch.randn(2, 19, 5, generator=g)) \
            if name == "d5" else (x, y)
        xr, yr = xs.clone().requires_grad_(), ys.clone().requires_grad_()
        loss, nl = ref_chamfer.chamfer_distance(xr, yr, norm=1, **kw)
        loss.sum().backward()
        out[f"{name}/x"], out[f"{name}/y"] = xs, ys
        out[f"{name}/loss"] = loss.detach()
        out[f"{name}/grad_x"], out[f"{name}/grad_y"] = xr.grad, yr.grad
        if nl is not None:
            out[f"{name}/normal_loss"] = nl.detach()
        if name != "d5":
            lxx = kw.get("x_lengths", torch.full((3,), 40))
            lyy = kw.get("y_lengths", torch.full((3,), 31))
            out[f"{name}/idx_x"] = ref_chamfer._nearest_indices(xs, ys, lxx, lyy, norm=1)
    out["inputs/x_lengths"], out["inputs/y_lengths"] = lx, ly
    out["inputs/x_normals"], out["inputs/y_normals"], out["inputs/weights"] = xn, yn, w
    save("chamfer_l1", **out)


# ------------------------------------------------------------------ flat (torch_cluster) API
def flat_cases():
    """The CPU path of mps_pointops/flat.py: _reference_search (:264-288) for
    padded kNN / radius indices, fps (:161-217) and the edge builders."""
    from mps_pointops import flat as ref_flat
    out = {}

    def ptr_of(lengths):
        p = [0]
        for n in lengths:
            p.append(p[-1] + n)
        return torch.tensor(p, dtype=torch.long)

    def search(name, x, y, lx, ly, width, radius=None):
        px, py = ptr_of(lx), ptr_of(ly)
        idx = ref_flat._reference_search(x, y, px, py, width, radius)
        out[f"{name}/x"], out[f"{name}/y"] = x, y
        out[f"{name}/ptr_x"], out[f"{name}/ptr_y"] = px, py
        out[f"{name}/meta"] = np.array([width, -1.0 if radius is None else radius])
        out[f"{name}/idx"] = idx

    g = torch.Generator().manual_seed(31)
    lx = [0, 1, 7, 33, 100, 257, 0, 64]
    ly = [5, 3, 0, 40, 17, 90, 2, 64]
    x = torch.randn(sum(lx), 3, generator=g)
    y = torch.randn(sum(ly), 3, generator=g)
    for k in (1, 5, 16, 40):
        search(f"knn3_k{k}", x, y, lx, ly, k)
    for r, m in ((0.5, 8), (1.0, 32), (0.21, 4), (3.0, 300)):
        search(f"radius_r{r}_m{m}", x, y, lx, ly, m, radius=r)
    xn, yn = x.clone(), y.clone()
    xn[10, 0] = float("nan")
    xn[11, 1] = float("inf")
    xn[50, 2] = -float("inf")
    yn[4, 0] = float("nan")
    yn[60, 1] = float("inf")
    search("knn3_nonfinite", xn, yn, lx, ly, 8)
    search("radius_nonfinite", xn, yn, lx, ly, 16, radius=1.5)
    xt = torch.randint(0, 3, (sum(lx), 3), generator=g).float()   # many exact ties
    yt = torch.randint(0, 3, (sum(ly), 3), generator=g).float()
    search("knn3_ties", xt, yt, lx, ly, 12)
    search("radius_ties", xt, yt, lx, ly, 20, radius=1.0)
    for d in (1, 5, 16, 64):
        xf = torch.randn(sum(lx), d, generator=g)
        yf = torch.randn(sum(ly), d, generator=g)
        search(f"knn_d{d}", xf, yf, lx, ly, 10)

    # FPS: per-cloud samples from given local starts (flat.py:208-217) and the
    # public call with random_start=False.
    lf = [1, 2, 30, 0, 257, 1000, 4]
    xf = torch.randn(sum(lf), 3, generator=g)
    starts = [0, 1, 17, 0, 200, 999, 3]
    counts = ref_flat._sample_counts(lf, ref_flat._ratio(0.37, torch.float32), mps=True)
    pf = ptr_of(lf).tolist()
    samples = []
    for b, (lo, hi) in enumerate(zip(pf, pf[1:])):
        if counts[b]:
            samples.append(reference.furthest_point_sample(
                xf[lo:hi].unsqueeze(0), counts[b], start_idx=starts[b])[0] + lo)
    out["fps_starts/x"], out["fps_starts/ptr"] = xf, torch.tensor(pf)
    out["fps_starts/starts"] = torch.tensor(starts)
    out["fps_starts/counts"] = torch.tensor(counts)
    out["fps_starts/idx"] = torch.cat(samples)
    out["fps_over/x"] = xf[:10]
    out["fps_over/idx"] = ref_flat.fps(xf[:10], ptr=[0, 4, 10], ratio=1.7, random_start=False)
    xd = torch.tensor([[0.0, 0, 0], [1, 0, 0], [1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, 1, 0]])
    out["fps_dup/x"] = xd
    out["fps_dup/idx"] = ref_flat.fps(xd, ratio=1.0, random_start=False)

    # Sample counts, CPU rule (float32 sizes) and GPU rule (ratio dtype).
    lengths = list(range(0, 300))
    for ratio in (0.05, 0.3, 1 / 3, 0.6, 0.95):
        r = ref_flat._ratio(ratio, torch.float32)
        out[f"counts_{ratio:.4f}/cpu"] = torch.tensor(ref_flat._sample_counts(lengths, r, mps=False))
        out[f"counts_{ratio:.4f}/gpu"] = torch.tensor(ref_flat._sample_counts(lengths, r, mps=True))

    # Public edge builders on one small ragged batch.
    xe = torch.randn(60, 3, generator=g)
    be = torch.tensor([0] * 20 + [1] * 15 + [3] * 25)
    ye = torch.randn(30, 3, generator=g)
    bye = torch.tensor([0] * 10 + [2] * 5 + [3] * 15)
    out["edges/x"], out["edges/batch_x"] = xe, be
    out["edges/y"], out["edges/batch_y"] = ye, bye
    out["edges/knn"] = ref_flat.knn(xe, ye, 4, be, bye)
    out["edges/radius"] = ref_flat.radius(xe, ye, 0.8, be, bye, max_num_neighbors=6)
    out["edges/knn_graph"] = ref_flat.knn_graph(xe, 3, be)
    out["edges/knn_graph_loop_t2s"] = ref_flat.knn_graph(xe, 3, be, loop=True,
                                                          flow="target_to_source")
    out["edges/radius_graph"] = ref_flat.radius_graph(xe, 0.9, be, max_num_neighbors=5)
    out["edges/radius_graph_loop"] = ref_flat.radius_graph(xe, 0.9, be, loop=True,
                                                           max_num_neighbors=5)
    save("flat", **out)


# ------------------------------------------------------------------ SA grouping
def grouping_cases():
    """compat.gather_operation / grouping_operation (compat.py:62-73, torch gather
    on CPU) and the set-abstraction grouping of tests/test_pointnet2_e2e.py:40-44,
    forward and backward with a fixed output gradient."""
    out = {}
    g = torch.Generator().manual_seed(404)
    B, Np, P, S, C = 2, 300, 40, 12, 5
    xyz = torch.rand(B, Np, 3, generator=g)
    feats = torch.randn(B, C, Np, generator=g)
    sampled = compat.furthest_point_sample(xyz, P)
    new_xyz = compat.gather_operation(xyz.transpose(1, 2).contiguous(), sampled)
    new_xyz = new_xyz.transpose(1, 2).contiguous()
    out["gather/features"], out["gather/idx"] = xyz.transpose(1, 2).contiguous(), sampled
    out["gather/out"] = compat.gather_operation(xyz.transpose(1, 2).contiguous(), sampled)
    for radius in (0.15, 0.4):
        xr = xyz.clone().requires_grad_()
        qr = new_xyz.clone().requires_grad_()
        fr = feats.clone().requires_grad_()
        neighbors = compat.ball_query(radius, S, xr, qr)
        grouped_xyz = compat.grouping_operation(xr.transpose(1, 2).contiguous(), neighbors)
        grouped_xyz = grouped_xyz - qr.transpose(1, 2).unsqueeze(-1)
        grouped = torch.cat((grouped_xyz, compat.grouping_operation(fr, neighbors)), dim=1)
        gout = torch.randn(grouped.shape, generator=g)
        grouped.backward(gout)
        name = f"qg_r{radius}"
        out[f"{name}/xyz"], out[f"{name}/new_xyz"], out[f"{name}/features"] = xyz, new_xyz, feats
        out[f"{name}/meta"] = np.array([radius, S])
        out[f"{name}/idx"], out[f"{name}/out"], out[f"{name}/grad_out"] = neighbors, grouped, gout
        out[f"{name}/grad_xyz"], out[f"{name}/grad_new_xyz"] = xr.grad, qr.grad
        out[f"{name}/grad_features"] = fr.grad
    save("grouping", **out)


# ------------------------------------------------------------------ Pointcept
def pointcept_cases():
    """mps_pointops/pointcept.py on CPU (the reference's own path): FPS with
    cumulative offsets (:77-98), padded kNN with the 1e10 ceiling (:101-165),
    grouping with relative xyz and its gradients (:168-203), and
    interpolation with its feature gradient (:219-243)."""
    from mps_pointops import pointcept as ref_pc
    out = {}
    g = torch.Generator().manual_seed(77)
    lx = [0, 5, 40, 300, 1, 128, 64]
    ly = [3, 2, 17, 90, 0, 128, 5]
    ends = lambda ls: torch.tensor(np.cumsum(ls), dtype=torch.int64)  # noqa: E731
    x = torch.randn(sum(lx), 3, generator=g)
    y = torch.randn(sum(ly), 3, generator=g)
    x[50, 1] = float("nan")               # cloud 2: a NaN reference
    x[60, 0] = float("inf")               # cloud 3: an inf reference
    x[100] = torch.tensor([1.0e5, 0.0, 0.0])  # cloud 3: beyond the 1e10 ceiling
    y[25] = torch.tensor([-1.0e5, 0.0, 0.0])  # cloud 3: a query far from all
    out["x"], out["y"] = x, y
    out["offset"], out["new_offset"] = ends(lx), ends(ly)
    for k in (1, 3, 16, 50):
        idx, dist = ref_pc.knn_query(k, x, ends(lx), y, ends(ly))
        out[f"knn_k{k}/idx"], out[f"knn_k{k}/dist"] = idx, dist
    # Self query (new_xyz omitted) and exact ties on a lattice.
    xt = torch.randint(0, 4, (sum(lx), 3), generator=g).float()
    out["ties/x"] = xt
    out["ties/idx"], out["ties/dist"] = ref_pc.knn_query(12, xt, ends(lx))
    # FPS: counts per batch at most the batch size, some zero.
    xf = torch.randn(sum(lx), 3, generator=g)
    counts = [0, 5, 13, 200, 1, 64, 0]
    out["fps/x"], out["fps/new_offset"] = xf, ends(counts)
    out["fps/idx"] = ref_pc.farthest_point_sampling(xf, ends(lx), ends(counts))
    # Interpolation and grouping, forward and backward.
    feat = torch.randn(sum(lx), 6, generator=g)
    f1 = feat.clone().requires_grad_()
    interp = ref_pc.interpolation(xf, y, f1, ends(lx), ends(ly), k=3)
    gi = torch.randn(interp.shape, generator=g)
    interp.backward(gi)
    out["interp/feat"], out["interp/out"] = feat, interp
    out["interp/grad_out"], out["interp/grad_feat"] = gi, f1.grad
    idx, _ = ref_pc.knn_query(8, xf, ends(lx), y, ends(ly))
    xr = xf.clone().requires_grad_()
    qr = y.clone().requires_grad_()
    f2 = feat.clone().requires_grad_()
    grouped = ref_pc.grouping(idx, f2, xr, qr, with_xyz=True)
    gg = torch.randn(grouped.shape, generator=g)
    grouped.backward(gg)
    out["group/idx"], out["group/out"], out["group/grad_out"] = idx, grouped, gg
    out["group/grad_xyz"], out["group/grad_new_xyz"] = xr.grad, qr.grad
    out["group/grad_feat"] = f2.grad
    save("pointcept", **out)


# ------------------------------------------------------------------ large FPS
def fps_large_cases():
    """Full-length config 3 (2^20 points -> 65,536 samples, about 4 minutes on
    8 cores) and 1024-step runs on 1.5 M and 4 M point clouds, all by
    reference.furthest_point_sample.  Only the indices and a digest of the
    input are stored; the tests rebuild the input with the same generator."""
    import hashlib
    out = {}
    for name, n, npoint, seed in (("config3", 1 << 20, 65536, 4),
                                  ("n1p5m", 1_500_000, 1024, 41),
                                  ("n4m", 4_000_000, 1024, 42)):
        xyz = sphere_cloud(n, seed)
        out[f"{name}/meta"] = np.array([n, npoint, seed], dtype=np.int64)
        out[f"{name}/sha256"] = np.frombuffer(
            hashlib.sha256(xyz.numpy().tobytes()).digest(), dtype=np.uint8)
        out[f"{name}/idx"] = reference.furthest_point_sample(xyz, npoint, 0, False).to(torch.int32)
        print(name, "done", flush=True)
    save("fps_large", **out)


CASES = {
    "fps": fps_cases, "fps_large": fps_large_cases, "knn": knn_cases,
    "feature_knn": feature_knn_cases,
    "ball_query": ball_query_cases, "pointnet2": pointnet2_cases, "chamfer": chamfer_cases,
    "flat": flat_cases, "grouping": grouping_cases, "chamfer_l1": chamfer_l1_cases,
    "chamfer_nd": chamfer_nd_cases,
    "pointcept": pointcept_cases,
}

if __name__ == "__main__":
    # python make_golden.py [case ...]   (default: every case)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in sys.argv[1:] or list(CASES):
        CASES[name]()
    for f in sorted(OUT.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size / 1024:.0f} KiB")
