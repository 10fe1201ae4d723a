"""CPU oracle for the mps_pointops hot path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes front end over ``oracle/pointops_oracle.c`` (built by
``oracle/Makefile`` into ``oracle/_build/liboracle.so``).  Each function
restates one CPU algorithm of the reference package gamzerA/mps-pointops
v1.0.0; the C source cites the reference file:line it follows.

Only the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module.  The product package never does: a
CUDA call that silently landed here would void every parity claim.

Work is split over independent clouds / query ranges on host threads
(ctypes drops the GIL during a foreign call).  The split never changes the
order of a floating-point accumulation that tests compare bit-for-bit.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64


def build() -> Path:
    """Compile the C oracle in place (idempotent)."""
    src = _HERE / "pointops_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.oracle_fps.argtypes = [_f32p, _i64, _i64, _i64, _i64, ctypes.c_int, _i64p]
        lib.oracle_knn.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _f32p, _i64p]
        lib.oracle_knn_sqdist.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64p, _f32p]
        lib.oracle_ball_query.argtypes = [_f32p, _f32p, _i64p, _i64p, _i64, _i64, _i64, _i64,
                                          ctypes.c_float, _f32p, _i64p]
        lib.oracle_three_nn.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p, _i32p]
        lib.oracle_three_interpolate.argtypes = [_f32p, _i64p, _f32p, _i64, _i64, _i64, _i64, _f32p]
        lib.oracle_three_interpolate_backward.argtypes = [_f32p, _i64p, _f32p, _i64, _i64, _i64,
                                                          _i64, _f32p]
        lib.oracle_chamfer_nearest.argtypes = [_f32p, _f32p, _i64p, _i64p, _i64, _i64, _i64, _i64,
                                               _f32p, _i64p]
        lib.oracle_chamfer_mean_loss_and_grad.argtypes = [
            _f32p, _f32p, _i64p, _i64p, _i64, _i64, _i64, _i64, _i64p, _i64p, _f32p, _f32p,
            _f32p, _f32p]
        lib.oracle_chamfer_mean_loss_and_grad.restype = ctypes.c_double
        lib.oracle_chamfer_nearest_l1.argtypes = [_f32p, _f32p, _i64p, _i64p, _i64, _i64, _i64,
                                                  _i64, _f32p, _i64p]
        lib.oracle_flat_search.argtypes = [_f32p, _f32p, _i64p, _i64p, _i64, _i64, _i64,
                                           ctypes.c_int, ctypes.c_float, ctypes.c_int, _i64, _i64,
                                           _i64p]
        _lib = lib
    return _lib


def _ptr(a: np.ndarray | None, kind):
    if a is None:
        return ctypes.cast(None, kind)
    return a.ctypes.data_as(kind)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64a(a) -> np.ndarray | None:
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def threads() -> int:
    env = os.environ.get("MPO_ORACLE_THREADS")
    return max(1, int(env)) if env else max(1, os.cpu_count() or 1)


def _parallel(jobs):
    jobs = list(jobs)
    n = min(threads(), len(jobs))
    if n <= 1:
        for j in jobs:
            j()
        return
    with ThreadPoolExecutor(n) as pool:
        for f in [pool.submit(j) for j in jobs]:
            f.result()


def _ranges(total: int, parts: int):
    parts = max(1, min(parts, total))
    step = -(-total // parts) if total else 0
    return [(lo, min(total, lo + step)) for lo in range(0, total, step)] if total else []


# ---------------------------------------------------------------- FPS
def furthest_point_sample(xyz, npoint: int, start_idx: int = 0,
                          skip_near_origin: bool = False) -> np.ndarray:
    """mps_pointops/reference.py:27-58.  (B,N,3) -> (B,npoint) int64."""
    lib = _load()
    xyz = _f32(xyz)
    B, N, _ = xyz.shape
    out = np.empty((B, npoint), dtype=np.int64)
    if B == 0 or npoint == 0:
        return out

    def job(b):
        return lambda: lib.oracle_fps(_ptr(xyz[b], _f32p), 1, N, npoint, start_idx,
                                      int(skip_near_origin), _ptr(out[b], _i64p))
    _parallel(job(b) for b in range(B))
    return out


# ---------------------------------------------------------------- kNN
def knn(query, ref, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Exact (SD, index) kNN: tests/test_knn.py:15-23, tests/test_feature_knn.py:16-35.

    Returns Euclidean distances (B,M,k) float32 and indices (B,M,k) int64.
    """
    lib = _load()
    query, ref = _f32(query), _f32(ref)
    B, M, D = query.shape
    N = ref.shape[1]
    dist = np.empty((B, M, k), dtype=np.float32)
    idx = np.empty((B, M, k), dtype=np.int64)
    if B == 0 or M == 0 or k == 0:
        return dist, idx
    jobs = []
    parts = max(1, threads() * 4 // max(1, B))
    for b in range(B):
        for lo, hi in _ranges(M, parts):
            def job(b=b, lo=lo, hi=hi):
                lib.oracle_knn(_ptr(query[b, lo:hi], _f32p), _ptr(ref[b], _f32p), 1, hi - lo, N,
                               D, k, _ptr(dist[b, lo:hi], _f32p), _ptr(idx[b, lo:hi], _i64p))
            jobs.append(job)
    _parallel(jobs)
    return dist, idx


def knn_sqdist(query, ref, idx) -> np.ndarray:
    """Squared distances of selected neighbours (inf for index -1)."""
    lib = _load()
    query, ref, idx = _f32(query), _f32(ref), _i64a(idx)
    B, M, D = query.shape
    out = np.empty(idx.shape, dtype=np.float32)
    lib.oracle_knn_sqdist(_ptr(query, _f32p), _ptr(ref, _f32p), B, M, ref.shape[1], D,
                          idx.shape[-1], _ptr(idx, _i64p), _ptr(out, _f32p))
    return out


# ---------------------------------------------------------------- ball query
def radius_squared(radius: float) -> float:
    """fl32(fl32(r) * fl32(r)) (mps_pointops/_ball_query_mps.py:104-119)."""
    r32 = np.float32(radius)
    with np.errstate(over="ignore"):
        return float(np.float32(r32 * r32))


def ball_query(query, ref, radius: float, K: int, query_lengths=None,
               point_lengths=None) -> tuple[np.ndarray, np.ndarray]:
    """mps_pointops/reference.py:83-121 (+ lengths, _ball_query_mps.py:73-84)."""
    lib = _load()
    query, ref = _f32(query), _f32(ref)
    ql, pl = _i64a(query_lengths), _i64a(point_lengths)
    B, M, _ = query.shape
    N = ref.shape[1]
    r2 = radius_squared(radius)
    dist2 = np.zeros((B, M, K), dtype=np.float32)
    idx = np.full((B, M, K), -1, dtype=np.int64)
    if B == 0 or M == 0 or K == 0:
        return dist2, idx
    jobs = []
    parts = max(1, threads() * 4 // max(1, B))
    for b in range(B):
        for lo, hi in _ranges(M, parts):
            def job(b=b, lo=lo, hi=hi):
                qlb = None if ql is None else np.array([max(0, min(hi, ql[b]) - lo)], np.int64)
                plb = None if pl is None else pl[b:b + 1].copy()
                lib.oracle_ball_query(_ptr(query[b, lo:hi], _f32p), _ptr(ref[b], _f32p),
                                      _ptr(qlb, _i64p), _ptr(plb, _i64p), 1, hi - lo, N, K,
                                      ctypes.c_float(r2), _ptr(dist2[b, lo:hi], _f32p),
                                      _ptr(idx[b, lo:hi], _i64p))
            jobs.append(job)
    _parallel(jobs)
    return dist2, idx


def ball_query_pointnet2(radius: float, nsample: int, xyz, new_xyz) -> np.ndarray:
    """mps_pointops/compat.py:76-85: misses repeat the first hit (0 if none), int32."""
    _, idx = ball_query(new_xyz, xyz, radius, nsample)
    first = np.maximum(idx[..., :1], 0)
    return np.where(idx >= 0, idx, first).astype(np.int32)


# ---------------------------------------------------------------- three_nn / interpolate
def three_nn(unknown, known) -> tuple[np.ndarray, np.ndarray]:
    """mps_pointops/pointnet2.py:54-72.  Euclidean distances, int32 indices."""
    lib = _load()
    unknown, known = _f32(unknown), _f32(known)
    B, N, _ = unknown.shape
    M = known.shape[1]
    dist = np.empty((B, N, 3), dtype=np.float32)
    idx = np.empty((B, N, 3), dtype=np.int32)
    if B == 0 or N == 0:
        return dist, idx
    jobs = []
    parts = max(1, threads() * 4 // max(1, B))
    for b in range(B):
        for lo, hi in _ranges(N, parts):
            def job(b=b, lo=lo, hi=hi):
                lib.oracle_three_nn(_ptr(unknown[b, lo:hi], _f32p), _ptr(known[b], _f32p), 1,
                                    hi - lo, M, _ptr(dist[b, lo:hi], _f32p),
                                    _ptr(idx[b, lo:hi], _i32p))
            jobs.append(job)
    _parallel(jobs)
    return dist, idx


def three_interpolate(features, indices, weights) -> np.ndarray:
    """mps_pointops/pointnet2.py:135-147."""
    lib = _load()
    features, weights = _f32(features), _f32(weights)
    indices = _i64a(indices)
    B, C, M = features.shape
    N = indices.shape[1]
    out = np.empty((B, C, N), dtype=np.float32)
    lib.oracle_three_interpolate(_ptr(features, _f32p), _ptr(indices, _i64p),
                                 _ptr(weights, _f32p), B, C, M, N, _ptr(out, _f32p))
    return out


def three_interpolate_backward(grad_out, indices, weights, M: int) -> np.ndarray:
    """mps_pointops/pointnet2.py:168-188 (feature gradient; weight grad is zero)."""
    lib = _load()
    grad_out, weights = _f32(grad_out), _f32(weights)
    indices = _i64a(indices)
    B, C, N = grad_out.shape
    out = np.empty((B, C, M), dtype=np.float32)
    lib.oracle_three_interpolate_backward(_ptr(grad_out, _f32p), _ptr(indices, _i64p),
                                          _ptr(weights, _f32p), B, C, M, N, _ptr(out, _f32p))
    return out


# ---------------------------------------------------------------- Chamfer
def chamfer_nearest(query, ref, query_lengths=None, ref_lengths=None, norm: int = 2):
    """mps_pointops/chamfer.py:161-212 + 297-320: first-minimum index and its
    distance (SD for norm 2, L1 for norm 1)."""
    lib = _load()
    fn = lib.oracle_chamfer_nearest_l1 if norm == 1 else lib.oracle_chamfer_nearest
    query, ref = _f32(query), _f32(ref)
    ql, rl = _i64a(query_lengths), _i64a(ref_lengths)
    B, P, D = query.shape
    Q = ref.shape[1]
    dist = np.empty((B, P), dtype=np.float32)
    idx = np.empty((B, P), dtype=np.int64)
    if B == 0 or P == 0:
        return dist, idx
    jobs = []
    parts = max(1, threads() * 4 // max(1, B))
    for b in range(B):
        for lo, hi in _ranges(P, parts):
            def job(b=b, lo=lo, hi=hi):
                qlb = None if ql is None else np.array([max(0, min(hi, ql[b]) - lo)], np.int64)
                rlb = None if rl is None else rl[b:b + 1].copy()
                fn(_ptr(query[b, lo:hi], _f32p), _ptr(ref[b], _f32p), _ptr(qlb, _i64p),
                   _ptr(rlb, _i64p), 1, hi - lo, Q, D, _ptr(dist[b, lo:hi], _f32p),
                   _ptr(idx[b, lo:hi], _i64p))
            jobs.append(job)
    _parallel(jobs)
    return dist, idx


def chamfer_mean_loss_and_grad(x, y, x_lengths=None, y_lengths=None):
    """Squared-L2 Chamfer, mean/mean reductions, loss and both gradients (float64 sums).

    mps_pointops/chamfer.py:342-488 (forward) and :215-251 (backward).
    Returns (loss, grad_x, grad_y, (dist_x, idx_x), (dist_y, idx_y)).
    """
    lib = _load()
    x, y = _f32(x), _f32(y)
    lx, ly = _i64a(x_lengths), _i64a(y_lengths)
    dx, ix = chamfer_nearest(x, y, lx, ly)
    dy, iy = chamfer_nearest(y, x, ly, lx)
    B, P, D = x.shape
    Q = y.shape[1]
    gx = np.empty_like(x)
    gy = np.empty_like(y)
    loss = lib.oracle_chamfer_mean_loss_and_grad(
        _ptr(x, _f32p), _ptr(y, _f32p), _ptr(lx, _i64p), _ptr(ly, _i64p), B, P, Q, D,
        _ptr(ix, _i64p), _ptr(iy, _i64p), _ptr(dx, _f32p), _ptr(dy, _f32p),
        _ptr(gx, _f32p), _ptr(gy, _f32p))
    return loss, gx, gy, (dx, ix), (dy, iy)


def chamfer_l1_grads(x, y, ix, iy, gdx, gdy):
    """Gradient of the selected L1 distances (mps_pointops/chamfer.py:269-293):
    g = s * gd with s = +1 where q > r and -1 otherwise, added to the query and
    subtracted from the selected reference (float64 sums)."""
    x, y = np.asarray(x, np.float64), np.asarray(y, np.float64)
    gx, gy = np.zeros_like(x), np.zeros_like(y)
    for q, r, idx, gd, gq, gr in ((x, y, ix, gdx, gx, gy), (y, x, iy, gdy, gy, gx)):
        if gd is None:
            continue
        for b in range(q.shape[0]):
            for i in range(q.shape[1]):
                j = idx[b, i]
                if j < 0:
                    continue
                g = np.where(q[b, i] > r[b, j], 1.0, -1.0) * float(gd[b, i])
                gq[b, i] += g
                gr[b, j] -= g
    return gx, gy


# ---------------------------------------------------------------- flat batches
def flat_sample_counts(lengths, ratio: float, ratio_dtype=np.float32) -> list[int]:
    """torch_cluster's GPU count rule (mps_pointops/flat.py:150-158): the batch
    sizes are converted to the ratio's dtype, multiplied, ceiled."""
    sizes = np.asarray(lengths, dtype=ratio_dtype)
    return [int(v) for v in np.ceil(sizes * ratio_dtype(ratio))]


def torch_cluster_radius_sq(r: float) -> float:
    """fl32(r * r) with r * r in double (mps_pointops/_flat_search_mps.py:66-76)."""
    with np.errstate(over="ignore"):
        return float(np.float32(r * r))


def _flat_search(x, y, ptr_x, ptr_y, width, radius_mode, r2=0.0, ignore_same=False):
    lib = _load()
    x, y = _f32(x), _f32(y)
    px, py = _i64a(ptr_x), _i64a(ptr_y)
    if y.ndim == 1:
        y = y.reshape(-1, 1)
    D = y.shape[1]
    ny = y.shape[0]
    out = np.full((ny, width), -1, dtype=np.int64)
    if ny == 0 or width == 0:
        return out
    xx = x if x.size else np.zeros((1, D), np.float32)
    jobs = []
    for lo, hi in _ranges(ny, threads() * 4):
        def job(lo=lo, hi=hi):
            lib.oracle_flat_search(_ptr(xx, _f32p), _ptr(y, _f32p), _ptr(px, _i64p),
                                   _ptr(py, _i64p), len(px) - 1, D, width, int(radius_mode),
                                   ctypes.c_float(r2), int(bool(ignore_same)), lo, hi,
                                   _ptr(out, _i64p))
        jobs.append(job)
    _parallel(jobs)
    return out


def flat_knn_indices(x, y, ptr_x, ptr_y, width: int) -> np.ndarray:
    """mps_pointops/flat.py:264-288, kNN branch: (ny, width) global x rows in
    ascending (SD, index) order over the query's cloud, non-finite SD dropped,
    -1 padded."""
    return _flat_search(x, y, ptr_x, ptr_y, width, False)


def flat_radius_indices(x, y, ptr_x, ptr_y, r: float, width: int,
                        ignore_same_index: bool = False) -> np.ndarray:
    """mps_pointops/flat.py:264-288, radius branch: the first `width` global x
    rows of the query's cloud in input order with SD < fl32(r * r)."""
    return _flat_search(x, y, ptr_x, ptr_y, width, True, torch_cluster_radius_sq(r),
                        ignore_same_index)


def flat_fps(x, ptr, counts, starts) -> np.ndarray:
    """mps_pointops/flat.py:208-217: per cloud, reference.furthest_point_sample
    from the local index starts[b] (reference.py:27-58), shifted to global rows."""
    lib = _load()
    x = _f32(x)
    ptr = [int(v) for v in ptr]
    counts = [int(c) for c in counts]
    outs = [np.empty(c, dtype=np.int64) for c in counts]

    def job(b):
        def run():
            lo, hi = ptr[b], ptr[b + 1]
            if counts[b] == 0:
                return
            seg = np.ascontiguousarray(x[lo:hi])
            lib.oracle_fps(_ptr(seg, _f32p), 1, hi - lo, counts[b], int(starts[b]), 0,
                           _ptr(outs[b], _i64p))
            outs[b] += lo
        return run
    _parallel(job(b) for b in range(len(counts)))
    return np.concatenate(outs) if outs else np.empty(0, dtype=np.int64)


def pointcept_fps(xyz, offset, new_offset) -> np.ndarray:
    """mps_pointops/pointcept.py:77-98: per batch (cumulative ends `offset`,
    sample ends `new_offset`), FPS from the batch's first point
    (reference.py:27-58), as global int32 rows."""
    ptr = [0, *[int(v) for v in offset]]
    tgt = [0, *[int(v) for v in new_offset]]
    counts = [b - a for a, b in zip(tgt, tgt[1:])]
    return flat_fps(xyz, ptr, counts, [0] * len(counts)).astype(np.int32)


def pointcept_knn(nsample: int, xyz, offset, new_xyz=None, new_offset=None):
    """mps_pointops/pointcept.py:101-165: per query, the nsample nearest rows
    of its batch in ascending (SD, index) order; a slot is kept only when the
    SD recomputed from the selected rows, ((dx*dx + dy*dy) + dz*dz), is
    finite and below 1e10, otherwise it holds (-1, 1e5).  Returns (int32
    global indices, float32 Euclidean distances)."""
    xyz = _f32(xyz)
    if new_xyz is None:
        new_xyz, new_offset = xyz, offset
    new_xyz = _f32(new_xyz)
    ptr_x = np.array([0, *[int(v) for v in offset]], dtype=np.int64)
    ptr_y = np.array([0, *[int(v) for v in new_offset]], dtype=np.int64)
    idx = flat_knn_indices(xyz, new_xyz, ptr_x, ptr_y, nsample)
    sel = idx >= 0
    rows = xyz[np.where(sel, idx, 0)] if len(xyz) else np.zeros(idx.shape + (3,), np.float32)
    delta = new_xyz[:, None, :] - rows
    with np.errstate(invalid="ignore", over="ignore"):
        sq = delta[..., 0] * delta[..., 0]
        sq = sq + delta[..., 1] * delta[..., 1]
        sq = sq + delta[..., 2] * delta[..., 2]
        valid = sel & (sq < np.float32(1e10))
        dist = np.where(valid, np.sqrt(sq), np.float32(1e5)).astype(np.float32)
    return np.where(valid, idx, -1).astype(np.int32), dist


def flat_edges(indices: np.ndarray) -> np.ndarray:
    """mps_pointops/flat.py:247-253: padded rows -> [query, reference] edges."""
    q, s = np.nonzero(indices >= 0)
    return np.stack([q.astype(np.int64), indices[q, s]])


# ---------------------------------------------------------------- SA grouping
def group_points(features, idx) -> np.ndarray:
    """mps_pointops/compat.py:68-73 (torch gather): out[b, c, p, s] =
    features[b, c, idx[b, p, s]] -- exact copies.  gather_operation
    (compat.py:62-65) is the nsample = 1 case."""
    features = _f32(features)
    idx = np.asarray(idx).astype(np.int64)
    return np.stack([features[b][:, idx[b]] for b in range(features.shape[0])])


def group_points_backward(grad_out, idx, n: int) -> np.ndarray:
    """Gradient of group_points: scatter-add of grad_out over idx, accumulated
    in float64 (the tests compare within a relative tolerance, as the order of
    float32 additions into one element is not fixed on either side)."""
    grad_out = np.asarray(grad_out, dtype=np.float64)
    idx = np.asarray(idx).astype(np.int64)
    B, C = grad_out.shape[:2]
    out = np.zeros((B, C, n), dtype=np.float64)
    for b in range(B):
        np.add.at(out[b], (slice(None), idx[b].reshape(-1)), grad_out[b].reshape(C, -1))
    return out


def query_and_group(xyz, new_xyz, features, radius: float, nsample: int, use_xyz=True):
    """tests/test_pointnet2_e2e.py:40-44: pointnet2 ball query, grouped xyz
    minus the centre (one float32 subtraction), grouped features, concatenated
    along channels.  Returns (out, idx int32)."""
    xyz, new_xyz = _f32(xyz), _f32(new_xyz)
    idx = ball_query_pointnet2(radius, nsample, xyz, new_xyz)
    parts = []
    if use_xyz:
        gx = group_points(np.ascontiguousarray(xyz.transpose(0, 2, 1)), idx)
        parts.append((gx - new_xyz.transpose(0, 2, 1)[..., None]).astype(np.float32))
    if features is not None:
        parts.append(group_points(features, idx))
    return np.concatenate(parts, axis=1), idx


def query_and_group_backward(grad_out, idx, n: int, use_xyz=True):
    """Gradients of query_and_group for (xyz, new_xyz, features), float64."""
    g = np.asarray(grad_out, dtype=np.float64)
    X = 3 if use_xyz else 0
    gxyz = group_points_backward(g[:, :X], idx, n).transpose(0, 2, 1) if X else None
    gnew = -g[:, :X].sum(axis=3).transpose(0, 2, 1) if X else None
    gfeat = group_points_backward(g[:, X:], idx, n) if g.shape[1] > X else None
    return gxyz, gnew, gfeat
