/*
 * CPU oracle for the mps_pointops hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the CPU algorithms of the reference package
 * gamzerA/mps-pointops v1.0.0 (paths below are relative to that project).  It
 * is the checker for the CUDA kernels: only the test suite, the smoke check
 * and the CPU-baseline leg of the benchmark load it.  The product library
 * never links or calls it.
 *
 * Arithmetic contract (every function): IEEE binary32, each add/sub/mul
 * rounded separately.  The build uses -ffp-contract=off and no fast-math so
 * the compiler can neither fuse a multiply-add nor reassociate a sum.
 *
 *   squared distance, D == 3 : ((d0*d0 + d1*d1) + d2*d2), d = a - b
 *                              (mps_pointops/reference.py:21-24)
 *   squared distance, D != 3 : s = d0*d0; s = s + dt*dt for t = 1..D-1
 *                              (mps_pointops/chamfer.py:199-201,
 *                               tests/test_feature_knn.py:16-35)
 *
 * Both orders give the same bits for D == 3, so one helper serves both.
 * Every function is single-threaded; the Python wrapper (oracle/oracle.py)
 * runs independent clouds or query ranges on several host threads, which
 * never changes the order of any accumulation that is compared bit-for-bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>


#define EXPORT __attribute__((visibility("default")))

static inline float sqdist(const float* a, const float* b, int64_t D) {
    float d = a[0] - b[0];
    float s = d * d;
    for (int64_t t = 1; t < D; ++t) {
        d = a[t] - b[t];
        float p = d * d;
        s = s + p;
    }
    return s;
}

EXPORT int oracle_version(void) { return 1; }

/* ------------------------------------------------------------------ FPS
 * mps_pointops/reference.py:27-58 (furthest_point_sample).
 *   min_d2 starts at +inf; with skip_near_origin the points whose
 *   ((x*x + y*y) + z*z) < fl32(1e-3) start at -inf (reference.py:46-50).
 *   Step i: out[i] = farthest; min_d2 = torch.minimum(min_d2, sqdist(xyz,
 *   xyz[farthest])) (NaN propagates); farthest = argmax(min_d2) -- the
 *   first maximum, where torch's argmax ranks NaN above every number and
 *   takes the first NaN.
 */
static inline int fps_greater(float a, float b) {
    /* "a ranks strictly above b" under torch.argmax's NaN-is-max order. */
    if (isnan(b)) return 0;
    if (isnan(a)) return 1;
    return a > b;
}

EXPORT void oracle_fps(const float* xyz, int64_t B, int64_t N, int64_t npoint,
                       int64_t start_idx, int skip_near_origin, int64_t* out) {
    for (int64_t b = 0; b < B; ++b) {
        const float* p = xyz + b * N * 3;
        float* md = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
        const float zero[3] = {0.f, 0.f, 0.f};
        for (int64_t j = 0; j < N; ++j) {
            md[j] = INFINITY;
            if (skip_near_origin && sqdist(p + 3 * j, zero, 3) < 1e-3f) md[j] = -INFINITY;
        }
        int64_t far = start_idx;
        for (int64_t i = 0; i < npoint; ++i) {
            out[b * npoint + i] = far;
            const float* c = p + 3 * far;
            int64_t best = 0;
            for (int64_t j = 0; j < N; ++j) {
                float d = sqdist(p + 3 * j, c, 3);
                float m = md[j];
                float v = (isnan(m) || isnan(d)) ? NAN : (d < m ? d : m);
                md[j] = v;
                if (j == 0 || fps_greater(v, md[best])) best = j;
            }
            far = best;
        }
        free(md);
    }
}

/* ------------------------------------------------------------------ kNN
 * Exact (squared distance, index) order: the oracles of
 * tests/test_knn.py:15-23 (D == 3, numpy lexsort), bench/bench_pointops.py:138-159
 * and tests/test_feature_knn.py:16-35 (D != 3, scalar loop).  Public output
 * contract of mps_pointops/ops.py:144-205: Euclidean distance = sqrt(SD)
 * taken after selection, int64 indices.
 * Non-finite candidates: D == 3 drops NaN and ranks +inf like a number
 * (kernels/knn.metal:27-31 ordering); D != 3 drops every non-finite SD
 * (kernels/feature_knn.metal:10, docs/feature-knn.md:40-47).  Unfilled slots
 * are (inf, -1).
 */
static inline int knn_before(float d, int64_t i, float e, int64_t j) {
    return d < e || (d == e && i < j);
}

EXPORT void oracle_knn(const float* query, const float* ref, int64_t B, int64_t M,
                       int64_t N, int64_t D, int64_t k, float* dist, int64_t* idx) {
    if (k <= 0) return;
    {
        float* ld = (float*)malloc(sizeof(float) * (size_t)k);
        int64_t* li = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
        for (int64_t b = 0; b < B; ++b) {
            for (int64_t q = 0; q < M; ++q) {
                const float* qp = query + (b * M + q) * D;
                const float* rp = ref + b * N * D;
                int64_t filled = 0;
                for (int64_t j = 0; j < N; ++j) {
                    float d = sqdist(qp, rp + j * D, D);
                    if (isnan(d)) continue;
                    if (D != 3 && !isfinite(d)) continue;
                    if (filled == k && !knn_before(d, j, ld[k - 1], li[k - 1])) continue;
                    int64_t pos = filled < k ? filled : k - 1;
                    while (pos > 0 && knn_before(d, j, ld[pos - 1], li[pos - 1])) {
                        ld[pos] = ld[pos - 1];
                        li[pos] = li[pos - 1];
                        --pos;
                    }
                    ld[pos] = d;
                    li[pos] = j;
                    if (filled < k) ++filled;
                }
                float* od = dist + (b * M + q) * k;
                int64_t* oi = idx + (b * M + q) * k;
                for (int64_t s = 0; s < k; ++s) {
                    if (s < filled) {
                        od[s] = sqrtf(ld[s]);
                        oi[s] = li[s];
                    } else {
                        od[s] = INFINITY;
                        oi[s] = -1;
                    }
                }
            }
        }
        free(ld);
        free(li);
    }
}

/* Squared distances of the selected neighbours, before the square root. */
EXPORT void oracle_knn_sqdist(const float* query, const float* ref, int64_t B, int64_t M,
                              int64_t N, int64_t D, int64_t k, const int64_t* idx,
                              float* sd) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t q = 0; q < M; ++q)
            for (int64_t s = 0; s < k; ++s) {
                int64_t j = idx[(b * M + q) * k + s];
                sd[(b * M + q) * k + s] =
                    j < 0 ? INFINITY : sqdist(query + (b * M + q) * D, ref + (b * N + j) * D, D);
            }
}

/* ------------------------------------------------------------------ ball query
 * mps_pointops/reference.py:83-121: the first K reference points in input
 * order with SD < r2 (strict), r2 = fl32(fl32(r)*fl32(r)) computed by the
 * caller (mps_pointops/_ball_query_mps.py:87-119).  Empty slots: index -1,
 * distance 0.  Optional per-cloud lengths follow _ball_query_mps.py:73-84 and
 * tests/test_ball_query_mps.py:16-51: queries at or beyond query_lengths[b]
 * are all padding; references at or beyond point_lengths[b] never match.
 * A non-finite coordinate gives a NaN or +inf SD, which fails the strict
 * compare, so it never matches (reference.py:115-116).
 */
EXPORT void oracle_ball_query(const float* query, const float* ref,
                              const int64_t* query_lengths, const int64_t* point_lengths,
                              int64_t B, int64_t M, int64_t N, int64_t K, float r2,
                              float* dist2, int64_t* idx) {
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t q = 0; q < M; ++q) {
            float* od = dist2 + (b * M + q) * K;
            int64_t* oi = idx + (b * M + q) * K;
            for (int64_t s = 0; s < K; ++s) {
                od[s] = 0.f;
                oi[s] = -1;
            }
            int64_t ql = query_lengths ? query_lengths[b] : M;
            int64_t pl = point_lengths ? point_lengths[b] : N;
            if (q >= ql) continue;
            const float* qp = query + (b * M + q) * 3;
            int64_t found = 0;
            for (int64_t j = 0; j < pl && found < K; ++j) {
                float d = sqdist(qp, ref + (b * N + j) * 3, 3);
                if (d < r2) {
                    od[found] = d;
                    oi[found] = j;
                    ++found;
                }
            }
        }
    }
}

/* ------------------------------------------------------------------ three_nn
 * mps_pointops/pointnet2.py:54-72 (_three_nn_reference): stable argsort of
 * SD, first three; Euclidean distance = sqrt after selection; int32 index.
 * torch's stable argsort places NaN after every number, in index order.
 */
static inline int tnn_before(float d, int64_t i, float e, int64_t j) {
    int dn = isnan(d), en = isnan(e);
    if (dn != en) return en;          /* a number precedes NaN */
    if (dn) return i < j;             /* NaN vs NaN: index order */
    return d < e || (d == e && i < j);
}

EXPORT void oracle_three_nn(const float* unknown, const float* known, int64_t B,
                            int64_t N, int64_t M, float* dist, int32_t* idx) {
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t n = 0; n < N; ++n) {
            const float* qp = unknown + (b * N + n) * 3;
            float bd[3];
            int64_t bi[3];
            int filled = 0;
            for (int64_t j = 0; j < M; ++j) {
                float d = sqdist(qp, known + (b * M + j) * 3, 3);
                if (filled == 3 && !tnn_before(d, j, bd[2], bi[2])) continue;
                int pos = filled < 3 ? filled : 2;
                while (pos > 0 && tnn_before(d, j, bd[pos - 1], bi[pos - 1])) {
                    bd[pos] = bd[pos - 1];
                    bi[pos] = bi[pos - 1];
                    --pos;
                }
                bd[pos] = d;
                bi[pos] = j;
                if (filled < 3) ++filled;
            }
            for (int t = 0; t < 3; ++t) {
                dist[(b * N + n) * 3 + t] = sqrtf(bd[t]);
                idx[(b * N + n) * 3 + t] = (int32_t)bi[t];
            }
        }
    }
}

/* ------------------------------------------------------------------ three_interpolate
 * mps_pointops/pointnet2.py:135-147 (_three_interpolate_reference):
 * out[b,c,n] = ((f0*w0 + f1*w1) + f2*w2), each product rounded, summed in
 * order (torch's sum over a contiguous length-3 axis is sequential).
 * Backward (pointnet2.py:168-188): grad_f[b,c,I[b,n,t]] += g[b,c,n]*W[b,n,t],
 * accumulated in (n, t) order per (b, c).
 */
EXPORT void oracle_three_interpolate(const float* features, const int64_t* indices,
                                     const float* weights, int64_t B, int64_t C, int64_t M,
                                     int64_t N, float* out) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t c = 0; c < C; ++c)
            for (int64_t n = 0; n < N; ++n) {
                const int64_t* I = indices + (b * N + n) * 3;
                const float* W = weights + (b * N + n) * 3;
                const float* F = features + (b * C + c) * M;
                float p0 = F[I[0]] * W[0];
                float p1 = F[I[1]] * W[1];
                float p2 = F[I[2]] * W[2];
                float s = p0 + p1;
                s = s + p2;
                out[(b * C + c) * N + n] = s;
            }
}

EXPORT void oracle_three_interpolate_backward(const float* grad_out, const int64_t* indices,
                                              const float* weights, int64_t B, int64_t C,
                                              int64_t M, int64_t N, float* grad_features) {
    memset(grad_features, 0, sizeof(float) * (size_t)(B * C * M));
    for (int64_t b = 0; b < B; ++b)
        for (int64_t c = 0; c < C; ++c)
            for (int64_t n = 0; n < N; ++n)
                for (int t = 0; t < 3; ++t) {
                    int64_t i = indices[(b * N + n) * 3 + t];
                    float g = grad_out[(b * C + c) * N + n] * weights[(b * N + n) * 3 + t];
                    grad_features[(b * C + c) * M + i] += g;
                }
}

/* ------------------------------------------------------------------ Chamfer nearest
 * mps_pointops/chamfer.py:161-212 (_nearest_indices, norm=2): for every
 * query the FIRST reference index among the valid ones (index < ref_lengths[b])
 * with the smallest SD; the first valid reference is taken unconditionally,
 * so a row whose every SD overflows to +inf still selects reference 0
 * (chamfer.py:205-209).  A cloud with no valid reference gives -1.
 * Distance: chamfer.py:297-308 (_selected_squared_distance) -- the SD of the
 * selected pair, 0 for padded query rows and for index -1.  Padded query rows
 * (q >= query_lengths[b]) report index -1, the convention of the native
 * nearest kernels (kernels/chamfer_nn.metal:35-39); the CPU path masks them
 * out of every later step, so this choice is not observable through the API.
 */
EXPORT void oracle_chamfer_nearest(const float* query, const float* ref,
                                   const int64_t* query_lengths, const int64_t* ref_lengths,
                                   int64_t B, int64_t P, int64_t Q, int64_t D,
                                   float* dist, int64_t* idx) {
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t i = 0; i < P; ++i) {
            int64_t ql = query_lengths ? query_lengths[b] : P;
            int64_t rl = ref_lengths ? ref_lengths[b] : Q;
            int64_t best = -1;
            float bd = INFINITY;
            if (i < ql) {
                const float* qp = query + (b * P + i) * D;
                for (int64_t j = 0; j < rl; ++j) {
                    float d = sqdist(qp, ref + (b * Q + j) * D, D);
                    if (best < 0 || d < bd) {
                        bd = d;
                        best = j;
                    }
                }
            }
            idx[b * P + i] = best;
            dist[b * P + i] = best < 0 ? 0.f : bd;
        }
    }
}

/* L1 variant (mps_pointops/chamfer.py:161-212 with norm == 1; distance of the
 * selected pair: _selected_l1_distance, chamfer.py:310-320): |d0| + |d1| + ...
 * in dimension order, d = query - ref, each operation rounded on its own;
 * the same first-minimum and padding rules as oracle_chamfer_nearest. */
static inline float l1dist(const float* a, const float* b, int64_t D) {
    float s = fabsf(a[0] - b[0]);
    for (int64_t t = 1; t < D; ++t) {
        float d = fabsf(a[t] - b[t]);
        s = s + d;
    }
    return s;
}

EXPORT void oracle_chamfer_nearest_l1(const float* query, const float* ref,
                                      const int64_t* query_lengths, const int64_t* ref_lengths,
                                      int64_t B, int64_t P, int64_t Q, int64_t D,
                                      float* dist, int64_t* idx) {
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t i = 0; i < P; ++i) {
            int64_t ql = query_lengths ? query_lengths[b] : P;
            int64_t rl = ref_lengths ? ref_lengths[b] : Q;
            int64_t best = -1;
            float bd = INFINITY;
            if (i < ql) {
                const float* qp = query + (b * P + i) * D;
                for (int64_t j = 0; j < rl; ++j) {
                    float d = l1dist(qp, ref + (b * Q + j) * D, D);
                    if (best < 0 || d < bd) {
                        bd = d;
                        best = j;
                    }
                }
            }
            idx[b * P + i] = best;
            dist[b * P + i] = best < 0 ? 0.f : bd;
        }
    }
}

/* Chamfer squared-L2 loss with point_reduction="mean", batch_reduction="mean"
 * and its gradients, accumulated in binary64 (chamfer.py:342-488 forward,
 * chamfer.py:215-251 backward).  loss = (1/B) sum_b (sum_i dx_i / Px_b +
 * sum_j dy_j / Py_b); grad_x_i = 2 (x_i - y_a(i)) g_x + sum_{j: b(j)=i}
 * 2 (x_i - y_j) g_y with g_x = 1/(B Px_b), g_y = 1/(B Py_b).
 */
EXPORT double oracle_chamfer_mean_loss_and_grad(
    const float* x, const float* y, const int64_t* x_lengths, const int64_t* y_lengths,
    int64_t B, int64_t P, int64_t Q, int64_t D, const int64_t* idx_x, const int64_t* idx_y,
    const float* dist_x, const float* dist_y, float* grad_x, float* grad_y) {
    double loss = 0.0;
    double* gx = (double*)calloc((size_t)(B * P * D > 0 ? B * P * D : 1), sizeof(double));
    double* gy = (double*)calloc((size_t)(B * Q * D > 0 ? B * Q * D : 1), sizeof(double));
    double denom_b = (double)(B > 0 ? B : 1);
    for (int64_t b = 0; b < B; ++b) {
        int64_t px = x_lengths ? x_lengths[b] : P;
        int64_t qy = y_lengths ? y_lengths[b] : Q;
        double sx = 0.0, sy = 0.0;
        double cx = 1.0 / ((double)(px > 0 ? px : 1) * denom_b);
        double cy = 1.0 / ((double)(qy > 0 ? qy : 1) * denom_b);
        for (int64_t i = 0; i < px; ++i) {
            int64_t j = idx_x[b * P + i];
            if (j < 0) continue;
            sx += dist_x[b * P + i];
            for (int64_t t = 0; t < D; ++t) {
                double g = 2.0 * ((double)x[(b * P + i) * D + t] - (double)y[(b * Q + j) * D + t]) * cx;
                gx[(b * P + i) * D + t] += g;
                gy[(b * Q + j) * D + t] -= g;
            }
        }
        for (int64_t j = 0; j < qy; ++j) {
            int64_t i = idx_y[b * Q + j];
            if (i < 0) continue;
            sy += dist_y[b * Q + j];
            for (int64_t t = 0; t < D; ++t) {
                double g = 2.0 * ((double)y[(b * Q + j) * D + t] - (double)x[(b * P + i) * D + t]) * cy;
                gy[(b * Q + j) * D + t] += g;
                gx[(b * P + i) * D + t] -= g;
            }
        }
        loss += sx / (double)(px > 0 ? px : 1) + sy / (double)(qy > 0 ? qy : 1);
    }
    for (int64_t e = 0; e < B * P * D; ++e) grad_x[e] = (float)gx[e];
    for (int64_t e = 0; e < B * Q * D; ++e) grad_y[e] = (float)gy[e];
    free(gx);
    free(gy);
    return loss / denom_b;
}

/* ------------------------------------------------------------------ flat batches
 * mps_pointops/flat.py:256-288 (_sqdist, _reference_search): the CPU path of
 * the torch_cluster-style flat API.  x (nx, D) reference rows and y (ny, D)
 * query rows are split into `segs` clouds by the offset arrays ptr_x and
 * ptr_y (segs + 1 entries, flat.py:67-97).  For every query row q of cloud b
 * the row out[q, :width] receives GLOBAL x rows, -1 padded:
 *   kNN    (radius_mode 0): torch.argsort(d2, stable=True) over the cloud,
 *          keep the finite d2 (torch.isfinite), first min(width, cloud size)
 *          -- the ascending (d2, index) order without non-finite entries.
 *   radius (radius_mode 1): torch.nonzero(d2 < r2)[:take] -- the first rows
 *          in input order with d2 < r2, r2 = fl32(r * r), r * r in double
 *          (flat.py:272, 286; mps_pointops/_flat_search_mps.py:66-76).  With
 *          ignore_same != 0 the x row whose global number equals q's is
 *          skipped before the cap (pyg-lib's radius, flat_search.metal:199).
 * d2 = _sqdist(y[q], x[j]) = sequential sum of (x - y)^2, each op rounded.
 * Only the query rows in [q_lo, q_hi) are written, so host threads can split
 * the queries without changing any result. */
EXPORT void oracle_flat_search(const float* x, const float* y, const int64_t* ptr_x,
                               const int64_t* ptr_y, int64_t segs, int64_t D, int64_t width,
                               int radius_mode, float r2, int ignore_same, int64_t q_lo,
                               int64_t q_hi, int64_t* out) {
    float* ld = (float*)malloc(sizeof(float) * (size_t)(width > 0 ? width : 1));
    int64_t* li = (int64_t*)malloc(sizeof(int64_t) * (size_t)(width > 0 ? width : 1));
    for (int64_t b = 0; b < segs; ++b) {
        const int64_t xa = ptr_x[b], xb = ptr_x[b + 1];
        const int64_t ya = ptr_y[b] > q_lo ? ptr_y[b] : q_lo;
        const int64_t yb = ptr_y[b + 1] < q_hi ? ptr_y[b + 1] : q_hi;
        const int64_t take = width < xb - xa ? width : xb - xa;
        for (int64_t q = ya; q < yb; ++q) {
            int64_t* row = out + q * width;
            int64_t filled = 0;
            for (int64_t s = 0; s < width; ++s) row[s] = -1;
            if (take <= 0) continue;
            for (int64_t j = 0; j < xb - xa; ++j) {
                const float d = sqdist(y + q * D, x + (xa + j) * D, D);
                if (radius_mode) {
                    if (filled == take) break;
                    if (ignore_same && xa + j == q) continue;
                    if (d < r2) row[filled++] = xa + j;
                    continue;
                }
                if (!isfinite(d)) continue;
                if (filled == take && !knn_before(d, j, ld[take - 1], li[take - 1])) continue;
                int64_t pos = filled < take ? filled : take - 1;
                while (pos > 0 && knn_before(d, j, ld[pos - 1], li[pos - 1])) {
                    ld[pos] = ld[pos - 1];
                    li[pos] = li[pos - 1];
                    --pos;
                }
                ld[pos] = d;
                li[pos] = j;
                if (filled < take) ++filled;
            }
            if (!radius_mode)
                for (int64_t s = 0; s < filled; ++s) row[s] = xa + li[s];
        }
    }
    free(ld);
    free(li);
}
