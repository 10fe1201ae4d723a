// Grid-accelerated exact search over one point cloud: the B200 counterpart of
// the reference's opt-in spatial index (gamzerA/mps-pointops
// mps_pointops/spatial.py:76-264, `SpatialIndex.knn` / `.ball_query`).
// Results equal the brute-force kernels' (knn_wq3_kernel / knn3p_kernel with
// the D == 3 kNN policy, ball_query_kernel): only the set of reference points
// that is evaluated changes, never the arithmetic or the selection order.
//
// Build (counting sort into a uniform grid; no comparison sort):
//   cell = (floor((x - ox) / h), ...) clamped to the grid, linear index
//   (ix * gy + iy) * gz + iz.  grid_count_kernel histograms the cells,
//   three scan kernels turn the counts into cell_start[cells + 1], and
//   grid_scatter_kernel writes every point as float4 (x, y, z, index bits)
//   into its cell's range (the order inside a cell does not matter: ties are
//   broken by the original index).  Points with a non-finite coordinate go to
//   a separate list that every kNN query scans (they can never lie inside a
//   ball).
// kNN (warp per query): the warp scans Chebyshev rings of cells around the
//   query's cell, ring r = 0, 1, ...; each lane walks one cell of the ring at
//   a time, and candidates below the bar enter a warp-wide top-k kept
//   unsorted one entry per lane ((SD key, index) order, two redux.sync per
//   insertion, one bitonic sort at the end).  After ring r every point not yet
//   scanned lies outside the block of cells [c - r, c + r], at distance >= lb
//   (the query's distance to the nearest block face that is not a grid
//   boundary).  The search stops once the list is full and
//   lb^2 * (1 - 2^-16) > the k-th squared distance: the fp32 squared distance
//   of any unscanned point is then larger than the k-th (its relative error is
//   a few ulps), so the exact (SD, index) top-k is already in the list.
// Ball query (warp per query): every cell of the cube of R = ceil(r (1 + 2^-16)
//   / h) rings holds all points with SD < r^2 (a point R + 1 cells away is more
//   than R h >= r away along one axis); hits enter a warp-wide list keyed by
//   original index, so the output is the first K hits in input order, exactly
//   as the full scan gives them.
#include <cmath>
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kSpWarps = 8;
constexpr uint32_t kMaxKey = 0xffffffffu;
constexpr uint32_t kNoIdx = 0xffffffffu;

struct Grid {
    float ox, oy, oz, h, inv_h;
    float slack;  // bound on the float rounding of cell assignment and cell faces
    int gx, gy, gz;
    const int* start;    // cells + 1
    const float4* pts;   // sorted (x, y, z, original index bits)
    const float4* extra; // points with a non-finite coordinate
    int n_extra;
};

__device__ __forceinline__ int cell_coord(float v, float o, float inv_h, int g) {
    const float t = floorf(__fmul_rn(__fsub_rn(v, o), inv_h));
    if (!(t >= 0.f)) return 0;  // also NaN
    return t >= (float)(g - 1) ? g - 1 : (int)t;
}

__device__ __forceinline__ uint32_t sd_key(float d) {
    return isnan(d) ? kMaxKey : ordered_key(d);
}

// Warp-wide top-k, one entry per lane s < k, kept unsorted; the worst entry
// (largest (key, index)) is the bar.  Empty slots are (kMaxKey, kNoIdx - s).
struct WarpTopK {
    uint32_t lk, lx;
    float ld;
    uint32_t wk, wi;
    int k;

    __device__ void init(int k_, int lane) {
        k = k_;
        lk = lane < k ? kMaxKey : 0u;
        lx = lane < k ? kNoIdx - (uint32_t)lane : 0u;
        ld = INFINITY;
        wk = kMaxKey;
        wi = kNoIdx;
    }
    __device__ bool full() const { return wi < 0x80000000u || wk != kMaxKey; }
    // Squared distance of the worst entry; +inf while a slot is empty, NaN
    // when the worst entry is a NaN distance.
    __device__ float bar() const {
        if (wk != kMaxKey) return ordered_key_inv(wk);
        return wi >= 0x80000000u ? INFINITY : __int_as_float(0x7fffffff);
    }
    // Warp-uniform candidate (key, index, distance).
    __device__ void offer(uint32_t ck, uint32_t ci, float cd, int lane) {
        if (!(ck < wk || (ck == wk && ci < wi))) return;
        if (lk == wk && lx == wi) {
            lk = ck;
            lx = ci;
            ld = cd;
        }
        (void)lane;
        wk = __reduce_max_sync(FULL_MASK, lk);
        wi = __reduce_max_sync(FULL_MASK, lk == wk ? lx : 0u);
    }
    // Sort ascending by (key, index) across the warp; lanes >= k last.
    __device__ void sort(int lane) {
        if (lane >= k) {
            lk = kMaxKey;
            lx = 0xffffffffu;
        }
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                const uint32_t ok = __shfl_xor_sync(FULL_MASK, lk, stride);
                const uint32_t ox = __shfl_xor_sync(FULL_MASK, lx, stride);
                const float od = __shfl_xor_sync(FULL_MASK, ld, stride);
                const bool ascending = (lane & size) == 0;
                const bool lower = (lane & stride) == 0;
                const bool other_first = ok < lk || (ok == lk && ox < lx);
                if ((lower == ascending) ? other_first : !other_first) {
                    lk = ok;
                    lx = ox;
                    ld = od;
                }
            }
        }
    }
};

// ------------------------------------------------------------------ build
__global__ void grid_count_kernel(const float* __restrict__ p, int64_t N, Grid g,
                                  int* __restrict__ cell_of, int* __restrict__ counts,
                                  int* __restrict__ n_extra) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float x = p[3 * i], y = p[3 * i + 1], z = p[3 * i + 2];
        int c = -1;
        if (isfinite(x) && isfinite(y) && isfinite(z)) {
            c = (cell_coord(x, g.ox, g.inv_h, g.gx) * g.gy + cell_coord(y, g.oy, g.inv_h, g.gy)) *
                    g.gz +
                cell_coord(z, g.oz, g.inv_h, g.gz);
            atomicAdd(counts + c, 1);
        } else {
            atomicAdd(n_extra, 1);
        }
        cell_of[i] = c;
    }
}

// Exclusive scan of `n` ints in three launches: per-block sums, a scan of the
// block sums in one CTA, then per-block scans plus their block offsets.
constexpr int kScanThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(FULL_MASK, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(FULL_MASK, wi, o);
            if (lane >= o) wi += t;
        }
        warp_sums[lane] = wi - w;  // exclusive prefix of the warp sums
        if (lane == 31) warp_sums[32] = wi;
    }
    __syncthreads();
    total = warp_sums[32];
    const int r = warp_sums[warp] + incl - v;
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kScanThreads)
scan_block_sums_kernel(const int* __restrict__ in, int64_t n, int* __restrict__ sums) {
    __shared__ int ws[33];
    const int64_t i = (int64_t)blockIdx.x * kScanThreads + threadIdx.x;
    int total;
    block_exclusive_scan(i < n ? in[i] : 0, ws, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kScanThreads)
scan_sums_kernel(int* __restrict__ sums, int64_t nb) {
    __shared__ int ws[33];
    int carry = 0;
    for (int64_t b0 = 0; b0 < nb; b0 += kScanThreads) {
        const int64_t i = b0 + threadIdx.x;
        const int v = i < nb ? sums[i] : 0;
        int total;
        const int ex = block_exclusive_scan(v, ws, total);
        if (i < nb) sums[i] = ex + carry;
        carry += total;
    }
}

__global__ void __launch_bounds__(kScanThreads)
scan_apply_kernel(const int* __restrict__ in, int64_t n, const int* __restrict__ sums,
                  int* __restrict__ out, int* __restrict__ cursor) {
    __shared__ int ws[33];
    const int64_t i = (int64_t)blockIdx.x * kScanThreads + threadIdx.x;
    int total;
    const int ex = block_exclusive_scan(i < n ? in[i] : 0, ws, total) + sums[blockIdx.x];
    if (i < n) {
        out[i] = ex;
        cursor[i] = ex;
    }
    if (i == n - 1) out[n] = ex + in[i];
}

__global__ void grid_scatter_kernel(const float* __restrict__ p, int64_t N,
                                    const int* __restrict__ cell_of, int* __restrict__ cursor,
                                    int* __restrict__ extra_cursor, float4* __restrict__ pts,
                                    float4* __restrict__ extra) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = make_float4(p[3 * i], p[3 * i + 1], p[3 * i + 2],
                                     __int_as_float((int)i));
        const int c = cell_of[i];
        if (c >= 0) pts[atomicAdd(cursor + c, 1)] = v;
        else extra[atomicAdd(extra_cursor, 1)] = v;
    }
}

// ------------------------------------------------------------------ search helpers
struct Block {
    int lo[3], hi[3];
};

// Distance from q to the nearest face of the block that is not a grid
// boundary (the unscanned points lie beyond such faces); +inf when the block
// covers the whole grid.
__device__ __forceinline__ float block_bound(const Grid& g, const Block& bl, float qx, float qy,
                                             float qz) {
    const float q[3] = {qx, qy, qz};
    const float o[3] = {g.ox, g.oy, g.oz};
    const int gd[3] = {g.gx, g.gy, g.gz};
    float lb = INFINITY;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        if (bl.lo[a] > 0) lb = fminf(lb, q[a] - (o[a] + (float)bl.lo[a] * g.h));
        if (bl.hi[a] < gd[a] - 1) lb = fminf(lb, (o[a] + (float)(bl.hi[a] + 1) * g.h) - q[a]);
    }
    // A point is assigned to its cell by floor((x - o) / h) in float, and the
    // faces are computed in float too: either can be off by a few ulps, so
    // the bound gives up `slack`.
    return fmaxf(lb - g.slack, 0.f);
}

// Visit the cells of ring r around (cx, cy, cz) (Chebyshev distance exactly
// r, inside the grid), one per lane per round, calling visit(start, end) with
// each lane's cell range (empty for lanes without a cell).  The ring's
// surface is enumerated directly: the two z faces ((2r+1)^2 cells each), the
// two y faces without their z edges ((2r+1)(2r-1)), the two x faces without
// either ((2r-1)^2).
template <typename F>
__device__ __forceinline__ void for_ring(const Grid& g, int cx, int cy, int cz, int r, int lane,
                                         F&& visit) {
    const int a = 2 * r + 1, b = 2 * r - 1;
    const int fa = a * a, fb = a * b, fc = b * b;
    const int total = r == 0 ? 1 : 2 * (fa + fb + fc);
    for (int t0 = 0; t0 < total; t0 += 32) {
        int t = t0 + lane;
        int s = 0, e = 0;
        if (t < total) {
            int dx = 0, dy = 0, dz = 0;
            if (r > 0) {
                if (t < 2 * fa) {
                    dz = t < fa ? -r : r;
                    const int u = t % fa;
                    dx = u / a - r;
                    dy = u % a - r;
                } else if ((t -= 2 * fa) < 2 * fb) {
                    dy = t < fb ? -r : r;
                    const int u = t % fb;
                    dx = u / b - r;
                    dz = u % b - (r - 1);
                } else {
                    t -= 2 * fb;
                    dx = t < fc ? -r : r;
                    const int u = t % fc;
                    dy = u / b - (r - 1);
                    dz = u % b - (r - 1);
                }
            }
            const int x = cx + dx, y = cy + dy, z = cz + dz;
            if (x >= 0 && x < g.gx && y >= 0 && y < g.gy && z >= 0 && z < g.gz) {
                const int c = (x * g.gy + y) * g.gz + z;
                s = g.start[c];
                e = g.start[c + 1];
            }
        }
        visit(s, e);
    }
}

// ------------------------------------------------------------------ kNN
__global__ void __launch_bounds__(kSpWarps * 32)
grid_knn_kernel(const float* __restrict__ query, int64_t Q, Grid g, int k,
                float* __restrict__ dist, int64_t* __restrict__ idx) {
    const int lane = threadIdx.x & 31;
    const int64_t q = (int64_t)blockIdx.x * kSpWarps + (threadIdx.x >> 5);
    if (q >= Q) return;
    const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
    WarpTopK top;
    top.init(k, lane);
    const bool finite_q = isfinite(qx) && isfinite(qy) && isfinite(qz);
    const int cx = cell_coord(qx, g.ox, g.inv_h, g.gx);
    const int cy = cell_coord(qy, g.oy, g.inv_h, g.gy);
    const int cz = cell_coord(qz, g.oz, g.inv_h, g.gz);
    const int rmax = max(max(g.gx, g.gy), g.gz);
    auto consider = [&](float d, uint32_t j, bool valid) {
        // Candidates of the lanes, one warp-wide offer each.  NaN distances
        // never enter (the D == 3 kNN policy); +inf is ranked.
        const float bar = top.bar();
        unsigned pending = __ballot_sync(FULL_MASK, valid && !isnan(d) && !(d > bar));
        while (pending) {
            const int src = __ffs(pending) - 1;
            pending &= pending - 1;
            const float cd = __shfl_sync(FULL_MASK, d, src);
            const uint32_t ci = __shfl_sync(FULL_MASK, j, src);
            top.offer(sd_key(cd), ci, cd, lane);
        }
    };
    // A query with a non-finite coordinate has no position in the grid: it
    // scans every point (its distances are NaN or +inf).
    const int n_grid = g.start[g.gx * g.gy * g.gz];
    for (int e0 = 0; !finite_q && e0 < n_grid; e0 += 32) {
        const int e = e0 + lane;
        const bool valid = e < n_grid;
        float d = INFINITY;
        uint32_t j = 0;
        if (valid) {
            const float4 p = g.pts[e];
            d = sqd3(qx, qy, qz, p.x, p.y, p.z);
            j = (uint32_t)__float_as_int(p.w);
        }
        consider(d, j, valid);
    }
    for (int r = 0; finite_q && r <= rmax; ++r) {
        for_ring(g, cx, cy, cz, r, lane, [&](int s, int e) {
            // Lanes walk their cells in lock step until every cell is done.
            int cur = s;
            while (__any_sync(FULL_MASK, cur < e)) {
                const bool valid = cur < e;
                float d = INFINITY;
                uint32_t j = 0;
                if (valid) {
                    const float4 p = g.pts[cur];
                    d = sqd3(qx, qy, qz, p.x, p.y, p.z);
                    j = (uint32_t)__float_as_int(p.w);
                }
                consider(d, j, valid);
                ++cur;
            }
        });
        Block bl;
        bl.lo[0] = max(cx - r, 0); bl.hi[0] = min(cx + r, g.gx - 1);
        bl.lo[1] = max(cy - r, 0); bl.hi[1] = min(cy + r, g.gy - 1);
        bl.lo[2] = max(cz - r, 0); bl.hi[2] = min(cz + r, g.gz - 1);
        const float lb = block_bound(g, bl, qx, qy, qz);
        if (lb == INFINITY) break;  // the whole grid is scanned
        const float kth = top.bar();
        if (top.full() && __fmul_rn(__fmul_rn(lb, lb), 1.0f - 1.52587890625e-05f) > kth) break;
    }
    // Points with a non-finite coordinate: scanned by every query.
    for (int e0 = 0; e0 < g.n_extra; e0 += 32) {
        const int e = e0 + lane;
        const bool valid = e < g.n_extra;
        float d = INFINITY;
        uint32_t j = 0;
        if (valid) {
            const float4 p = g.extra[e];
            d = sqd3(qx, qy, qz, p.x, p.y, p.z);
            j = (uint32_t)__float_as_int(p.w);
        }
        consider(d, j, valid);
    }
    top.sort(lane);
    if (lane >= k) return;
    const bool filled = top.lx < 0x80000000u;
    const float dd = filled ? top.ld : INFINITY;
    dist[q * k + lane] = sqrtf(dd);
    idx[q * k + lane] = filled ? (int64_t)top.lx : -1;
}

// ------------------------------------------------------------------ ball query
__global__ void __launch_bounds__(kSpWarps * 32)
grid_ball_query_kernel(const float* __restrict__ query, int64_t Q, Grid g, int R, float r2,
                       int K, float* __restrict__ dist2, int64_t* __restrict__ idx) {
    const int lane = threadIdx.x & 31;
    const int64_t q = (int64_t)blockIdx.x * kSpWarps + (threadIdx.x >> 5);
    if (q >= Q) return;
    const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
    WarpTopK top;  // keyed by original index only: the first K hits in input order
    top.init(K, lane);
    if (isfinite(qx) && isfinite(qy) && isfinite(qz)) {
        const int cx = cell_coord(qx, g.ox, g.inv_h, g.gx);
        const int cy = cell_coord(qy, g.oy, g.inv_h, g.gy);
        const int cz = cell_coord(qz, g.oz, g.inv_h, g.gz);
        for (int r = 0; r <= R; ++r) {
            for_ring(g, cx, cy, cz, r, lane, [&](int s, int e) {
                int cur = s;
                while (__any_sync(FULL_MASK, cur < e)) {
                    bool hit = false;
                    float d = 0.f;
                    uint32_t j = 0;
                    if (cur < e) {
                        const float4 p = g.pts[cur];
                        d = sqd3(qx, qy, qz, p.x, p.y, p.z);
                        j = (uint32_t)__float_as_int(p.w);
                        hit = d < r2 && (!top.full() || j < top.wi);
                    }
                    unsigned pending = __ballot_sync(FULL_MASK, hit);
                    while (pending) {
                        const int src = __ffs(pending) - 1;
                        pending &= pending - 1;
                        const float cd = __shfl_sync(FULL_MASK, d, src);
                        const uint32_t ci = __shfl_sync(FULL_MASK, j, src);
                        top.offer(0u, ci, cd, lane);
                    }
                    ++cur;
                }
            });
        }
    }
    top.sort(lane);
    if (lane >= K) return;
    const bool filled = top.lx < 0x80000000u;
    dist2[q * K + lane] = filled ? top.ld : 0.f;
    idx[q * K + lane] = filled ? (int64_t)top.lx : -1;
}

Grid make_grid(const float* origin, float h, const int* dims, const int* start, const float4* pts,
               const float4* extra, int n_extra) {
    Grid g;
    g.ox = origin[0];
    g.oy = origin[1];
    g.oz = origin[2];
    g.h = h;
    g.inv_h = 1.0f / h;
    // 2^-20 of the largest coordinate magnitude the grid spans: about 16
    // float ulps, far above the rounding of one subtraction and one multiply.
    const float reach = fmaxf(fmaxf(fabsf(origin[0]), fabsf(origin[1])), fabsf(origin[2])) +
                        (float)max(max(dims[0], dims[1]), dims[2]) * h;
    g.slack = reach * 9.5367431640625e-07f;
    g.gx = dims[0];
    g.gy = dims[1];
    g.gz = dims[2];
    g.start = start;
    g.pts = pts;
    g.extra = extra;
    g.n_extra = n_extra;
    return g;
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_grid_workspace_bytes(int64_t N, int64_t cells) {
    if (N < 0 || cells <= 0) return 0;
    const int64_t nb = mpo::ceil_div(cells, mpo::kScanThreads);
    // cell_of (N), counts (cells), cursor (cells), block sums (nb), extra counters (2)
    return (size_t)(N + 2 * cells + nb + 2) * sizeof(int) + 256;
}

int mpo_grid_build(const float* points, int64_t N, const float* origin, float cell_size,
                   const int* dims, int* cell_start, float* sorted_points, float* extra_points,
                   int32_t* n_extra_out, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(N >= 0 && N < (int64_t)0x7fffffff, "N must be in [0, 2**31)");
    MPO_REQUIRE(origin && dims && cell_start && n_extra_out, "null pointer");
    MPO_REQUIRE(cell_size > 0.f && isfinite(cell_size), "cell_size must be positive and finite");
    MPO_REQUIRE(dims[0] >= 1 && dims[1] >= 1 && dims[2] >= 1, "grid dims must be positive");
    const int64_t cells = (int64_t)dims[0] * dims[1] * dims[2];
    MPO_REQUIRE(cells < (int64_t)1 << 28, "at most 2**28 grid cells");
    const size_t need = mpo_grid_workspace_bytes(N, cells);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(kWorkspaceTooSmall, "mpo_grid_build: workspace must hold " +
                                            std::to_string(need) + " bytes");
    MPO_REQUIRE((points && sorted_points && extra_points) || N == 0, "null pointer");
    MPO_REQUIRE_WORKSPACE(workspace);
    MPO_REQUIRE(aligned_to(sorted_points, 16) && aligned_to(extra_points, 16),
                "sorted_points and extra_points must be 16-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    int* cell_of = static_cast<int*>(workspace);
    int* counts = cell_of + N;
    int* cursor = counts + cells;
    int* sums = cursor + cells;
    const int64_t nb = ceil_div(cells, kScanThreads);
    int* extra_counters = sums + nb;  // [0] count, [1] cursor
    if (cudaMemsetAsync(counts, 0, sizeof(int) * cells, s) != cudaSuccess ||
        cudaMemsetAsync(extra_counters, 0, 2 * sizeof(int), s) != cudaSuccess)
        return fail(kCudaError, "mpo_grid_build: memset failed");
    const Grid g = make_grid(origin, cell_size, dims, nullptr, nullptr, nullptr, 0);
    const unsigned pgrid = (unsigned)max64(1, min64(ceil_div(N, 256), (int64_t)sm_count() * 16));
    if (N > 0) {
        grid_count_kernel<<<pgrid, 256, 0, s>>>(points, N, g, cell_of, counts, extra_counters);
        int st = check_launch("grid_count_kernel");
        if (st) return st;
    }
    scan_block_sums_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(counts, cells, sums);
    int st = check_launch("scan_block_sums_kernel");
    if (st) return st;
    scan_sums_kernel<<<1, kScanThreads, 0, s>>>(sums, nb);
    st = check_launch("scan_sums_kernel");
    if (st) return st;
    scan_apply_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(counts, cells, sums, cell_start, cursor);
    st = check_launch("scan_apply_kernel");
    if (st) return st;
    if (N > 0) {
        grid_scatter_kernel<<<pgrid, 256, 0, s>>>(points, N, cell_of, cursor, extra_counters + 1,
                                                  reinterpret_cast<float4*>(sorted_points),
                                                  reinterpret_cast<float4*>(extra_points));
        st = check_launch("grid_scatter_kernel");
        if (st) return st;
    }
    if (cudaMemcpyAsync(n_extra_out, extra_counters, sizeof(int32_t), cudaMemcpyDeviceToDevice,
                        s) != cudaSuccess)
        return fail(kCudaError, "mpo_grid_build: copy failed");
    return kOk;
}

int mpo_grid_knn(const float* query, int64_t Q, const float* origin, float cell_size,
                 const int* dims, const int* cell_start, const float* sorted_points,
                 const float* extra_points, int32_t n_extra, int64_t k, float* dist, int64_t* idx,
                 void* stream) {
    using namespace mpo;
    MPO_REQUIRE(Q >= 0 && k >= 0 && k <= 32, "k must be in [0, 32]");
    MPO_REQUIRE(n_extra >= 0, "negative extra count");
    if (Q == 0 || k == 0) return kOk;
    MPO_REQUIRE(query && origin && dims && cell_start && dist && idx, "null pointer");
    MPO_REQUIRE(aligned_to(sorted_points, 16) && aligned_to(extra_points, 16),
                "sorted_points and extra_points must be 16-byte aligned");
    const Grid g = make_grid(origin, cell_size, dims, cell_start,
                             reinterpret_cast<const float4*>(sorted_points),
                             reinterpret_cast<const float4*>(extra_points), n_extra);
    grid_knn_kernel<<<(unsigned)ceil_div(Q, kSpWarps), kSpWarps * 32, 0, (cudaStream_t)stream>>>(
        query, Q, g, (int)k, dist, idx);
    return check_launch("grid_knn_kernel");
}

int mpo_grid_ball_query(const float* query, int64_t Q, const float* origin, float cell_size,
                        const int* dims, const int* cell_start, const float* sorted_points,
                        float radius, float radius_sq, int64_t K, float* dist2, int64_t* idx,
                        void* stream) {
    using namespace mpo;
    MPO_REQUIRE(Q >= 0 && K >= 0 && K <= 32, "K must be in [0, 32]");
    if (Q == 0 || K == 0) return kOk;
    MPO_REQUIRE(query && origin && dims && cell_start && dist2 && idx, "null pointer");
    MPO_REQUIRE(aligned_to(sorted_points, 16), "sorted_points must be 16-byte aligned");
    MPO_REQUIRE(radius >= 0.f, "radius must be non-negative");
    const Grid g = make_grid(origin, cell_size, dims, cell_start,
                             reinterpret_cast<const float4*>(sorted_points), nullptr, 0);
    // Rings that can hold a point with SD < r^2, with a relative margin for
    // the fp32 rounding of the distance; the whole grid when that is larger.
    const double reach =
        ((double)radius * (1.0 + 1.0 / 65536.0) + (double)g.slack) / (double)cell_size;
    const int gmax = max(max(dims[0], dims[1]), dims[2]);
    const int R = (!(reach < (double)gmax)) ? gmax : (int)std::ceil(reach);
    grid_ball_query_kernel<<<(unsigned)ceil_div(Q, kSpWarps), kSpWarps * 32, 0,
                             (cudaStream_t)stream>>>(query, Q, g, R, radius_sq, (int)K, dist2,
                                                     idx);
    return check_launch("grid_ball_query_kernel");
}

}  // extern "C"
