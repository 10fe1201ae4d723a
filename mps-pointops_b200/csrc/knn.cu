// Brute-force k-nearest-neighbour search (xyz and feature space) and the
// k = 3 PointNet++ specialisation, on sm_100a.
//
// Contracts (gamzerA/mps-pointops):
//   knn       mps_pointops/ops.py:144-205; exact order of tests/test_knn.py:15-23
//             and tests/test_feature_knn.py:16-35: ascending (SD, index),
//             Euclidean distance = sqrt(SD) taken after selection.
//   three_nn  mps_pointops/pointnet2.py:54-100: the same order with NaN after
//             every number (torch's stable argsort), int32 indices.
//
// Design (B200):
//   * One thread owns one (query, split).  A CTA of 256 threads covers
//     256/S queries of one cloud and S splits; split s scans the s-th slice
//     of every reference tile, so each warp (one split, 32 queries) reads the
//     same shared-memory address -> broadcast, no bank conflicts.
//   * Reference tiles (1024 points, stored as float4) are staged through
//     shared memory, double-buffered: the next tile is loaded into registers
//     with coalesced scalar loads while the current one is scanned.
//   * The running top-k list (capacity K in {4, 8, 16, 32}) lives in
//     registers, sorted by (SD, index).  The hot loop costs the 8 rounded
//     float ops of the distance plus ONE compare against the current k-th
//     distance (`!(d > kth)`); the register insertion runs only for the rare
//     candidate that passes.  Within one thread the reference index grows
//     monotonically, so a tie with the k-th entry never displaces it.
//   * After the scan, splits 1..S-1 publish their lists to shared memory and
//     split 0 merges them with the full (SD, index) order.
//   * k in (32, 256] uses a warp-per-query kernel whose sorted list is spread
//     over the 32 lanes (8 slots each) and updated with ballot/shuffle.
//   * k <= 32 on clouds up to 2^18 points (and three_nn) uses a warp-per-query
//     kernel (knn_wq3_kernel) with the 32 best kept sorted across the lanes
//     and candidates merged 32 at a time: a thread-owned list makes the whole
//     warp replay the insertion whenever any lane inserts, which on moderate
//     clouds happens on almost every step.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"
#include "knn_select.cuh"
#include "segments.cuh"

namespace mpo {
namespace {

constexpr int kThreads = 256;
constexpr int kTile = 1024;  // reference points per shared-memory tile (D == 3)
constexpr int kQueue = 16;   // per-lane candidate queue (D == 3 thread kernel)

// --------------------------------------------------------------------------
// D == 3 kernel.
template <int K, int POLICY>
__global__ void __launch_bounds__(kThreads, 2)
knn3_kernel(const float* __restrict__ query, const float* __restrict__ ref, int64_t M, int64_t N,
            int k, int S, float* __restrict__ dist, int64_t* __restrict__ idx64,
            int32_t* __restrict__ idx32, float* __restrict__ sqdist) {
    extern __shared__ float4 smem4[];
    float4* tile = smem4;  // [2][kTile]
    const int b = blockIdx.y;
    const int qpc = kThreads / S;
    const int tid = threadIdx.x;
    const int split = tid / qpc;
    const int ql = tid % qpc;
    const int64_t q = (int64_t)blockIdx.x * qpc + ql;
    const bool active = q < M;
    const float* __restrict__ r = ref + (size_t)b * (size_t)N * 3;

    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (active) {
        const float* qp = query + ((size_t)b * (size_t)M + (size_t)q) * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    TopK<K, POLICY> top;
    top.init(k);

    const int64_t ntiles = ceil_div(N, kTile);
    const int slice = kTile / S;
    constexpr int kLoads = 3 * kTile / kThreads;  // 12 scalar loads per thread per tile
    float pre[kLoads];

#define MPO_LOAD_TILE(t)                                                   \
    do {                                                                   \
        const int64_t base_ = (t) * kTile * 3;                             \
        _Pragma("unroll") for (int u = 0; u < kLoads; ++u) {               \
            const int64_t e_ = base_ + tid + (int64_t)u * kThreads;        \
            pre[u] = e_ < N * 3 ? r[e_] : 0.f;                             \
        }                                                                  \
    } while (0)
#define MPO_STORE_TILE(buf)                                                \
    do {                                                                   \
        float* t_ = reinterpret_cast<float*>(tile + (buf) * kTile);        \
        _Pragma("unroll") for (int u = 0; u < kLoads; ++u) {               \
            const int e_ = tid + u * kThreads;                             \
            t_[(e_ / 3) * 4 + (e_ % 3)] = pre[u];                          \
        }                                                                  \
    } while (0)

    // Candidates that pass the threshold are queued per lane in shared memory
    // ([slot][thread], conflict-free) and inserted in bulk when some lane's
    // queue is nearly full: the warp then replays ONE insertion round for all
    // lanes instead of one per candidate of any lane.
    uint32_t* qi = reinterpret_cast<uint32_t*>(tile + 2 * kTile);
    float* qd = reinterpret_cast<float*>(qi + kQueue * kThreads);
    int qn = 0;
    auto flush = [&]() {
        for (int e = 0; e < qn; ++e) top.offer(qd[e * kThreads + tid], qi[e * kThreads + tid]);
        qn = 0;
    };
    if (ntiles > 0) {
        MPO_LOAD_TILE(0);
        MPO_STORE_TILE(0);
    }
    __syncthreads();
    float thr = top.kth();
    for (int64_t t = 0; t < ntiles; ++t) {
        const int buf = (int)(t & 1);
        if (t + 1 < ntiles) MPO_LOAD_TILE(t + 1);
        if (active) {
            const float4* tp = tile + buf * kTile + split * slice;
            const int64_t j0 = t * kTile + split * slice;
            const int cnt = (int)max64(0, min64(slice, N - j0));
            for (int e = 0; e < cnt; e += 4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 p = tp[e + u];
                    const float d = sqd3(qx, qy, qz, p.x, p.y, p.z);
                    if (!(d > thr) && e + u < cnt) {
                        qd[qn * kThreads + tid] = d;
                        qi[qn * kThreads + tid] = (uint32_t)(j0 + e + u);
                        ++qn;
                    }
                }
                if (__any_sync(__activemask(), qn > kQueue - 4)) {
                    flush();
                    thr = top.kth();
                }
            }
        }
        if (t + 1 < ntiles) MPO_STORE_TILE(buf ^ 1);
        __syncthreads();
    }
    if (active) flush();
    // The merge below reuses the tile and queue memory: every warp must have
    // drained its queue first.
    __syncthreads();
#undef MPO_LOAD_TILE
#undef MPO_STORE_TILE

    // Merge the S split lists into split 0 (full (SD, index) order).
    if (S > 1) {
        float* md = reinterpret_cast<float*>(smem4);
        uint32_t* mi = reinterpret_cast<uint32_t*>(md + (size_t)kThreads * K);
        if (split > 0) {
#pragma unroll
            for (int s = 0; s < K; ++s) {
                md[(size_t)tid * K + s] = top.d[s];
                mi[(size_t)tid * K + s] = top.i[s];
            }
        }
        __syncthreads();
        if (split == 0 && active) {
            for (int o = 1; o < S; ++o) {
                const int src = o * qpc + ql;
                for (int s = K - k; s < K; ++s) {
                    const uint32_t j = mi[(size_t)src * K + s];
                    if (j == kNoIndex) break;
                    const float d = md[(size_t)src * K + s];
                    if (top.full() && !before<POLICY>(d, j, top.d[K - 1], top.i[K - 1])) break;
                    top.offer(d, j);
                }
            }
        }
    }
    if (split != 0 || !active) return;
    const size_t row = ((size_t)b * (size_t)M + (size_t)q) * (size_t)k;
#pragma unroll
    for (int s = 0; s < K; ++s) {
        const int l = s - top.base;
        if (l >= 0) {
            const bool filled = l < top.cnt;
            const float d = filled ? top.d[s] : INFINITY;
            dist[row + l] = sqrtf(d);
            if (sqdist) sqdist[row + l] = d;
            if (idx64) idx64[row + l] = filled ? (int64_t)top.i[s] : -1;
            if (idx32) idx32[row + l] = filled ? (int32_t)top.i[s] : -1;
        }
    }
}

// --------------------------------------------------------------------------
// D == 3, large reference clouds (N > 2^18): thread per (query, split) as in
// knn3_kernel, but packed over references -- the query sits duplicated in
// f32x2 registers, (qx, qx), and one packed pass evaluates two reference
// points, so the distance costs half the issue slots of the scalar loop (the
// FP32 pipe then bounds the kernel).  The tile stores reference points in
// structure-of-arrays pairs: (x_2p, x_2p+1, y_2p, y_2p+1) per point pair and
// (z_4i .. z_4i+3) per four points.
template <int K, int POLICY, bool FLAT>
__global__ void __launch_bounds__(kThreads, 2)
knn3p_kernel(const float* __restrict__ query, const float* __restrict__ ref, Layout L, int k,
             int S, float* __restrict__ dist, int64_t* __restrict__ idx64,
             int32_t* __restrict__ idx32, float* __restrict__ sqdist) {
    extern __shared__ float4 smem4[];
    float4* txy = smem4;                    // [2][kTile / 2]
    float4* tz = smem4 + kTile;             // [2][kTile / 4]
    const int qpc = kThreads / S;
    Span sp;
    if (!locate<FLAT>(L, qpc, sp)) return;  // CTA-uniform
    const int tid = threadIdx.x;
    const int split = tid / qpc;
    const int ql = tid % qpc;
    const int64_t q = sp.q0 + ql;
    const bool active = q < sp.q1;
    const int64_t N = sp.n;
    const float* __restrict__ r = ref + (size_t)sp.r0 * 3;

    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (active) {
        const float* qp = query + (size_t)q * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    const f32x2 X = pack2(qx, qx), Y = pack2(qy, qy), Z = pack2(qz, qz);
    TopK<K, POLICY> top;
    top.init(k);

    const int64_t ntiles = ceil_div(N, kTile);
    const int slice = kTile / S;  // multiple of 4
    constexpr int kLoads = 3 * kTile / kThreads;
    float pre[kLoads];
    uint32_t* qi = reinterpret_cast<uint32_t*>(smem4 + kTile + kTile / 2);
    float* qd = reinterpret_cast<float*>(qi + kQueue * kThreads);
    int qn = 0;
    auto flush = [&]() {
        for (int e = 0; e < qn; ++e) top.offer(qd[e * kThreads + tid], qi[e * kThreads + tid]);
        qn = 0;
    };
    auto load_tile = [&](int64_t t) {
        const int64_t base = t * kTile * 3;
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t e = base + tid + (int64_t)u * kThreads;
            pre[u] = e < N * 3 ? r[e] : 0.f;
        }
    };
    auto store_tile = [&](int buf) {
        float* xy = reinterpret_cast<float*>(txy + buf * (kTile / 2));
        float* zz = reinterpret_cast<float*>(tz + buf * (kTile / 4));
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int e = tid + u * kThreads;
            const int pnt = e / 3, crd = e % 3;
            if (crd < 2) xy[(pnt >> 1) * 4 + 2 * crd + (pnt & 1)] = pre[u];
            else zz[pnt] = pre[u];
        }
    };
    if (ntiles > 0) {
        load_tile(0);
        store_tile(0);
    }
    __syncthreads();
    float thr = top.kth();
    for (int64_t t = 0; t < ntiles; ++t) {
        const int buf = (int)(t & 1);
        if (t + 1 < ntiles) load_tile(t + 1);
        if (active) {
            const ulonglong2* xy =
                reinterpret_cast<const ulonglong2*>(txy + buf * (kTile / 2) + split * (slice / 2));
            const ulonglong2* zz =
                reinterpret_cast<const ulonglong2*>(tz + buf * (kTile / 4) + split * (slice / 4));
            const int64_t j0 = t * kTile + split * slice;
            const int cnt = (int)max64(0, min64(slice, N - j0));
            // Eight points per step: the common case (no candidate below the
            // threshold) costs six loads, the packed distances, one min per
            // point and one compare-and-branch.  Full steps run without
            // bounds checks and with running shared-memory pointers: once the
            // distances are packed, the integer and branch work per point is
            // what bounds this loop.  The queue gains at most 8 entries per
            // step and is drained above kQueue - 8.
            // a, z: shared-window byte addresses of the step's four point
            // pairs and its eight z values.
            auto step = [&](uint32_t a, uint32_t z, int e, int valid) {
                f32x2 ax0, ay0, ax1, ay1, ax2, ay2, ax3, ay3, z01, z23, z45, z67;
                lds_pairs<0>(a, ax0, ay0);
                lds_pairs<16>(a, ax1, ay1);
                lds_pairs<32>(a, ax2, ay2);
                lds_pairs<48>(a, ax3, ay3);
                lds_pairs<0>(z, z01, z23);
                lds_pairs<16>(z, z45, z67);
                float d[8];
                unpack2(sqd3x2(X, Y, Z, ax0, ay0, z01), d[0], d[1]);
                unpack2(sqd3x2(X, Y, Z, ax1, ay1, z23), d[2], d[3]);
                unpack2(sqd3x2(X, Y, Z, ax2, ay2, z45), d[4], d[5]);
                unpack2(sqd3x2(X, Y, Z, ax3, ay3, z67), d[6], d[7]);
                // fminf skips NaN, which this policy drops anyway.
                const float m = fminf(fminf(fminf(d[0], d[1]), fminf(d[2], d[3])),
                                      fminf(fminf(d[4], d[5]), fminf(d[6], d[7])));
                if (!(m > thr)) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        if (!(d[u] > thr) && u < valid) {
                            qd[qn * kThreads + tid] = d[u];
                            qi[qn * kThreads + tid] = (uint32_t)(j0 + e + u);
                            ++qn;
                        }
                    }
                }
                if (__any_sync(__activemask(), qn > kQueue - 8)) {
                    flush();
                    thr = top.kth();
                }
            };
            const int full = cnt & ~7;
            uint32_t a = (uint32_t)__cvta_generic_to_shared(xy);
            uint32_t z = (uint32_t)__cvta_generic_to_shared(zz);
            for (int e = 0; e < full; e += 8, a += 64, z += 32) step(a, z, e, 8);
            // Ragged end of the slice (the last tile only): one step whose
            // points past cnt (zero-filled tile slots inside the slice) are
            // not offered.
            if (full < cnt) step(a, z, full, cnt - full);
        }
        if (t + 1 < ntiles) store_tile(buf ^ 1);
        __syncthreads();
    }
    if (active) flush();
    __syncthreads();  // the merge reuses the tile and queue memory

    if (S > 1) {
        float* md = reinterpret_cast<float*>(smem4);
        uint32_t* mi = reinterpret_cast<uint32_t*>(md + (size_t)kThreads * K);
        if (split > 0) {
#pragma unroll
            for (int s2 = 0; s2 < K; ++s2) {
                md[(size_t)tid * K + s2] = top.d[s2];
                mi[(size_t)tid * K + s2] = top.i[s2];
            }
        }
        __syncthreads();
        if (split == 0 && active) {
            for (int o = 1; o < S; ++o) {
                const int src = o * qpc + ql;
                for (int s2 = K - k; s2 < K; ++s2) {
                    const uint32_t j = mi[(size_t)src * K + s2];
                    if (j == kNoIndex) break;
                    const float dd = md[(size_t)src * K + s2];
                    if (top.full() && !before<POLICY>(dd, j, top.d[K - 1], top.i[K - 1])) break;
                    top.offer(dd, j);
                }
            }
        }
    }
    if (split != 0 || !active) return;
    const size_t row = (size_t)q * (size_t)k;
#pragma unroll
    for (int s2 = 0; s2 < K; ++s2) {
        const int l = s2 - top.base;
        if (l >= 0) {
            const bool filled = l < top.cnt;
            const float dd = filled ? top.d[s2] : INFINITY;
            if (dist) dist[row + l] = sqrtf(dd);
            if (sqdist) sqdist[row + l] = dd;
            if (idx64) idx64[row + l] = filled ? sp.obase + (int64_t)top.i[s2] : -1;
            if (idx32) idx32[row + l] = filled ? (int32_t)top.i[s2] : -1;
        }
    }
}

// --------------------------------------------------------------------------
// k <= 3 (three_nn, and kNN with k <= 3), D == 3: thread per (query, split)
// with the three best held in registers and updated without branches.  A
// warp's 32 queries differ, so on moderate clouds some lane improves its list
// on almost every step; a divergent insertion would make the whole warp
// replay it, and a 32-wide warp select (knn_wq3_kernel) spends most of its
// instructions merging candidates that k = 3 never needs.  Here a point
// costs its share of the packed distance (four f32x2 instructions), and, in
// steps where some lane of the warp has a point below its third distance,
// one sorted-triple update per point: three compares, three min/max and
// five selects, issued whether or not the point enters.  Within a thread the
// reference index grows, so strict < keeps the lowest index on ties.  While a
// list is not full, or holds a NaN (three_nn ranks NaN last), a step takes
// the general TopK::offer instead.  Splits merge in (SD, index) order as in
// knn3p_kernel.
template <int POLICY, bool FLAT>
__global__ void __launch_bounds__(kThreads, 2)
knn3t_kernel(const float* __restrict__ query, const float* __restrict__ ref, Layout L, int k,
             int S, float* __restrict__ dist, int64_t* __restrict__ idx64,
             int32_t* __restrict__ idx32, float* __restrict__ sqdist) {
    constexpr int K = 3;
    extern __shared__ float4 smem4[];
    float4* txy = smem4;                    // [2][kTile / 2]
    float4* tz = smem4 + kTile;             // [2][kTile / 4]
    const int qpc = kThreads / S;
    Span sp;
    if (!locate<FLAT>(L, qpc, sp)) return;  // CTA-uniform
    const int tid = threadIdx.x;
    const int split = tid / qpc;
    const int ql = tid % qpc;
    const int64_t q = sp.q0 + ql;
    const bool active = q < sp.q1;
    const int64_t N = sp.n;
    const float* __restrict__ r = ref + (size_t)sp.r0 * 3;

    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (active) {
        const float* qp = query + (size_t)q * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    const f32x2 X = pack2(qx, qx), Y = pack2(qy, qy), Z = pack2(qz, qz);
    TopK<K, POLICY> top;
    top.init(k);

    const int64_t ntiles = ceil_div(N, kTile);
    const int slice = kTile / S;  // multiple of 8
    constexpr int kLoads = 3 * kTile / kThreads;
    float pre[kLoads];
    auto load_tile = [&](int64_t t) {
        const int64_t base = t * kTile * 3;
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int64_t e = base + tid + (int64_t)u * kThreads;
            pre[u] = e < N * 3 ? r[e] : 0.f;
        }
    };
    auto store_tile = [&](int buf) {
        float* xy = reinterpret_cast<float*>(txy + buf * (kTile / 2));
        float* zz = reinterpret_cast<float*>(tz + buf * (kTile / 4));
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int e = tid + u * kThreads;
            const int pnt = e / 3, crd = e % 3;
            if (crd < 2) xy[(pnt >> 1) * 4 + 2 * crd + (pnt & 1)] = pre[u];
            else zz[pnt] = pre[u];
        }
    };
    if (ntiles > 0) {
        load_tile(0);
        store_tile(0);
    }
    __syncthreads();
    for (int64_t t = 0; t < ntiles; ++t) {
        const int buf = (int)(t & 1);
        if (t + 1 < ntiles) load_tile(t + 1);
        if (active) {
            const ulonglong2* xy =
                reinterpret_cast<const ulonglong2*>(txy + buf * (kTile / 2) + split * (slice / 2));
            const ulonglong2* zz =
                reinterpret_cast<const ulonglong2*>(tz + buf * (kTile / 4) + split * (slice / 4));
            const int64_t j0 = t * kTile + split * slice;
            const int cnt = (int)max64(0, min64(slice, N - j0));
            auto step = [&](uint32_t a, uint32_t z, int e, int valid) {
                f32x2 ax0, ay0, ax1, ay1, ax2, ay2, ax3, ay3, z01, z23, z45, z67;
                lds_pairs<0>(a, ax0, ay0);
                lds_pairs<16>(a, ax1, ay1);
                lds_pairs<32>(a, ax2, ay2);
                lds_pairs<48>(a, ax3, ay3);
                lds_pairs<0>(z, z01, z23);
                lds_pairs<16>(z, z45, z67);
                float d[8];
                unpack2(sqd3x2(X, Y, Z, ax0, ay0, z01), d[0], d[1]);
                unpack2(sqd3x2(X, Y, Z, ax1, ay1, z23), d[2], d[3]);
                unpack2(sqd3x2(X, Y, Z, ax2, ay2, z45), d[4], d[5]);
                unpack2(sqd3x2(X, Y, Z, ax3, ay3, z67), d[6], d[7]);
                const uint32_t jb = (uint32_t)(j0 + e);
                if (!top.full() || isnan(top.d[K - 1])) {
                    for (int u = 0; u < valid; ++u) top.offer(d[u], jb + u);
                    return;
                }
                const unsigned mask = __activemask();
                const float m = fminf(fminf(fminf(d[0], d[1]), fminf(d[2], d[3])),
                                      fminf(fminf(d[4], d[5]), fminf(d[6], d[7])));
                if (!__any_sync(mask, m < top.d[K - 1])) return;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    // Sorted-triple update (no branch: a per-point vote would
                    // serialise the warp on the list's dependency chain); a
                    // NaN or a point past the slice compares false
                    // everywhere and leaves the list as it is.
                    const float v = u < valid ? d[u] : NAN;
                    const uint32_t j = jb + u;
                    const bool c0 = v < top.d[0], c1 = v < top.d[1], c2 = v < top.d[2];
                    top.d[2] = c1 ? top.d[1] : (c2 ? v : top.d[2]);
                    top.i[2] = c1 ? top.i[1] : (c2 ? j : top.i[2]);
                    top.d[1] = c0 ? top.d[0] : (c1 ? v : top.d[1]);
                    top.i[1] = c0 ? top.i[0] : (c1 ? j : top.i[1]);
                    top.d[0] = c0 ? v : top.d[0];
                    top.i[0] = c0 ? j : top.i[0];
                }
            };
            const int full = cnt & ~7;
            uint32_t a = (uint32_t)__cvta_generic_to_shared(xy);
            uint32_t z = (uint32_t)__cvta_generic_to_shared(zz);
            for (int e = 0; e < full; e += 8, a += 64, z += 32) step(a, z, e, 8);
            if (full < cnt) step(a, z, full, cnt - full);
        }
        if (t + 1 < ntiles) store_tile(buf ^ 1);
        __syncthreads();
    }

    if (S > 1) {
        float* md = reinterpret_cast<float*>(smem4);
        uint32_t* mi = reinterpret_cast<uint32_t*>(md + (size_t)kThreads * K);
        if (split > 0) {
#pragma unroll
            for (int s2 = 0; s2 < K; ++s2) {
                md[(size_t)tid * K + s2] = top.d[s2];
                mi[(size_t)tid * K + s2] = top.i[s2];
            }
        }
        __syncthreads();
        if (split == 0 && active) {
            for (int o = 1; o < S; ++o) {
                const int src = o * qpc + ql;
                for (int s2 = K - k; s2 < K; ++s2) {
                    const uint32_t j = mi[(size_t)src * K + s2];
                    if (j == kNoIndex) break;
                    const float dd = md[(size_t)src * K + s2];
                    if (top.full() && !before<POLICY>(dd, j, top.d[K - 1], top.i[K - 1])) break;
                    top.offer(dd, j);
                }
            }
        }
    }
    if (split != 0 || !active) return;
    const size_t row = (size_t)q * (size_t)k;
#pragma unroll
    for (int s2 = 0; s2 < K; ++s2) {
        const int l = s2 - top.base;
        if (l >= 0) {
            const bool filled = l < top.cnt;
            const float dd = filled ? top.d[s2] : INFINITY;
            if (dist) dist[row + l] = sqrtf(dd);
            if (sqdist) sqdist[row + l] = dd;
            if (idx64) idx64[row + l] = filled ? sp.obase + (int64_t)top.i[s2] : -1;
            if (idx32) idx32[row + l] = filled ? (int32_t)top.i[s2] : -1;
        }
    }
}

// --------------------------------------------------------------------------
// Generic D kernel (feature space): the query row and the reference tile
// both sit in shared memory; SD accumulates in increasing dimension order.
constexpr int kFeatThreads = 128;

template <int K, int POLICY, bool FLAT>
__global__ void __launch_bounds__(kFeatThreads)
knnd_kernel(const float* __restrict__ query, const float* __restrict__ ref, Layout L, int D,
            int k, int S, int tileN, float* __restrict__ dist, int64_t* __restrict__ idx64,
            float* __restrict__ sqdist) {
    extern __shared__ float smemf[];
    const int qpc = kFeatThreads / S;
    Span sp;
    if (!locate<FLAT>(L, qpc, sp)) return;  // CTA-uniform
    const int tid = threadIdx.x;
    const int split = tid / qpc;
    const int ql = tid % qpc;
    const int64_t q = sp.q0 + ql;
    const bool active = q < sp.q1;
    const int64_t N = sp.n;
    const int qstride = D + 1;  // odd stride: conflict-free per-thread rows
    float* sq = smemf;                          // [qpc][D+1]
    float* st = smemf + (size_t)qpc * qstride;  // [tileN][D]
    for (int e = tid; e < qpc * D; e += kFeatThreads) {
        const int qq = e / D, t = e % D;
        const int64_t gq = sp.q0 + qq;
        sq[qq * qstride + t] = gq < sp.q1 ? query[(size_t)gq * D + t] : 0.f;
    }
    TopK<K, POLICY> top;
    top.init(k);
    const float* __restrict__ r = ref + (size_t)sp.r0 * D;
    const float* myq = sq + ql * qstride;
    const int slice = tileN / S;
    for (int64_t t0 = 0; t0 < N; t0 += tileN) {
        __syncthreads();
        const int64_t lim = min64((int64_t)tileN * D, (N - t0) * D);
        for (int64_t e = tid; e < lim; e += kFeatThreads) st[e] = r[t0 * D + e];
        __syncthreads();
        if (!active) continue;
        const int64_t j0 = t0 + (int64_t)split * slice;
        const int cnt = (int)max64(0, min64(slice, N - j0));
        const float* tp = st + (size_t)split * slice * D;
        float thr = top.kth();
        for (int e = 0; e < cnt; ++e) {
            const float* rp = tp + (size_t)e * D;
            float dd = __fsub_rn(myq[0], rp[0]);
            float s = __fmul_rn(dd, dd);
            for (int u = 1; u < D; ++u) {
                dd = __fsub_rn(myq[u], rp[u]);
                s = __fadd_rn(s, __fmul_rn(dd, dd));
            }
            if (!(s > thr)) {
                top.offer(s, (uint32_t)(j0 + e));
                thr = top.kth();
            }
        }
    }
    if (S > 1) {
        __syncthreads();
        float* md = smemf;
        uint32_t* mi = reinterpret_cast<uint32_t*>(md + (size_t)kFeatThreads * K);
        if (split > 0) {
#pragma unroll
            for (int s = 0; s < K; ++s) {
                md[(size_t)tid * K + s] = top.d[s];
                mi[(size_t)tid * K + s] = top.i[s];
            }
        }
        __syncthreads();
        if (split == 0 && active) {
            for (int o = 1; o < S; ++o) {
                const int src = o * qpc + ql;
                for (int s = K - k; s < K; ++s) {
                    const uint32_t j = mi[(size_t)src * K + s];
                    if (j == kNoIndex) break;
                    const float d = md[(size_t)src * K + s];
                    if (top.full() && !before<POLICY>(d, j, top.d[K - 1], top.i[K - 1])) break;
                    top.offer(d, j);
                }
            }
        }
    }
    if (split != 0 || !active) return;
    const size_t row = (size_t)q * (size_t)k;
#pragma unroll
    for (int s = 0; s < K; ++s) {
        const int l = s - top.base;
        if (l >= 0) {
            const bool filled = l < top.cnt;
            const float d = filled ? top.d[s] : INFINITY;
            if (dist) dist[row + l] = sqrtf(d);
            if (sqdist) sqdist[row + l] = d;
            idx64[row + l] = filled ? sp.obase + (int64_t)top.i[s] : -1;
        }
    }
}

// --------------------------------------------------------------------------
// Large k (32 < k <= 256): one warp per query, sorted list spread over the
// lanes, slot s held by lane s % 32 in register s / 32.
constexpr int kWarpSlots = 8;  // 8 * 32 = 256

constexpr int kWarpQueries = 8;  // warps (queries) per CTA

template <int POLICY, bool FLAT>
__global__ void __launch_bounds__(32 * kWarpQueries)
knn_warp_kernel(const float* __restrict__ query, const float* __restrict__ ref, Layout L, int D,
                int k, float* __restrict__ dist, int64_t* __restrict__ idx64,
                float* __restrict__ sqdist) {
    const int lane = threadIdx.x & 31;
    Span sp;
    if (!locate<FLAT>(L, kWarpQueries, sp)) return;
    const int64_t q = sp.q0 + (threadIdx.x >> 5);
    if (q >= sp.q1) return;
    const int64_t N = sp.n;
    const float* __restrict__ qp = query + (size_t)q * D;
    const float* __restrict__ r = ref + (size_t)sp.r0 * D;
    float ld[kWarpSlots];
    uint32_t li[kWarpSlots];
#pragma unroll
    for (int t = 0; t < kWarpSlots; ++t) {
        ld[t] = INFINITY;
        li[t] = kNoIndex;
    }
    int cnt = 0;  // warp-uniform
    auto kth_pair = [&](float& kd, uint32_t& ki) {
        const int tk = (k - 1) / 32;
        float v = ld[0];
        uint32_t w = li[0];
#pragma unroll
        for (int t = 1; t < kWarpSlots; ++t) {
            v = (t == tk) ? ld[t] : v;
            w = (t == tk) ? li[t] : w;
        }
        kd = __shfl_sync(FULL_MASK, v, (k - 1) % 32);
        ki = __shfl_sync(FULL_MASK, w, (k - 1) % 32);
    };
    for (int64_t j0 = 0; j0 < N; j0 += 32) {
        const int64_t j = j0 + lane;
        float d = INFINITY;
        if (j < N) d = (D == 3) ? sqd3(qp[0], qp[1], qp[2], r[3 * j], r[3 * j + 1], r[3 * j + 2])
                                : sqd_seq(qp, r + (size_t)j * D, D);
        // k-th entry (slot k-1) lives in lane (k-1)%32, register (k-1)/32.
        float kd;
        uint32_t ki;
        kth_pair(kd, ki);
        const bool cand = j < N && admissible<POLICY>(d) &&
                          (cnt < k || before<POLICY>(d, (uint32_t)j, kd, ki));
        unsigned pending = __ballot_sync(FULL_MASK, cand);
        while (pending) {
            const int src = __ffs(pending) - 1;
            pending &= pending - 1;
            const float cd = __shfl_sync(FULL_MASK, d, src);
            const uint32_t ci = (uint32_t)(j0 + src);
            // re-check against the (possibly updated) k-th entry
            if (cnt >= k) {
                float kd2;
                uint32_t ki2;
                kth_pair(kd2, ki2);
                if (!before<POLICY>(cd, ci, kd2, ki2)) continue;
            }
            // position = number of filled entries ordered before the candidate
            int below = 0;
#pragma unroll
            for (int t = 0; t < kWarpSlots; ++t) {
                const int s = t * 32 + lane;
                below += (s < cnt && before<POLICY>(ld[t], li[t], cd, ci)) ? 1 : 0;
            }
            const int pos = __reduce_add_sync(FULL_MASK, below);
            // shift slots [pos, k-1) right by one
            float prev_d_last = 0.f;
            uint32_t prev_i_last = 0;
#pragma unroll
            for (int t = 0; t < kWarpSlots; ++t) {
                float up_d = __shfl_up_sync(FULL_MASK, ld[t], 1);
                uint32_t up_i = __shfl_up_sync(FULL_MASK, li[t], 1);
                const float last_d = __shfl_sync(FULL_MASK, ld[t], 31);
                const uint32_t last_i = __shfl_sync(FULL_MASK, li[t], 31);
                if (lane == 0) {
                    up_d = prev_d_last;
                    up_i = prev_i_last;
                }
                prev_d_last = last_d;
                prev_i_last = last_i;
                const int s = t * 32 + lane;
                if (s < k) {
                    if (s > pos) {
                        ld[t] = up_d;
                        li[t] = up_i;
                    } else if (s == pos) {
                        ld[t] = cd;
                        li[t] = ci;
                    }
                }
            }
            cnt = min(cnt + 1, k);
        }
    }
    const size_t row = (size_t)q * (size_t)k;
#pragma unroll
    for (int t = 0; t < kWarpSlots; ++t) {
        const int s = t * 32 + lane;
        if (s < k) {
            const bool filled = s < cnt;
            const float d = filled ? ld[t] : INFINITY;
            if (dist) dist[row + s] = sqrtf(d);
            if (sqdist) sqdist[row + s] = d;
            idx64[row + s] = filled ? sp.obase + (int64_t)li[t] : -1;
        }
    }
}

// --------------------------------------------------------------------------
// Warp per query, k <= 32 (D == 3).  Eight queries of one cloud per CTA share
// a reference tile of kWqTile points in shared memory.
//
// Each warp step covers 128 references as four 32-point chunks; lane l takes
// point l of every chunk, and the four distances are evaluated as two packed
// f32x2 pairs with the query duplicated in both halves -- half the issue
// slots of scalar distances.  The tile is stored for that access: for step s
// and lane l, A = (x, x', y, y') of chunk points 0 and 1, B the same for
// chunks 2 and 3, Z = (z0, z1, z2, z3), so a lane's three loads are
// consecutive across the warp (conflict-free).  Candidates are offered chunk
// by chunk, in index order, with the bar updated between chunks.
//
// Selection (FAISS-style warp select): the 32 best so far live sorted across
// the warp, one 64-bit key per lane (the ordered bits of the squared distance
// << 32 | index; every NaN maps above +inf, which is the order of every
// policy here, so the key order is the (SD, index) order).  A chunk's points
// that are admissible and not above the bar (the SD of rank k - 1) are
// appended to a 32-entry per-warp buffer in shared memory through one ballot
// (prefix popcounts give the slots); a full buffer is merged into the list by
// one bitonic sort of the buffer across the lanes and one bitonic merge.  The
// bar is stale between merges, which only admits more candidates, so every
// point of the final top k passes it.  This replaced a per-candidate insertion
// (replace the worst entry, two redux.sync to find the next worst) that made
// the kernel ALU-bound.  One min over a lane's
// four distances and one ballot against the bar skip a step without
// candidates (fminf ignores NaN, which can only enter a list whose rank k - 1
// is empty or NaN; the bar then lets every lane through).
constexpr int kWqWarps = 8;
constexpr int kWqTile = 2048;  // multiple of 128
constexpr uint32_t kEmptyKey = 0xffffffffu;

__device__ __forceinline__ uint32_t sd_key(float d) {
    return isnan(d) ? kEmptyKey : ordered_key(d);
}

// The k-th smallest (k <= 32) of 64 values held two per lane (va: element
// lane, vb: element 32 + lane), by a warp bitonic sort; every lane gets it.
__device__ __forceinline__ float warp_kth_of_64(float va, float vb, int k) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 32) {
                // Partner of element lane is element 32 + lane (same lane).
                const bool up = (lane & size) == 0;  // size == 64: always ascending
                const float lo = fminf(va, vb), hi = fmaxf(va, vb);
                va = up ? lo : hi;
                vb = up ? hi : lo;
            } else {
                const float oa = __shfl_xor_sync(FULL_MASK, va, stride);
                const float ob = __shfl_xor_sync(FULL_MASK, vb, stride);
                const bool lower = (lane & stride) == 0;
                const bool upa = (lane & size) == 0, upb = ((32 + lane) & size) == 0;
                va = (lower == upa) ? fminf(va, oa) : fmaxf(va, oa);
                vb = (lower == upb) ? fminf(vb, ob) : fmaxf(vb, ob);
            }
        }
    }
    return __shfl_sync(FULL_MASK, va, k - 1);
}

template <int POLICY, bool FLAT>
__global__ void __launch_bounds__(kWqWarps * 32)
knn_wq3_kernel(const float* __restrict__ query, const float* __restrict__ ref, Layout L, int k,
               float* __restrict__ dist, int64_t* __restrict__ idx64,
               int32_t* __restrict__ idx32, float* __restrict__ sqdist) {
    __shared__ float4 tA[kWqTile / 4], tB[kWqTile / 4], tZ[kWqTile / 4];
    __shared__ unsigned long long s_buf[kWqWarps * 32];  // per-warp candidate buffers
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    Span sp;
    if (!locate<FLAT>(L, kWqWarps, sp)) return;  // CTA-uniform
    const int64_t q = sp.q0 + warp;
    const bool active = q < sp.q1;
    const int64_t N = sp.n;
    const float* __restrict__ r = ref + (size_t)sp.r0 * 3;
    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (active) {
        const float* qp = query + (size_t)q * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    const f32x2 X = pack2(qx, qx), Y = pack2(qy, qy), Z = pack2(qz, qz);
    // The 32 best so far, sorted across the warp: lane s holds rank s as a
    // 64-bit key (ordered SD bits << 32 | index); empty ranks are all ones.
    unsigned long long best = ~0ull;
    float thr = INFINITY;  // SD of rank k - 1; +inf while that rank is empty
    // Exact upper bound of the k-th smallest SD: lane l keeps the minimum SD of
    // two buckets of points (chunks 0-1 and 2-3 of every step); the k-th
    // smallest of the 64 bucket minima is the SD of k distinct points, so no
    // point above it can be among the k nearest.  A pass over the first tile
    // before its candidate scan computes it, so the scan starts with a bar
    // near the final one instead of +inf and merges far fewer candidates.
    float bkt0 = INFINITY, bkt1 = INFINITY, ubound = INFINITY;
    unsigned long long* const buf = s_buf + warp * 32;
    int bc = 0;  // candidates waiting in buf (warp-uniform)
    // Merge the bc buffered candidates into `best`: bitonic sort of the
    // buffer across the lanes, then the 32 smallest of both sorted lists
    // (min of rank i and reversed rank 31 - i: a bitonic sequence) and a
    // bitonic clean; thr follows rank k - 1.
    auto merge = [&]() {
        __syncwarp();
        unsigned long long b = lane < bc ? buf[lane] : ~0ull;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                const unsigned long long o = __shfl_xor_sync(FULL_MASK, b, stride);
                const bool keep_min = ((lane & size) == 0) == ((lane & stride) == 0);
                b = keep_min ? (o < b ? o : b) : (o < b ? b : o);
            }
        }
        const unsigned long long rb = __shfl_sync(FULL_MASK, b, 31 - lane);
        best = rb < best ? rb : best;
#pragma unroll
        for (int stride = 16; stride > 0; stride >>= 1) {
            const unsigned long long o = __shfl_xor_sync(FULL_MASK, best, stride);
            const bool lower = (lane & stride) == 0;
            best = lower ? (o < best ? o : best) : (o < best ? best : o);
        }
        const unsigned long long kth = __shfl_sync(FULL_MASK, best, k - 1);
        const uint32_t kk = (uint32_t)(kth >> 32);
        // A NaN (three_nn) or empty rank k - 1 lets every candidate through.
        thr = kk != kEmptyKey ? ordered_key_inv(kk)
                              : ((uint32_t)kth >= 0x80000000u ? INFINITY : __int_as_float(0x7fffffff));
        thr = fminf(thr, ubound);
        bc = 0;
        __syncwarp();
    };
    // Tile fill: tile point p is point l = p % 32 of chunk v = (p / 32) % 4 of
    // step p / 128.  Thread t stores points t, t + 256, ...; l and v are fixed
    // per thread, so each thread always writes the same fields.
    const int fl = threadIdx.x & 31, fv = (threadIdx.x >> 5) & 3;
    float* const fxy = reinterpret_cast<float*>(fv < 2 ? tA : tB) + (fv & 1);
    float* const fz = reinterpret_cast<float*>(tZ) + fv;
    const unsigned lt = (1u << lane) - 1u;
    for (int64_t t0 = 0; t0 < N; t0 += kWqTile) {
        const int tn = (int)min64(kWqTile, N - t0);
        __syncthreads();
        for (int p = threadIdx.x; p < tn; p += kWqWarps * 32) {
            const float* rp = r + (size_t)(t0 + p) * 3;
            const int e = 4 * ((p >> 7) * 32 + fl);  // float offset of (step, lane)
            fxy[e] = rp[0];
            fxy[e + 2] = rp[1];
            fz[e] = rp[2];
        }
        __syncthreads();
        if (!active) continue;
        // Bound pass over the first tile only (points past tn are not in
        // it): afterwards the list's own rank k - 1 is about as tight, and
        // re-scanning every tile of a long cloud costs more than it saves.
        for (int c0 = 0; c0 < (t0 == 0 ? tn : 0); c0 += 128) {
            const int g = (c0 >> 2) + lane;
            const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(tA + g);
            const ulonglong2 b = *reinterpret_cast<const ulonglong2*>(tB + g);
            const ulonglong2 z = *reinterpret_cast<const ulonglong2*>(tZ + g);
            float d[4];
            unpack2(sqd3x2(X, Y, Z, a.x, a.y, z.x), d[0], d[1]);
            unpack2(sqd3x2(X, Y, Z, b.x, b.y, z.y), d[2], d[3]);
            const int e = c0 + lane;
            // fminf ignores NaN; a +inf or dropped point only loosens the bound.
            bkt0 = fminf(bkt0, fminf(e < tn ? d[0] : INFINITY, e + 32 < tn ? d[1] : INFINITY));
            bkt1 = fminf(bkt1, fminf(e + 64 < tn ? d[2] : INFINITY, e + 96 < tn ? d[3] : INFINITY));
        }
        if (t0 == 0) {
            ubound = warp_kth_of_64(bkt0, bkt1, k);
            thr = fminf(thr, ubound);
        }
        for (int c0 = 0; c0 < tn; c0 += 128) {
            const int g = (c0 >> 2) + lane;
            const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(tA + g);
            const ulonglong2 b = *reinterpret_cast<const ulonglong2*>(tB + g);
            const ulonglong2 z = *reinterpret_cast<const ulonglong2*>(tZ + g);
            float d[4];
            unpack2(sqd3x2(X, Y, Z, a.x, a.y, z.x), d[0], d[1]);
            unpack2(sqd3x2(X, Y, Z, b.x, b.y, z.y), d[2], d[3]);
            const float m = fminf(fminf(d[0], d[1]), fminf(d[2], d[3]));
            if (__ballot_sync(FULL_MASK, !(m > thr)) == 0u) continue;
            // Buffer every admissible point not above the bar (stale between
            // merges: it only ever admits more); a full buffer is merged
            // first and the chunk re-filtered against the new bar.
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int e = c0 + 32 * v + lane;
                bool cand = e < tn && !(d[v] > thr) && admissible<POLICY>(d[v]);
                unsigned mk = __ballot_sync(FULL_MASK, cand);
                if (mk == 0u) continue;
                if (bc + __popc(mk) > 32) {
                    merge();
                    cand = cand && !(d[v] > thr);
                    mk = __ballot_sync(FULL_MASK, cand);
                }
                if (cand) {
                    buf[bc + __popc(mk & lt)] =
                        ((unsigned long long)sd_key(d[v]) << 32) | (uint32_t)(t0 + e);
                }
                bc += __popc(mk);
            }
        }
    }
    if (!active) return;
    if (bc > 0) merge();
    if (lane >= k) return;
    const size_t row = (size_t)q * (size_t)k;
    const uint32_t lx = (uint32_t)best;
    const bool filled = lx < 0x80000000u;  // real rows are below 2**31
    const float ld = ordered_key_inv((uint32_t)(best >> 32));
    const float dd = filled ? ld : INFINITY;
    if (dist) dist[row + lane] = sqrtf(dd);
    if (sqdist) sqdist[row + lane] = dd;
    if (idx64) idx64[row + lane] = filled ? sp.obase + (int64_t)lx : -1;
    if (idx32) idx32[row + lane] = filled ? (int32_t)lx : -1;
}

// Grid of a search launch: (ceil(M / qpc), B) dense, virtual tiles flat.
inline dim3 search_grid(const Layout& L, int64_t B, int qpc, bool flat) {
    if (flat) return dim3((unsigned)flat_tiles(L.M, L.segs, qpc), 1u);
    return dim3((unsigned)ceil_div(L.M, qpc), (unsigned)B);
}

template <int POLICY, bool FLAT = false>
int launch_wq3(const float* query, const float* ref, const Layout& L, int64_t B, int k,
               float* dist, int64_t* idx64, int32_t* idx32, float* sqdist, cudaStream_t s) {
    knn_wq3_kernel<POLICY, FLAT><<<search_grid(L, B, kWqWarps, FLAT), kWqWarps * 32, 0, s>>>(
        query, ref, L, k, dist, idx64, idx32, sqdist);
    return check_launch("knn_wq3_kernel");
}

// Warp-per-query for moderate clouds; thread-per-query (rare, non-divergent
// insertions relative to a long scan) for very large reference clouds.
inline bool use_wq3(int64_t N) { return N <= (int64_t)1 << 18; }

int choose_splits(int64_t B, int64_t M, int64_t N) {
    const int64_t want = (int64_t)sm_count() * 1024;
    int S = 1;
    while (S < 8 && B * M * S < want && N / (kTile / (S * 2)) > 0 && kTile / (S * 2) >= 32) S *= 2;
    return S;
}

template <int K, int POLICY>
int launch_knn3(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int k,
                float* dist, int64_t* idx64, int32_t* idx32, float* sqdist, cudaStream_t s) {
    const int S = choose_splits(B, M, N);
    const int qpc = kThreads / S;
    size_t smem = 2 * kTile * sizeof(float4) + (size_t)kQueue * kThreads * 8;
    const size_t merge = (size_t)kThreads * K * 8;
    if (merge > smem) smem = merge;
    auto kern = knn3_kernel<K, POLICY>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    dim3 grid((unsigned)ceil_div(M, qpc), (unsigned)B);
    kern<<<grid, kThreads, smem, s>>>(query, ref, M, N, k, S, dist, idx64, idx32, sqdist);
    return check_launch("knn3_kernel");
}

// max_n: the longest reference cloud (segment) of the launch.
template <int K, int POLICY, bool FLAT = false>
int launch_knn3p(const float* query, const float* ref, const Layout& L, int64_t B,
                 int64_t max_n, int k, float* dist, int64_t* idx64, int32_t* idx32,
                 float* sqdist, cudaStream_t s) {
    const int S = choose_splits(B, L.M, max_n);
    const int qpc = kThreads / S;
    size_t smem = (size_t)(kTile + kTile / 2) * sizeof(float4) + (size_t)kQueue * kThreads * 8;
    const size_t merge = (size_t)kThreads * K * 8;
    if (merge > smem) smem = merge;
    auto kern = knn3p_kernel<K, POLICY, FLAT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    kern<<<search_grid(L, B, qpc, FLAT), kThreads, smem, s>>>(query, ref, L, k, S, dist, idx64,
                                                              idx32, sqdist);
    return check_launch("knn3p_kernel");
}

// Splits for knn3t_kernel: enough threads for about 256 per SM; each split
// keeps its own list, so fewer splits mean fewer list updates per point
// (three_nn at config 1: 0.059 / 0.047 / 0.057 / 0.082 ms with about 128 /
// 256 / 512 / 1024 threads per SM).
template <int POLICY, bool FLAT = false>
int launch_knn3t(const float* query, const float* ref, const Layout& L, int64_t B,
                 int64_t max_n, int k, float* dist, int64_t* idx64, int32_t* idx32,
                 float* sqdist, cudaStream_t s) {
    const int64_t want = (int64_t)sm_count() * 256;
    int S = 1;
    while (S < 8 && B * L.M * S < want && max_n >= (int64_t)kTile / S) S *= 2;
    const int qpc = kThreads / S;
    const size_t smem = (size_t)(kTile + kTile / 2) * sizeof(float4);
    auto kern = knn3t_kernel<POLICY, FLAT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    kern<<<search_grid(L, B, qpc, FLAT), kThreads, smem, s>>>(query, ref, L, k, S, dist, idx64,
                                                              idx32, sqdist);
    return check_launch("knn3t_kernel");
}

template <int K, bool FLAT = false>
int launch_knnd(const float* query, const float* ref, const Layout& L, int64_t B, int D, int k,
                float* dist, int64_t* idx64, float* sqdist, cudaStream_t s) {
    int S = 1;
    while (S < 4 && B * L.M * S < (int64_t)sm_count() * 512) S *= 2;
    const int qpc = kFeatThreads / S;
    int tileN = 64 * S;
    size_t smem = ((size_t)qpc * (D + 1) + (size_t)tileN * D) * sizeof(float);
    while (smem > 200 * 1024 && tileN > S) {
        tileN /= 2;
        smem = ((size_t)qpc * (D + 1) + (size_t)tileN * D) * sizeof(float);
    }
    if (smem > 200 * 1024) return fail(kUnsupported, "knn: feature dimension too large");
    const size_t merge = (size_t)kFeatThreads * K * 8;
    if (merge > smem) smem = merge;
    auto kern = knnd_kernel<K, kDropNonFinite, FLAT>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    kern<<<search_grid(L, B, qpc, FLAT), kFeatThreads, smem, s>>>(query, ref, L, D, k, S, tileN,
                                                                  dist, idx64, sqdist);
    return check_launch("knnd_kernel");
}

// Exact kNN over a dense or flat layout.  POLICY3 is the candidate policy for
// D == 3 (every D != 3 search drops non-finite distances); max_n is the
// longest reference cloud or segment, which picks the D == 3 kernel.
template <int POLICY3, bool FLAT>
int run_knn(const float* query, const float* ref, const Layout& L, int64_t B, int64_t max_n,
            int64_t D, int k, float* dist, int64_t* idx, float* sqdist, cudaStream_t s) {
    if (D == 3 && k <= 3)
        return launch_knn3t<POLICY3, FLAT>(query, ref, L, B, max_n, k, dist, idx, nullptr, sqdist,
                                           s);
    if (D == 3 && k <= 32 && use_wq3(max_n))
        return launch_wq3<POLICY3, FLAT>(query, ref, L, B, k, dist, idx, nullptr, sqdist, s);
    if (D == 3 && k <= 32) {
        if (k <= 4) return launch_knn3p<4, POLICY3, FLAT>(query, ref, L, B, max_n, k, dist, idx, nullptr, sqdist, s);
        if (k <= 8) return launch_knn3p<8, POLICY3, FLAT>(query, ref, L, B, max_n, k, dist, idx, nullptr, sqdist, s);
        if (k <= 16) return launch_knn3p<16, POLICY3, FLAT>(query, ref, L, B, max_n, k, dist, idx, nullptr, sqdist, s);
        return launch_knn3p<32, POLICY3, FLAT>(query, ref, L, B, max_n, k, dist, idx, nullptr, sqdist, s);
    }
    if (D != 3 && D <= 4096 && k <= 32) {
        if (k <= 4) return launch_knnd<4, FLAT>(query, ref, L, B, (int)D, k, dist, idx, sqdist, s);
        if (k <= 8) return launch_knnd<8, FLAT>(query, ref, L, B, (int)D, k, dist, idx, sqdist, s);
        if (k <= 16) return launch_knnd<16, FLAT>(query, ref, L, B, (int)D, k, dist, idx, sqdist, s);
        return launch_knnd<32, FLAT>(query, ref, L, B, (int)D, k, dist, idx, sqdist, s);
    }
    // Large k (or very wide features): warp per query.
    const dim3 grid = search_grid(L, B, kWarpQueries, FLAT);
    if (D == 3)
        knn_warp_kernel<POLICY3, FLAT><<<grid, 32 * kWarpQueries, 0, s>>>(query, ref, L, (int)D, k,
                                                                         dist, idx, sqdist);
    else
        knn_warp_kernel<kDropNonFinite, FLAT><<<grid, 32 * kWarpQueries, 0, s>>>(
            query, ref, L, (int)D, k, dist, idx, sqdist);
    return check_launch("knn_warp_kernel");
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_knn_workspace_bytes(int64_t B, int64_t M, int64_t N, int64_t D, int64_t k) {
    if (B <= 0 || M <= 0 || !mpo::fknn_tc_eligible(M, N, D, k)) return 0;
    return mpo::fknn_tc_workspace_bytes(B, M, N, D);
}

int mpo_knn(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int64_t D,
            int64_t k, float* dist, int64_t* idx, float* sqdist, void* workspace,
            size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && M >= 0 && N >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE(k >= 0 && k <= N, "k must be in [0, N]");
    MPO_REQUIRE(k <= 256, "k must be at most 256");
    MPO_REQUIRE(N < (int64_t)0x7fffffff && M < (int64_t)0x7fffffff, "M and N must be below 2**31");
    if (B == 0 || M == 0 || k == 0) return kOk;
    MPO_REQUIRE(query && ref && dist && idx, "null pointer");
    MPO_REQUIRE_WORKSPACE(workspace);
    cudaStream_t s = (cudaStream_t)stream;
    if (fknn_tc_eligible(M, N, D, k))
        return fknn_tc_run(query, ref, B, M, N, D, k, dist, idx, sqdist, workspace,
                           workspace_bytes, s);
    return run_knn<kDropNaN, false>(query, ref, dense_layout(M, N), B, N, D, (int)k, dist, idx,
                                    sqdist, s);
}

int mpo_flat_knn(const float* x, const float* y, const int64_t* ptr_x, const int64_t* ptr_y,
                 int64_t segments, int64_t nx, int64_t ny, int64_t D, int64_t k,
                 int64_t max_segment_x, int64_t* out, int32_t* status, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(segments >= 0 && nx >= 0 && ny >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE(k >= 0 && k <= 256, "k must be in [0, 256]");
    MPO_REQUIRE(nx < (int64_t)0x7fffffff && ny < (int64_t)0x7fffffff,
                "the flat row counts must be below 2**31");
    MPO_REQUIRE(status != nullptr, "status must not be null");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(status, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(kCudaError, "mpo_flat_knn: status reset failed");
    if (ny == 0 || k == 0) return kOk;
    MPO_REQUIRE(segments >= 1, "a nonempty query set needs at least one segment");
    MPO_REQUIRE(y && ptr_x && ptr_y && out && (x || nx == 0), "null pointer");
    int st = flat_offsets_check(ptr_y, ptr_x, segments, ny, nx, status, s);
    if (st) return st;
    Layout L{ny, nx, ptr_y, ptr_x, segments, status};
    const int64_t max_n = max64(0, min64(max_segment_x, nx));
    return run_knn<kDropNonFinite, true>(y, x, L, 1, max_n, D, (int)k, nullptr, out, nullptr,
                                         s);
}

int mpo_three_nn(const float* unknown, const float* known, int64_t B, int64_t N, int64_t M,
                 float* dist, int32_t* idx, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && M >= 0, "bad sizes");
    if (B == 0 || N == 0) return kOk;
    MPO_REQUIRE(M >= 3, "three_nn needs at least 3 known points");
    MPO_REQUIRE(M < (int64_t)0x7fffffff, "M must be below 2**31");
    MPO_REQUIRE(unknown && known && dist && idx, "null pointer");
    return launch_knn3t<kNaNLast>(unknown, known, dense_layout(N, M), B, M, 3, dist, nullptr,
                                  idx, nullptr, (cudaStream_t)stream);
}

}  // extern "C"
