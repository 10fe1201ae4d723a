// Squared-L2 Chamfer nearest-neighbour search, its backward and its input
// check, on sm_100a.
//
// Contract: gamzerA/mps-pointops mps_pointops/chamfer.py:161-212 and 297-308
// (norm = 2): for each query row i < query_lengths[b], the FIRST reference
// index j < ref_lengths[b] with the smallest SD; if every SD overflows to
// +inf the first valid reference (index 0) is still selected; dist = SD of the
// selected pair.  Padded query rows and clouds without a valid reference give
// (dist 0, index -1).  Backward: chamfer.py:227-251.
//
// Design (B200), per direction:
//   * One thread owns one (query, split); a CTA of 256 threads covers 256/S
//     queries of one cloud and S splits.  Reference tiles of 1024 points are
//     staged as float4 in shared memory (double-buffered through registers)
//     and read with warp-broadcast loads.
//   * Hot loop: 4 distances, their minimum (3 min ops) and ONE compare with
//     the running best; only when the block minimum improves does the thread
//     locate the first position attaining it.  Within a thread indices grow,
//     so strict < keeps the lowest index; splits merge with (SD, index) order.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kThreads = 256;
constexpr int kTile = 1024;
constexpr uint32_t kNone = 0xffffffffu;

// L1 distance for D == 3: (|dx| + |dy|) + |dz|, each operation rounded.
__device__ __forceinline__ float l1d3(float ax, float ay, float az, float bx, float by,
                                      float bz) {
    return __fadd_rn(__fadd_rn(fabsf(__fsub_rn(ax, bx)), fabsf(__fsub_rn(ay, by))),
                     fabsf(__fsub_rn(az, bz)));
}

// NORM 2: squared L2; NORM 1: L1.
template <int NORM>
__device__ __forceinline__ float dist3(float ax, float ay, float az, float bx, float by,
                                       float bz) {
    return NORM == 1 ? l1d3(ax, ay, az, bx, by, bz) : sqd3(ax, ay, az, bx, by, bz);
}

// Packed forms for two (a, b) pairs: NORM 2 sqd3x2; NORM 1 ((|d0| + |d1|) +
// |d2|), the absolute values by clearing both sign bits (exact).
__device__ __forceinline__ f32x2 abs2(f32x2 v) { return v & 0x7fffffff7fffffffull; }
template <int NORM>
__device__ __forceinline__ f32x2 dist3x2(f32x2 ax, f32x2 ay, f32x2 az, f32x2 bx, f32x2 by,
                                         f32x2 bz) {
    if (NORM == 2) return sqd3x2(ax, ay, az, bx, by, bz);
    return add2(add2(abs2(sub2(ax, bx)), abs2(sub2(ay, by))), abs2(sub2(az, bz)));
}

template <int NORM>
__global__ void __launch_bounds__(kThreads)
nearest3_kernel(const float* __restrict__ query, const float* __restrict__ ref,
                const int64_t* __restrict__ query_lengths, const int64_t* __restrict__ ref_lengths,
                int64_t M, int64_t N, int S, float* __restrict__ out_dist,
                int64_t* __restrict__ out_idx) {
    extern __shared__ float4 tile[];  // [2][kTile]
    __shared__ float m_d[kThreads];
    __shared__ uint32_t m_i[kThreads];
    const int b = blockIdx.y;
    const int qpc = kThreads / S;
    const int tid = threadIdx.x;
    const int split = tid / qpc;
    const int ql = tid % qpc;
    const int64_t q = (int64_t)blockIdx.x * qpc + ql;
    const int64_t qlen = query_lengths ? query_lengths[b] : M;
    const int64_t nl = ref_lengths ? min64(ref_lengths[b], N) : N;
    const bool active = q < M && q < qlen;
    const float* __restrict__ r = ref + (size_t)b * (size_t)N * 3;

    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (active) {
        const float* qp = query + ((size_t)b * (size_t)M + (size_t)q) * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    float bd = INFINITY;
    uint32_t bj = kNone;

    const int64_t ntiles = ceil_div(nl, kTile);
    const int slice = kTile / S;
    constexpr int kLoads = 3 * kTile / kThreads;
    float pre[kLoads];
#define MPO_LOAD_TILE(t)                                                   \
    do {                                                                   \
        const int64_t base_ = (t) * kTile * 3;                             \
        _Pragma("unroll") for (int u = 0; u < kLoads; ++u) {               \
            const int64_t e_ = base_ + tid + (int64_t)u * kThreads;        \
            pre[u] = e_ < nl * 3 ? r[e_] : 0.f;                            \
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
    if (ntiles > 0) {
        MPO_LOAD_TILE(0);
        MPO_STORE_TILE(0);
    }
    __syncthreads();
    for (int64_t t = 0; t < ntiles; ++t) {
        const int buf = (int)(t & 1);
        if (t + 1 < ntiles) MPO_LOAD_TILE(t + 1);
        if (active) {
            const float4* tp = tile + buf * kTile + split * slice;
            const int64_t j0 = t * kTile + (int64_t)split * slice;
            const int cnt = (int)max64(0, min64(slice, nl - j0));
            int e = 0;
            for (; e + 4 <= cnt; e += 4) {
                float dd[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 p = tp[e + u];
                    dd[u] = dist3<NORM>(qx, qy, qz, p.x, p.y, p.z);
                }
                const float m = fminf(fminf(dd[0], dd[1]), fminf(dd[2], dd[3]));
                if (m < bd) {
                    const int u = dd[0] == m ? 0 : dd[1] == m ? 1 : dd[2] == m ? 2 : 3;
                    bd = m;
                    bj = (uint32_t)(j0 + e + u);
                }
            }
            for (; e < cnt; ++e) {
                const float4 p = tp[e];
                const float d = dist3<NORM>(qx, qy, qz, p.x, p.y, p.z);
                if (d < bd) {
                    bd = d;
                    bj = (uint32_t)(j0 + e);
                }
            }
        }
        if (t + 1 < ntiles) MPO_STORE_TILE(buf ^ 1);
        __syncthreads();
    }
#undef MPO_LOAD_TILE
#undef MPO_STORE_TILE
    if (S > 1) {
        m_d[tid] = bd;
        m_i[tid] = bj;
        __syncthreads();
        if (split == 0) {
            for (int o = 1; o < S; ++o) {
                const float d = m_d[o * qpc + ql];
                const uint32_t j = m_i[o * qpc + ql];
                if (j != kNone && (bj == kNone || d < bd || (d == bd && j < bj))) {
                    bd = d;
                    bj = j;
                }
            }
        }
    }
    if (split != 0 || q >= M) return;
    const size_t o = (size_t)b * (size_t)M + (size_t)q;
    if (!active || nl <= 0) {
        out_dist[o] = 0.f;
        out_idx[o] = -1;
        return;
    }
    if (bj == kNone) {  // every SD overflowed: the first valid reference
        bj = 0;
        bd = dist3<NORM>(qx, qy, qz, r[0], r[1], r[2]);
    }
    out_dist[o] = bd;
    out_idx[o] = (int64_t)bj;
}

// --------------------------------------------------------------------------
// Symmetric D == 3 search: every (x_i, y_j) squared distance is evaluated
// ONCE and feeds both the row minimum (x -> y) and the column minimum
// (y -> x).
//
// Work item = (cloud, 1024 x-rows, 1024 y-columns); CTAs take items from an
// atomic counter.  The y tile is staged in shared memory so that warp-
// broadcast loads yield packed f32x2 operands: one float4 (y.x, y.x, y.y,
// y.y) per column and one float4 (z_j, z_j, z_j+1, z_j+1) per column pair
// (three 16-byte loads per two columns).  Lane l of warp w owns x-rows
// i0 + (32 w + l) * R .. + R - 1 (contiguous, so row order = (warp, lane, k)),
// packed two per f32x2 register, and a warp walks the columns together:
//   * rows: a running minimum over blocks of C columns (one min per pair),
//     compared with the row's best once per block as raw bits (SD >= 0, so
//     bit order == value order); the column inside the winning block is
//     recovered at the end of the item by recomputing C distances;
//   * columns: the lane's minimum over its R rows, then one redux.sync.min
//     over the warp and one ballot of the lanes holding it; the C records of
//     a block are kept in registers and written once per block as 64-bit
//     (min bits, lane mask) words (lane c stores column c).  At the end of
//     the item a thread per column picks the first warp, the first lane and
//     (recomputing R distances) the first row holding the minimum.
// Both directions are committed as 64-bit keys (SD bits << 32 | index) with
// atomicMin into global scratch, which yields the smallest SD and, among
// equal SDs, the lowest index -- the reference's first-minimum rule.
// Padding (index >= length) enters as +inf coordinates: it ties valid
// entries only at +inf and then loses on index, and padding-vs-padding pairs
// are NaN, which never wins a min.
//
// Cost model (B200, measured): a packed f32x2 op holds the FP32 pipe for two
// cycles, i.e. the pipe does 128 rounded fp32 ops per SM per clock whether
// packed or not; packing halves the issue slots the distance needs, so the
// min/ballot bookkeeping (about 3 issue slots per pair-row) is what separates
// the kernel from the FP32 bound of 8 ops per pair.
constexpr unsigned long long kMaxKeyAll = ~0ull;
namespace sym {
constexpr unsigned long long kMaxKey = kMaxKeyAll;

// Tile shape: kWarps warps, kR x-rows per lane (even: packed in pairs), kC
// columns per row-minimum block (even), kBN y-columns per item, kMinBlocks
// CTAs per SM for the register budget.
template <int kWarps, int kR, int kC, int kBN, int kMinBlocks>
struct Shape {
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kBM = kWarps * 32 * kR;
    static constexpr int kCols = kBN;
    static constexpr size_t kColBytes = (size_t)kBN * 16 + (size_t)kBN / 2 * 16;
    static constexpr size_t kSmem = kColBytes + (size_t)kWarps * kBN * 8;
};

template <int kWarps, int kR, int kC, int kBN, int kMinBlocks, int NORM = 2>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks)
chamfer_sym3_kernel(const float* __restrict__ x, const float* __restrict__ y,
                    const int64_t* __restrict__ x_lengths, const int64_t* __restrict__ y_lengths,
                    int64_t B, int64_t P, int64_t Q, unsigned long long* __restrict__ keys_x,
                    unsigned long long* __restrict__ keys_y, unsigned* __restrict__ counter) {
    using S = Shape<kWarps, kR, kC, kBN, kMinBlocks>;
    extern __shared__ float4 smem4[];
    float4* s_xy = smem4;        // [kBN]      (y.x, y.x, y.y, y.y)
    float4* s_z = smem4 + kBN;   // [kBN / 2]  (z_2i, z_2i, z_2i+1, z_2i+1)
    unsigned long long* s_part =
        reinterpret_cast<unsigned long long*>(reinterpret_cast<unsigned char*>(smem4) + S::kColBytes);
    __shared__ unsigned s_item;
    constexpr int kThreads = S::kThreads;
    constexpr int kBM = S::kBM;
    static_assert(kR % 2 == 0 && kC % 2 == 0 && kC <= 32 && kBN % kC == 0, "bad tile shape");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row_blocks = ceil_div(P, kBM), col_blocks = ceil_div(Q, kBN);
    const int64_t per_cloud = row_blocks * col_blocks, total = B * per_cloud;
    const float* s_zf = reinterpret_cast<const float*>(s_z);

    for (;;) {
        if (tid == 0) s_item = atomicAdd(counter, 1u);
        __syncthreads();
        const int64_t item = s_item;
        __syncthreads();
        if (item >= total) break;
        const int64_t b = item / per_cloud;
        const int64_t rem = item % per_cloud;
        const int64_t i0 = (rem / col_blocks) * kBM, j0 = (rem % col_blocks) * kBN;
        const int64_t xlen = x_lengths ? min64(max64(x_lengths[b], 0), P) : P;
        const int64_t ylen = y_lengths ? min64(max64(y_lengths[b], 0), Q) : Q;
        if (i0 >= xlen || j0 >= ylen) continue;  // uniform: nothing valid here
        const float* __restrict__ xb = x + (size_t)b * P * 3;
        const float* __restrict__ yb = y + (size_t)b * Q * 3;

        float* s_zw = reinterpret_cast<float*>(s_z);
        for (int e = tid; e < kBN; e += kThreads) {
            const int64_t j = j0 + e;
            float px = INFINITY, py = INFINITY, pz = INFINITY;
            if (j < ylen) {
                px = yb[3 * j];
                py = yb[3 * j + 1];
                pz = yb[3 * j + 2];
            }
            s_xy[e] = make_float4(px, px, py, py);
            s_zw[2 * e] = pz;
            s_zw[2 * e + 1] = pz;
        }
        const int64_t rbase = i0 + (int64_t)(warp * 32 + lane) * kR;
        f32x2 X[kR / 2], Y[kR / 2], Z[kR / 2];
#pragma unroll
        for (int q = 0; q < kR / 2; ++q) {
            float c[6];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t r = rbase + 2 * q + h;
                const bool ok = r < xlen;
                c[3 * h + 0] = ok ? xb[3 * r + 0] : INFINITY;
                c[3 * h + 1] = ok ? xb[3 * r + 1] : INFINITY;
                c[3 * h + 2] = ok ? xb[3 * r + 2] : INFINITY;
            }
            X[q] = pack2(c[0], c[3]);
            Y[q] = pack2(c[1], c[4]);
            Z[q] = pack2(c[2], c[5]);
        }
        __syncthreads();

        uint32_t best[kR];
        int blk[kR];
#pragma unroll
        for (int k = 0; k < kR; ++k) {
            best[k] = 0xffffffffu;
            blk[k] = -1;
        }
        for (int jb = 0; jb < kBN; jb += kC) {
            float m[kR];
            unsigned pmin[kC], pmask[kC];
#pragma unroll
            for (int c2 = 0; c2 < kC; c2 += 2) {
                const ulonglong2 a0 = *reinterpret_cast<const ulonglong2*>(&s_xy[jb + c2]);
                const ulonglong2 a1 = *reinterpret_cast<const ulonglong2*>(&s_xy[jb + c2 + 1]);
                const ulonglong2 zz = *reinterpret_cast<const ulonglong2*>(&s_z[(jb + c2) >> 1]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = c2 + h;
                    const ulonglong2 a = h ? a1 : a0;
                    const f32x2 bz = h ? zz.y : zz.x;
                    float d[kR];
#pragma unroll
                    for (int q = 0; q < kR / 2; ++q) {
                        const f32x2 dd = dist3x2<NORM>(X[q], Y[q], Z[q], a.x, a.y, bz);
                        unpack2(dd, d[2 * q], d[2 * q + 1]);
                    }
#pragma unroll
                    for (int k = 0; k < kR; ++k) m[k] = (c == 0) ? d[k] : fminf(m[k], d[k]);
                    float t[kR];
#pragma unroll
                    for (int k = 0; k < kR; ++k) t[k] = d[k];
#pragma unroll
                    for (int w2 = kR / 2; w2 >= 1; w2 /= 2) {
#pragma unroll
                        for (int k = 0; k < w2; ++k) t[k] = fminf(t[k], t[k + w2]);
                    }
                    const unsigned cb = __float_as_uint(t[0]);
                    pmin[c] = __reduce_min_sync(FULL_MASK, cb);
                    pmask[c] = __ballot_sync(FULL_MASK, cb == pmin[c]);
                }
            }
            if (lane < kC) {
                unsigned v = pmin[0], mk = pmask[0];
#pragma unroll
                for (int c = 1; c < kC; ++c) {
                    if (lane == c) {
                        v = pmin[c];
                        mk = pmask[c];
                    }
                }
                s_part[warp * kBN + jb + lane] = ((unsigned long long)v << 32) | mk;
            }
#pragma unroll
            for (int k = 0; k < kR; ++k) {
                const uint32_t mb = __float_as_uint(m[k]);
                if (mb < best[k]) {
                    best[k] = mb;
                    blk[k] = jb;
                }
            }
        }

        // Rows: recover the first column of the winning block and commit.
#pragma unroll
        for (int k = 0; k < kR; ++k) {
            const int64_t r = rbase + k;
            if (r < xlen && blk[k] >= 0) {
                float rx, ry, rz, t0, t1;
                unpack2(X[k / 2], t0, t1);
                rx = (k & 1) ? t1 : t0;
                unpack2(Y[k / 2], t0, t1);
                ry = (k & 1) ? t1 : t0;
                unpack2(Z[k / 2], t0, t1);
                rz = (k & 1) ? t1 : t0;
                int col = blk[k];
                for (int c = 0; c < kC; ++c) {
                    const int j = blk[k] + c;
                    const float4 pa = s_xy[j];
                    if (__float_as_uint(dist3<NORM>(rx, ry, rz, pa.x, pa.z, s_zf[2 * j])) ==
                        best[k]) {
                        col = j;
                        break;
                    }
                }
                atomicMin(&keys_x[(size_t)b * P + r],
                          ((unsigned long long)best[k] << 32) | (unsigned long long)(j0 + col));
            }
        }
        __syncthreads();
        // Columns: first warp, first lane, first row holding the minimum.
        for (int e = tid; e < kBN; e += kThreads) {
            const int64_t j = j0 + e;
            if (j >= ylen) continue;
            unsigned bv = 0xffffffffu, bm = 0u;
            int bw = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const unsigned long long pv = s_part[w * kBN + e];
                const unsigned v = (unsigned)(pv >> 32);
                if (v < bv) {
                    bv = v;
                    bw = w;
                    bm = (unsigned)pv;
                }
            }
            const int l = __ffs(bm) - 1;
            const int64_t r0 = i0 + (int64_t)(bw * 32 + l) * kR;
            const float4 pa = s_xy[e];
            const float pz = s_zf[2 * e];
            int64_t row = r0;
            for (int k = 0; k < kR; ++k) {
                const int64_t r = r0 + k;
                if (r >= xlen) break;
                const float d =
                    dist3<NORM>(xb[3 * r], xb[3 * r + 1], xb[3 * r + 2], pa.x, pa.z, pz);
                if (__float_as_uint(d) == bv) {
                    row = r;
                    break;
                }
            }
            atomicMin(&keys_y[(size_t)b * Q + j],
                      ((unsigned long long)bv << 32) | (unsigned long long)row);
        }
        __syncthreads();
    }
}

// Keys -> (squared distance, index) in the public layout; padded rows and
// clouds whose other side is empty give (0, -1).
__global__ void finalize_kernel(const unsigned long long* __restrict__ keys,
                                const int64_t* __restrict__ self_lengths,
                                const int64_t* __restrict__ other_lengths, int64_t B, int64_t M,
                                int64_t N, float* __restrict__ dist, int64_t* __restrict__ idx) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= B * M) return;
    const int64_t b = e / M, i = e % M;
    const int64_t len = self_lengths ? self_lengths[b] : M;
    const int64_t olen = other_lengths ? other_lengths[b] : N;
    const unsigned long long key = keys[e];
    if (i >= len || olen <= 0 || key == kMaxKey) {
        dist[e] = 0.f;
        idx[e] = -1;
        return;
    }
    dist[e] = __uint_as_float((unsigned)(key >> 32));
    idx[e] = (int64_t)(key & 0xffffffffull);
}

// The same with the keys held in the idx array itself (the allocation-free
// L1 entry): each thread reads its key before it writes its (dist, idx).
__global__ void finalize_inplace_kernel(int64_t* idx_keys, const int64_t* __restrict__ self_lengths,
                                        const int64_t* __restrict__ other_lengths, int64_t B,
                                        int64_t M, int64_t N, float* __restrict__ dist) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= B * M) return;
    const int64_t b = e / M, i = e % M;
    const int64_t len = self_lengths ? self_lengths[b] : M;
    const int64_t olen = other_lengths ? other_lengths[b] : N;
    const unsigned long long key = static_cast<unsigned long long>(idx_keys[e]);
    if (i >= len || olen <= 0 || key == kMaxKey) {
        dist[e] = 0.f;
        idx_keys[e] = -1;
        return;
    }
    dist[e] = __uint_as_float((unsigned)(key >> 32));
    idx_keys[e] = (int64_t)(key & 0xffffffffull);
}

inline bool use_sym(int64_t P, int64_t Q, int64_t D) { return D == 3 && P >= 512 && Q >= 512; }

// The tile shape used by mpo_chamfer_nearest.
#define MPO_SYM_DEFAULT 4, 8, 8, 1024, 3
using Default = Shape<MPO_SYM_DEFAULT>;

inline size_t scratch_bytes(int64_t B, int64_t P, int64_t Q) {
    return ((size_t)B * (P + Q)) * sizeof(unsigned long long) + 256;
}
}  // namespace sym

// ---------------------------------------------------------------------------
// Symmetric tile kernel for D != 3 (feature-space Chamfer, both directions
// from ONE evaluation per pair, like chamfer_sym3_kernel).  A CTA takes one
// item (cloud, kBM x rows, kBN y columns):
//   * x rows are staged transposed in shared memory, [D][kBM], so a lane's two
//     consecutive rows at dimension t are one packed f32x2 load; y columns as
//     (y_j, y_j, y_j+1, y_j+1) float4s, [kBN / 2][D], read by warp broadcast.
//   * Per block of kC = 8 columns the dimension loop accumulates the 16
//     distances of the lane's two rows in packed registers, in the
//     reference's order (s = d0*d0, then s = s + dt*dt; L1: |d0| + |d1| ...).
//   * Row minima: the block minimum per row in registers; the first column of
//     the winning block is recovered by recomputation.  Column minima: one
//     redux.sync.min and one ballot per (warp, column) into shared memory,
//     then the first warp, lane and row holding it.  Both directions commit
//     64-bit keys (distance bits << 32 | index) with atomicMin, exactly as
//     the D == 3 kernel, so finalize_kernel and the fused loss serve both.
template <int kWarps, int kBN>
struct ShapeD {
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kBM = kThreads * 2;  // two rows per lane
    static constexpr int kC = 8;
    static size_t smem(int64_t D) {
        return (size_t)kBM * D * 4 + (size_t)(kBN / 2) * D * 16 + (size_t)kWarps * kBN * 8;
    }
};
// D <= 64: 8 warps x 128 columns (204,800 B of shared memory at D = 64);
// 64 < D <= 144: 4 warps x 64 columns (223,232 B at D = 144).
constexpr int64_t kSymDMaxSmall = 64;
constexpr int64_t kSymDMax = 144;

// One (row, column) distance recomputed from the staged tiles, scalar, in
// the same order and rounding as the packed loop.
template <int NORM>
__device__ __forceinline__ float symd_dist(const float* __restrict__ sx, int kBM, int r,
                                           const float* __restrict__ sy, int col, int D) {
    const float* yc = sy + (size_t)(col >> 1) * D * 4 + (col & 1) * 2;
    float d = __fsub_rn(sx[r], yc[0]);
    float acc = NORM == 1 ? fabsf(d) : __fmul_rn(d, d);
    for (int t = 1; t < D; ++t) {
        d = __fsub_rn(sx[(size_t)t * kBM + r], yc[(size_t)t * 4]);
        acc = __fadd_rn(acc, NORM == 1 ? fabsf(d) : __fmul_rn(d, d));
    }
    return acc;
}

template <int kWarps, int kBN, int NORM>
__global__ void __launch_bounds__(kWarps * 32)
chamfer_symd_kernel(const float* __restrict__ x, const float* __restrict__ y,
                    const int64_t* __restrict__ x_lengths, const int64_t* __restrict__ y_lengths,
                    int64_t B, int64_t P, int64_t Q, int D,
                    unsigned long long* __restrict__ keys_x,
                    unsigned long long* __restrict__ keys_y) {
    using S = ShapeD<kWarps, kBN>;
    constexpr int kThreads = S::kThreads, kBM = S::kBM, kC = S::kC;
    extern __shared__ float4 smem4[];
    float* s_x = reinterpret_cast<float*>(smem4);                       // [D][kBM]
    float4* s_y = smem4 + (size_t)kBM * D / 4;                          // [kBN/2][D]
    unsigned long long* s_part =
        reinterpret_cast<unsigned long long*>(s_y + (size_t)(kBN / 2) * D);  // [kWarps][kBN]
    const float* s_yf = reinterpret_cast<const float*>(s_y);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row_blocks = ceil_div(P, kBM), col_blocks = ceil_div(Q, kBN);
    const int64_t item = blockIdx.x;
    const int64_t b = item / (row_blocks * col_blocks);
    const int64_t rem = item % (row_blocks * col_blocks);
    const int64_t i0 = (rem / col_blocks) * kBM, j0 = (rem % col_blocks) * kBN;
    const int64_t xlen = x_lengths ? min64(max64(x_lengths[b], 0), P) : P;
    const int64_t ylen = y_lengths ? min64(max64(y_lengths[b], 0), Q) : Q;
    if (i0 >= xlen || j0 >= ylen) return;  // uniform: nothing valid here
    const float* __restrict__ xb = x + (size_t)b * P * D;
    const float* __restrict__ yb = y + (size_t)b * Q * D;

    // Stage: a thread per x row (conflict-free transposed stores), a thread
    // per y column pair; padding is +inf (ties only at +inf, where the lower
    // valid index wins; padding x padding is NaN, which never wins).
    for (int r = tid; r < kBM; r += kThreads) {
        const int64_t gr = i0 + r;
        const bool ok = gr < xlen;
        const float* src = xb + (size_t)gr * D;
        for (int t = 0; t < D; ++t) s_x[(size_t)t * kBM + r] = ok ? src[t] : INFINITY;
    }
    for (int cp = tid; cp < kBN / 2; cp += kThreads) {
        const int64_t j = j0 + 2 * cp;
        const bool ok0 = j < ylen, ok1 = j + 1 < ylen;
        const float* s0 = yb + (size_t)j * D;
        for (int t = 0; t < D; ++t) {
            const float a = ok0 ? s0[t] : INFINITY;
            const float c = ok1 ? s0[D + t] : INFINITY;
            s_y[(size_t)cp * D + t] = make_float4(a, a, c, c);
        }
    }
    __syncthreads();

    const int lrow = (warp * 32 + lane) * 2;
    const f32x2* xcol = reinterpret_cast<const f32x2*>(s_x + lrow);  // stride kBM / 2 pairs
    uint32_t best[2] = {0xffffffffu, 0xffffffffu};
    int blk[2] = {-1, -1};
    for (int jb = 0; jb < kBN; jb += kC) {
        const ulonglong2* yv = reinterpret_cast<const ulonglong2*>(s_y + (size_t)(jb >> 1) * D);
        f32x2 acc[kC];
        {
            const f32x2 X = xcol[0];
#pragma unroll
            for (int cp = 0; cp < kC / 2; ++cp) {
                const ulonglong2 yy = yv[(size_t)cp * D];
                const f32x2 d0 = sub2(X, yy.x), d1 = sub2(X, yy.y);
                acc[2 * cp] = NORM == 1 ? abs2(d0) : sq2(d0);
                acc[2 * cp + 1] = NORM == 1 ? abs2(d1) : sq2(d1);
            }
        }
        for (int t = 1; t < D; ++t) {
            const f32x2 X = xcol[(size_t)t * (kBM / 2)];
#pragma unroll
            for (int cp = 0; cp < kC / 2; ++cp) {
                const ulonglong2 yy = yv[(size_t)cp * D + t];
                const f32x2 d0 = sub2(X, yy.x), d1 = sub2(X, yy.y);
                acc[2 * cp] = add2(acc[2 * cp], NORM == 1 ? abs2(d0) : sq2(d0));
                acc[2 * cp + 1] = add2(acc[2 * cp + 1], NORM == 1 ? abs2(d1) : sq2(d1));
            }
        }
        float m0 = INFINITY, m1 = INFINITY;
        unsigned pmin[kC], pmask[kC];
#pragma unroll
        for (int c = 0; c < kC; ++c) {
            float d0, d1;
            unpack2(acc[c], d0, d1);
            m0 = c == 0 ? d0 : fminf(m0, d0);
            m1 = c == 0 ? d1 : fminf(m1, d1);
            const unsigned cb = __float_as_uint(fminf(d0, d1));
            pmin[c] = __reduce_min_sync(FULL_MASK, cb);
            pmask[c] = __ballot_sync(FULL_MASK, cb == pmin[c]);
        }
        if (lane < kC) {
            unsigned v = pmin[0], mk = pmask[0];
#pragma unroll
            for (int c = 1; c < kC; ++c) {
                if (lane == c) {
                    v = pmin[c];
                    mk = pmask[c];
                }
            }
            s_part[warp * kBN + jb + lane] = ((unsigned long long)v << 32) | mk;
        }
        const uint32_t mb0 = __float_as_uint(m0), mb1 = __float_as_uint(m1);
        if (mb0 < best[0]) {
            best[0] = mb0;
            blk[0] = jb;
        }
        if (mb1 < best[1]) {
            best[1] = mb1;
            blk[1] = jb;
        }
    }

    // Rows: the first column of the winning block, then commit.
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int64_t r = i0 + lrow + k;
        if (r < xlen && blk[k] >= 0) {
            int col = blk[k];
            for (int c = 0; c < kC; ++c) {
                const int j = blk[k] + c;
                if (__float_as_uint(symd_dist<NORM>(s_x, kBM, lrow + k, s_yf, j, D)) == best[k]) {
                    col = j;
                    break;
                }
            }
            atomicMin(&keys_x[(size_t)b * P + r],
                      ((unsigned long long)best[k] << 32) | (unsigned long long)(j0 + col));
        }
    }
    __syncthreads();
    // Columns: first warp, first lane, first row holding the minimum.
    for (int e = tid; e < kBN; e += kThreads) {
        const int64_t j = j0 + e;
        if (j >= ylen) continue;
        unsigned bv = 0xffffffffu, bm = 0u;
        int bw = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const unsigned long long pv = s_part[w * kBN + e];
            const unsigned v = (unsigned)(pv >> 32);
            if (v < bv) {
                bv = v;
                bw = w;
                bm = (unsigned)pv;
            }
        }
        const int l = __ffs(bm) - 1;
        const int r0 = (bw * 32 + l) * 2;
        int row = r0;
        for (int k = 0; k < 2; ++k) {
            if (i0 + r0 + k >= xlen) break;
            if (__float_as_uint(symd_dist<NORM>(s_x, kBM, r0 + k, s_yf, e, D)) == bv) {
                row = r0 + k;
                break;
            }
        }
        atomicMin(&keys_y[(size_t)b * Q + j],
                  ((unsigned long long)bv << 32) | (unsigned long long)(i0 + row));
    }
}

inline bool use_symd(int64_t P, int64_t Q, int64_t D) {
    return D != 3 && D <= kSymDMax && P >= 1 && Q >= 1;
}

// Launch of the D != 3 symmetric kernel over every item; keys pre-set to all
// ones by the caller.
template <int NORM>
int launch_symd(const float* x, const float* y, const int64_t* xl, const int64_t* yl, int64_t B,
                int64_t P, int64_t Q, int64_t D, unsigned long long* keys_x,
                unsigned long long* keys_y, cudaStream_t s, const char* who) {
    auto run = [&](auto kern, int threads, int64_t bm, int64_t bn, size_t smem) -> int {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return fail(kCudaError, std::string(who) + ": shared-memory limit");
        const int64_t items = B * ceil_div(P, bm) * ceil_div(Q, bn);
        if (items > 0x7fffffff)
            return fail(kUnsupported, std::string(who) + ": too many tiles for one launch");
        kern<<<(unsigned)items, threads, smem, s>>>(x, y, xl, yl, B, P, Q, (int)D, keys_x, keys_y);
        return check_launch("chamfer_symd_kernel");
    };
    if (D <= kSymDMaxSmall) {
        using Sh = ShapeD<8, 128>;
        return run(chamfer_symd_kernel<8, 128, NORM>, Sh::kThreads, Sh::kBM, 128, Sh::smem(D));
    }
    using Sh = ShapeD<4, 64>;
    return run(chamfer_symd_kernel<4, 64, NORM>, Sh::kThreads, Sh::kBM, 64, Sh::smem(D));
}

// Generic D (feature-space Chamfer): query row and reference tile in shared
// memory, SD accumulated in increasing dimension order.
constexpr int kDThreads = 128;


// Separately rounded arithmetic for float and double (the float64 Chamfer of
// mps_pointops/chamfer.py:101-102 runs the same kernels in double).
__device__ __forceinline__ float rn_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double rn_sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float rn_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double rn_mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float rn_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double rn_add(double a, double b) { return __dadd_rn(a, b); }

template <int NORM, typename T>
__device__ __forceinline__ T dist_seq(const T* a, const T* b, int D) {
    T d = rn_sub(a[0], b[0]);
    T s = NORM == 1 ? fabs(d) : rn_mul(d, d);
    for (int t = 1; t < D; ++t) {
        d = rn_sub(a[t], b[t]);
        s = rn_add(s, NORM == 1 ? fabs(d) : rn_mul(d, d));
    }
    return s;
}

// NORM 2: squared L2 (sequential sum of squares); NORM 1: L1.  T = float, or
// double for the float64 entry points (every D, D == 3 included: the
// sequential sum is the reference's ((d0^2 + d1^2) + d2^2) order).
template <int NORM, typename T = float>
__global__ void __launch_bounds__(kDThreads)
nearestd_kernel(const T* __restrict__ query, const T* __restrict__ ref,
                const int64_t* __restrict__ query_lengths, const int64_t* __restrict__ ref_lengths,
                int64_t M, int64_t N, int D, int tileN, T* __restrict__ out_dist,
                int64_t* __restrict__ out_idx) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* smemf = reinterpret_cast<T*>(smem_raw);
    const int tid = threadIdx.x;
    const int b = blockIdx.y;
    const int64_t q = (int64_t)blockIdx.x * kDThreads + tid;
    const int64_t qlen = query_lengths ? query_lengths[b] : M;
    const int64_t nl = ref_lengths ? min64(ref_lengths[b], N) : N;
    const bool active = q < M && q < qlen;
    const int qs = D + 1;
    T* sq = smemf;
    T* st = smemf + (size_t)kDThreads * qs;
    for (int e = tid; e < kDThreads * D; e += kDThreads) {
        const int qq = e / D, t = e % D;
        const int64_t gq = (int64_t)blockIdx.x * kDThreads + qq;
        sq[qq * qs + t] = gq < M ? query[((size_t)b * M + gq) * D + t] : T(0);
    }
    const T* __restrict__ r = ref + (size_t)b * (size_t)N * D;
    const T* myq = sq + tid * qs;
    T bd = T(INFINITY);
    uint32_t bj = kNone;
    for (int64_t t0 = 0; t0 < nl; t0 += tileN) {
        __syncthreads();
        const int64_t lim = min64((int64_t)tileN * D, (nl - t0) * D);
        for (int64_t e = tid; e < lim; e += kDThreads) st[e] = r[t0 * D + e];
        __syncthreads();
        if (!active) continue;
        const int cnt = (int)min64(tileN, nl - t0);
        for (int e = 0; e < cnt; ++e) {
            const T* rp = st + (size_t)e * D;
            const T s = dist_seq<NORM>(myq, rp, D);
            if (s < bd) {
                bd = s;
                bj = (uint32_t)(t0 + e);
            }
        }
    }
    if (q >= M) return;
    const size_t o = (size_t)b * (size_t)M + (size_t)q;
    if (!active || nl <= 0) {
        out_dist[o] = T(0);
        out_idx[o] = -1;
        return;
    }
    if (bj == kNone) {
        bj = 0;
        bd = dist_seq<NORM>(query + o * D, r, D);
    }
    out_dist[o] = bd;
    out_idx[o] = (int64_t)bj;
}

// Backward for one direction: rows with idx >= 0 add
// g = 2 * gd * (q - r[idx]) to grad_q and -g to grad_r[idx].
template <typename T = float>
__global__ void chamfer_bwd_kernel(const T* __restrict__ qpts, const T* __restrict__ rpts,
                                   int64_t B, int64_t M, int64_t N, int64_t D,
                                   const int64_t* __restrict__ idx, const T* __restrict__ gd,
                                   T* __restrict__ grad_q, T* __restrict__ grad_r) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= B * M) return;
    const int64_t j = idx[row];
    if (j < 0) return;
    const int64_t b = row / M;
    const T c = T(2) * gd[row];
    const T* qp = qpts + row * D;
    const T* rp = rpts + (b * N + j) * D;
    T* gq = grad_q + row * D;
    T* gr = grad_r + (b * N + j) * D;
    for (int64_t t = 0; t < D; ++t) {
        const T g = rn_mul(rn_sub(qp[t], rp[t]), c);
        atomicAdd(gq + t, g);
        atomicAdd(gr + t, -g);
    }
}

// L1 backward for one direction (mps_pointops/chamfer.py:269-293, PyTorch3D's
// subgradient): rows with idx >= 0 add g = s * gd, s = +1 where q > r[idx]
// and -1 otherwise (at equality too), to grad_q and -g to grad_r[idx].
template <typename T = float>
__global__ void chamfer_l1_bwd_kernel(const T* __restrict__ qpts,
                                      const T* __restrict__ rpts, int64_t B, int64_t M,
                                      int64_t N, int64_t D, const int64_t* __restrict__ idx,
                                      const T* __restrict__ gd, T* __restrict__ grad_q,
                                      T* __restrict__ grad_r) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= B * M) return;
    const int64_t j = idx[row];
    if (j < 0) return;
    const int64_t b = row / M;
    const T c = gd[row];
    const T* qp = qpts + row * D;
    const T* rp = rpts + (b * N + j) * D;
    T* gq = grad_q + row * D;
    T* gr = grad_r + (b * N + j) * D;
    for (int64_t t = 0; t < D; ++t) {
        const T g = qp[t] > rp[t] ? c : -c;
        atomicAdd(gq + t, g);
        atomicAdd(gr + t, -g);
    }
}

// Both clouds in one grid-stride launch: flags {x value, y value, x length,
// y length}; a warp sets a flag once.
__global__ void check_inputs_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                    const int64_t* __restrict__ xl,
                                    const int64_t* __restrict__ yl, int64_t B, int64_t P,
                                    int64_t Q, int64_t D, int32_t* __restrict__ flags) {
    const int64_t nx = B * P * D, total = nx + B * Q * D;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t b = t0; b < B; b += stride) {
        if (xl && (xl[b] < 0 || xl[b] > P)) flags[2] = 1;
        if (yl && (yl[b] < 0 || yl[b] > Q)) flags[3] = 1;
    }
    bool bad_x = false, bad_y = false;
    if (xl == nullptr && yl == nullptr) {
        // Every coordinate is valid: a flat scan, 16-byte loads where the
        // array allows them (no per-element row arithmetic).
        for (int a = 0; a < 2; ++a) {
            const float* p = a ? y : x;
            const int64_t n = a ? total - nx : nx;
            bool bad = false;
            int64_t head = 0;
            if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
                const float4* p4 = reinterpret_cast<const float4*>(p);
                const int64_t n4 = n / 4;
                // Four independent loads in flight per thread: the grid is
                // small (one CTA per SM) so that, beside a search kernel, the
                // check holds few SM slots.
                for (int64_t e = t0; e < n4; e += 4 * stride) {
                    float4 v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int64_t f = e + u * stride;
                        v[u] = f < n4 ? p4[f] : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        bad |= !(isfinite(v[u].x) && isfinite(v[u].y) && isfinite(v[u].z) &&
                                 isfinite(v[u].w));
                }
                head = n4 * 4;
            }
            for (int64_t e = head + t0; e < n; e += stride) bad |= !isfinite(p[e]);
            if (a) bad_y = bad;
            else bad_x = bad;
        }
    } else {
        for (int64_t e = t0; e < total; e += stride) {
            const bool is_y = e >= nx;
            const int64_t f = is_y ? e - nx : e;
            const int64_t M = is_y ? Q : P;
            const int64_t row = f / D, b = row / M, i = row % M;
            const int64_t* l = is_y ? yl : xl;
            const int64_t len = l ? l[b] : M;
            if (i < len && !isfinite((is_y ? y : x)[f])) {
                bad_x |= !is_y;
                bad_y |= is_y;
            }
        }
    }
    if (__any_sync(FULL_MASK, bad_x) && (threadIdx.x & 31) == 0) flags[0] = 1;
    if (__any_sync(FULL_MASK, bad_y) && (threadIdx.x & 31) == 0) flags[1] = 1;
}


// --------------------------------------------------------------------------
// Fused loss for the common reductions (no weights, no normals).
// finalize_reduce_kernel: kRedChunks(M) CTAs per (cloud, direction) segment,
// each over a contiguous chunk of its rows; a CTA turns the chunk's 64-bit
// keys into the public (dist, idx) arrays (FROM_KEYS) or reads the dist array
// written by a per-direction search, and sums the chunk's distances in a
// fixed order (strided per thread, then a fixed tree) ->
// partial[(b * 2 + dir) * kMaxRedChunks + chunk].  loss_kernel then adds the
// chunks and combines the segments in a fixed order, so the loss is
// bit-reproducible from run to run (the chunk count depends on the sizes
// only).  At config 2 (32 clouds x 2 directions x 8192 rows) one CTA per
// segment left 84 SMs idle: 8.6 us; four chunks per segment spread it.
constexpr int kRedThreads = 256;
constexpr int kMaxRedChunks = 8;
__host__ __device__ inline int red_chunks(int64_t M) {
    return (int)min64(kMaxRedChunks, max64(1, ceil_div(M, 2048)));
}

__device__ void loss_from_partials(const float* partial, const int64_t* __restrict__ xl,
                                   const int64_t* __restrict__ yl, int64_t B, int64_t P,
                                   int64_t Q, int bidirectional, int point_mode, int batch_mode,
                                   float* __restrict__ per_cloud, float* __restrict__ loss);

// LossArgs.done (nullable): a zeroed counter; the CTA that finishes last
// (of `blocks` CTAs that have rows) computes the loss from every partial, so
// no separate loss launch follows.
struct LossArgs {
    unsigned* done;
    int blocks;
    int bidirectional, point_mode, batch_mode;
    float* per_cloud;
    float* loss;
};

template <bool FROM_KEYS>
__global__ void __launch_bounds__(kRedThreads)
finalize_reduce_kernel(const unsigned long long* __restrict__ keys_x,
                       const unsigned long long* __restrict__ keys_y,
                       const int64_t* __restrict__ xl, const int64_t* __restrict__ yl, int64_t B,
                       int64_t P, int64_t Q, float* __restrict__ dist_x,
                       int64_t* __restrict__ idx_x, float* __restrict__ dist_y,
                       int64_t* __restrict__ idx_y, float* __restrict__ partial, LossArgs la) {
    __shared__ float s_red[kRedThreads];
    const int64_t b = blockIdx.x;
    const int dir = blockIdx.y;
    const int64_t M = dir ? Q : P, Nn = dir ? P : Q;
    const int S = red_chunks(M);
    if ((int)blockIdx.z >= S) return;  // CTA-uniform (the grid is sized for max(P, Q))
    const int64_t csize = ceil_div(M, S);
    const int64_t r0 = (int64_t)blockIdx.z * csize, r1 = min64(M, r0 + csize);
    const int64_t* self_l = dir ? yl : xl;
    const int64_t* other_l = dir ? xl : yl;
    const unsigned long long* keys = dir ? keys_y : keys_x;
    float* dist = dir ? dist_y : dist_x;
    int64_t* idx = dir ? idx_y : idx_x;
    const int64_t len = self_l ? min64(max64(self_l[b], 0), M) : M;
    const int64_t olen = other_l ? min64(max64(other_l[b], 0), Nn) : Nn;
    float acc = 0.f;
    for (int64_t i = r0 + threadIdx.x; i < r1; i += kRedThreads) {
        const int64_t e = b * M + i;
        float d;
        if (FROM_KEYS) {
            const unsigned long long key = keys[e];
            const bool valid = i < len && olen > 0 && key != kMaxKeyAll;
            d = valid ? __uint_as_float((unsigned)(key >> 32)) : 0.f;
            dist[e] = d;
            idx[e] = valid ? (int64_t)(key & 0xffffffffull) : -1;
        } else {
            d = i < len ? dist[e] : 0.f;
        }
        acc = __fadd_rn(acc, d);
    }
    s_red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = kRedThreads / 2; w >= 1; w >>= 1) {
        if (threadIdx.x < w) s_red[threadIdx.x] = __fadd_rn(s_red[threadIdx.x], s_red[threadIdx.x + w]);
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[(b * 2 + dir) * kMaxRedChunks + blockIdx.z] = s_red[0];
    if (la.done == nullptr) return;  // grid-uniform
    // Last CTA: publish this partial (fence), count, and the CTA that sees
    // the final count reads every partial after a fence of its own.
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(la.done, 1u) == (unsigned)(la.blocks - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    loss_from_partials(partial, xl, yl, B, P, Q, la.bidirectional, la.point_mode, la.batch_mode,
                       la.per_cloud, la.loss);
}

// point_mode: 0 sum, 1 mean over valid points; batch_mode: 0 none (loss[b]),
// 1 sum, 2 mean.  One thread per cloud (segment sums: their chunks in
// order), then thread 0 sums the clouds in order.  Run by a whole CTA; the
// partials are read through L2 (other CTAs wrote them).
__device__ void loss_from_partials(const float* partial, const int64_t* __restrict__ xl,
                                   const int64_t* __restrict__ yl, int64_t B, int64_t P,
                                   int64_t Q, int bidirectional, int point_mode, int batch_mode,
                                   float* __restrict__ per_cloud, float* __restrict__ loss) {
    auto seg = [&](int64_t b, int dir, int64_t M) {
        const float* c = partial + (b * 2 + dir) * kMaxRedChunks;
        float v = __ldcg(c);
        for (int k = 1; k < red_chunks(M); ++k) v = __fadd_rn(v, __ldcg(c + k));
        return v;
    };
    for (int64_t b = threadIdx.x; b < B; b += blockDim.x) {
        float v = seg(b, 0, P);
        if (point_mode == 1) {
            const int64_t n = xl ? min64(max64(xl[b], 0), P) : P;
            v = __fdiv_rn(v, (float)max64(n, 1));
        }
        if (bidirectional) {
            float w = seg(b, 1, Q);
            if (point_mode == 1) {
                const int64_t n = yl ? min64(max64(yl[b], 0), Q) : Q;
                w = __fdiv_rn(w, (float)max64(n, 1));
            }
            v = __fadd_rn(v, w);
        }
        per_cloud[b] = v;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (batch_mode == 0) {
        for (int64_t b = 0; b < B; ++b) loss[b] = per_cloud[b];
        return;
    }
    float t = 0.f;
    for (int64_t b = 0; b < B; ++b) t = __fadd_rn(t, per_cloud[b]);
    if (batch_mode == 2) t = __fdiv_rn(t, (float)max64(B, 1));
    loss[0] = t;
}

// The loss from the partials in a launch of its own (the per-direction
// search path, whose workspace holds no zeroed counter).
__global__ void loss_kernel(const float* __restrict__ partial, const int64_t* __restrict__ xl,
                            const int64_t* __restrict__ yl, int64_t B, int64_t P, int64_t Q,
                            int bidirectional, int point_mode, int batch_mode,
                            float* __restrict__ per_cloud, float* __restrict__ loss) {
    loss_from_partials(partial, xl, yl, B, P, Q, bidirectional, point_mode, batch_mode,
                       per_cloud, loss);
}

// Both gradient arrays to zero in one launch (the backward accumulates into
// them with atomics).
__global__ void zero2_kernel(float* __restrict__ a, int64_t na, float* __restrict__ b,
                             int64_t nb) {
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int h = 0; h < 2; ++h) {
        float* p = h ? b : a;
        const int64_t n = h ? nb : na;
        int64_t head = 0;
        if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
            float4* p4 = reinterpret_cast<float4*>(p);
            for (int64_t e = t0; e < n / 4; e += stride) p4[e] = make_float4(0.f, 0.f, 0.f, 0.f);
            head = n / 4 * 4;
        }
        for (int64_t e = head + t0; e < n; e += stride) p[e] = 0.f;
    }
}

// (a, b, c) added to the three floats of row r of a D = 3 array whose base
// is 8-byte aligned: one float2 atomic on the row's 8-byte aligned pair and
// one scalar atomic (each element is added atomically on its own).
__device__ __forceinline__ void atomic_add3(float* base, int64_t r, float a, float b, float c) {
    float* p = base + 3 * r;
    if ((r & 1) == 0) {
        atomicAdd(reinterpret_cast<float2*>(p), make_float2(a, b));
        atomicAdd(p + 2, c);
    } else {
        atomicAdd(p, a);
        atomicAdd(reinterpret_cast<float2*>(p + 1), make_float2(b, c));
    }
}

// Backward of the fused loss: element e of the x rows (then of the y rows)
// gets coefficient c = g_b * (1/len for the mean) and adds 2c(q - r[idx]) to
// its own gradient and -2c(q - r[idx]) to its match's.  pairs: both gradient
// arrays are 8-byte aligned (D = 3 then uses atomic_add3).
__global__ void loss_bwd_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                const int64_t* __restrict__ xl, const int64_t* __restrict__ yl,
                                int64_t B, int64_t P, int64_t Q, int64_t D, int bidirectional,
                                int point_mode, int batch_mode, const int64_t* __restrict__ idx_x,
                                const int64_t* __restrict__ idx_y,
                                const float* __restrict__ grad_loss, float* __restrict__ grad_x,
                                float* __restrict__ grad_y, int pairs) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nx = B * P;
    const int64_t total = nx + (bidirectional ? B * Q : 0);
    if (e >= total) return;
    const bool dir = e >= nx;
    const int64_t M = dir ? Q : P, Nn = dir ? P : Q;
    const int64_t row = dir ? e - nx : e;
    int64_t b, i;
    if (total <= 0x7fffffff) {  // 32-bit division (the 64-bit one is a long sequence)
        const uint32_t r32 = (uint32_t)row, m32 = (uint32_t)M;
        b = r32 / m32;
        i = r32 - (uint32_t)b * m32;
    } else {
        b = row / M;
        i = row % M;
    }
    const int64_t* self_l = dir ? yl : xl;
    const int64_t len = self_l ? min64(max64(self_l[b], 0), M) : M;
    if (i >= len) return;
    const int64_t j = (dir ? idx_y : idx_x)[row];
    if (j < 0) return;
    float c = batch_mode == 0 ? grad_loss[b] : grad_loss[0];
    if (batch_mode == 2) c = __fdiv_rn(c, (float)max64(B, 1));
    if (point_mode == 1) c = __fdiv_rn(c, (float)max64(len, 1));
    c = 2.0f * c;
    const float* qp = (dir ? y : x) + row * D;
    const float* rp = (dir ? x : y) + (b * Nn + j) * D;
    float* gq = (dir ? grad_y : grad_x) + row * D;
    float* gr = (dir ? grad_x : grad_y) + (b * Nn + j) * D;
    if (D == 3 && pairs) {
        // Two atomics per 12-byte row instead of three: with 8-byte aligned
        // gradient arrays, row r's floats (0, 1) are 8-byte aligned for even r
        // and (1, 2) for odd r.
        const float g0 = __fmul_rn(__fsub_rn(qp[0], rp[0]), c);
        const float g1 = __fmul_rn(__fsub_rn(qp[1], rp[1]), c);
        const float g2 = __fmul_rn(__fsub_rn(qp[2], rp[2]), c);
        atomic_add3(dir ? grad_y : grad_x, row, g0, g1, g2);
        atomic_add3(dir ? grad_x : grad_y, b * Nn + j, -g0, -g1, -g2);
        return;
    }
    for (int64_t t = 0; t < D; ++t) {
        const float g = __fmul_rn(__fsub_rn(qp[t], rp[t]), c);
        atomicAdd(gq + t, g);
        atomicAdd(gr + t, -g);
    }
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_chamfer_workspace_bytes(int64_t B, int64_t P, int64_t Q, int64_t D,
                                   int bidirectional) {
    if (B <= 0 || !(mpo::sym::use_sym(P, Q, D) || (bidirectional && mpo::use_symd(P, Q, D))))
        return 0;
    return mpo::sym::scratch_bytes(B, P, Q);
}

static int nearest_dir(const float* q, const float* r, const int64_t* ql, const int64_t* rl,
                       int64_t B, int64_t M, int64_t N, int64_t D, float* dist, int64_t* idx,
                       cudaStream_t s) {
    using namespace mpo;
    if (B == 0 || M == 0) return kOk;
    if (D == 3) {
        int S = 1;
        while (S < 8 && B * M * S < (int64_t)sm_count() * 1024) S *= 2;
        const int qpc = kThreads / S;
        const size_t smem = 2 * kTile * sizeof(float4);
        if (cudaFuncSetAttribute(nearest3_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return fail(kCudaError, "chamfer: cannot raise the shared-memory limit");
        dim3 grid((unsigned)ceil_div(M, qpc), (unsigned)B);
        nearest3_kernel<2><<<grid, kThreads, smem, s>>>(q, r, ql, rl, M, N, S, dist, idx);
        return check_launch("nearest3_kernel");
    }
    int tileN = 256;
    size_t smem = ((size_t)kDThreads * (D + 1) + (size_t)tileN * D) * sizeof(float);
    while (smem > 200 * 1024 && tileN > 1) {
        tileN /= 2;
        smem = ((size_t)kDThreads * (D + 1) + (size_t)tileN * D) * sizeof(float);
    }
    if (smem > 200 * 1024) return fail(kUnsupported, "chamfer: coordinate dimension too large");
    if (cudaFuncSetAttribute(nearestd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return fail(kCudaError, "chamfer: cannot raise the shared-memory limit");
    dim3 grid((unsigned)ceil_div(M, kDThreads), (unsigned)B);
    nearestd_kernel<2><<<grid, kDThreads, smem, s>>>(q, r, ql, rl, M, N, (int)D, tileN, dist, idx);
    return check_launch("nearestd_kernel");
}

static int nearest_l1_dir(const float* q, const float* r, const int64_t* ql, const int64_t* rl,
                          int64_t B, int64_t M, int64_t N, int64_t D, float* dist, int64_t* idx,
                          cudaStream_t s) {
    using namespace mpo;
    if (B == 0 || M == 0) return kOk;
    if (D == 3) {
        int S = 1;
        while (S < 8 && B * M * S < (int64_t)sm_count() * 1024) S *= 2;
        const int qpc = kThreads / S;
        const size_t smem3 = 2 * kTile * sizeof(float4);
        if (cudaFuncSetAttribute(nearest3_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem3) != cudaSuccess)
            return fail(kCudaError, "chamfer: cannot raise the shared-memory limit");
        dim3 grid((unsigned)ceil_div(M, qpc), (unsigned)B);
        nearest3_kernel<1><<<grid, kThreads, smem3, s>>>(q, r, ql, rl, M, N, S, dist, idx);
        return check_launch("nearest3_kernel<L1>");
    }
    int tileN = 256;
    size_t smem = ((size_t)kDThreads * (D + 1) + (size_t)tileN * D) * sizeof(float);
    while (smem > 200 * 1024 && tileN > 1) {
        tileN /= 2;
        smem = ((size_t)kDThreads * (D + 1) + (size_t)tileN * D) * sizeof(float);
    }
    if (smem > 200 * 1024) return fail(kUnsupported, "chamfer: coordinate dimension too large");
    if (cudaFuncSetAttribute(nearestd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return fail(kCudaError, "chamfer: cannot raise the shared-memory limit");
    dim3 grid((unsigned)ceil_div(M, kDThreads), (unsigned)B);
    nearestd_kernel<1><<<grid, kDThreads, smem, s>>>(q, r, ql, rl, M, N, (int)D, tileN, dist, idx);
    return check_launch("nearestd_kernel<L1>");
}

int mpo_chamfer_nearest_l1(const float* x, const float* y, const int64_t* x_lengths,
                           const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                           int bidirectional, float* dist_x, int64_t* idx_x, float* dist_y,
                           int64_t* idx_y, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && P >= 0 && Q >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    MPO_REQUIRE(P < (int64_t)0x7fffffff && Q < (int64_t)0x7fffffff, "P and Q must be below 2**31");
    if (B == 0) return kOk;
    MPO_REQUIRE((x || P == 0) && (y || Q == 0), "null pointer");
    MPO_REQUIRE((dist_x && idx_x) || P == 0, "null output pointer");
    MPO_REQUIRE(!bidirectional || (dist_y && idx_y) || Q == 0, "null output pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (bidirectional && (sym::use_sym(P, Q, D) || use_symd(P, Q, D))) {
        // Both directions from one evaluation per pair (the symmetric tile
        // kernel with the L1 metric).  This entry takes no workspace: the
        // 64-bit keys live in the idx arrays until the in-place finalize,
        // and the work-item counter in the first word of dist_x, which the
        // finalize overwrites.
        // The scratch lives in the outputs, so they must not overlap each
        // other or the inputs, and the key arrays need 8-byte alignment.
        {
            const size_t nx = (size_t)B * P, ny = (size_t)B * Q;
            const struct {
                const void* p;
                size_t bytes;
            } in[2] = {{x, nx * D * 4}, {y, ny * D * 4}},
              out[4] = {{dist_x, nx * 4}, {idx_x, nx * 8}, {dist_y, ny * 4}, {idx_y, ny * 8}};
            auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
                const uintptr_t ua = reinterpret_cast<uintptr_t>(a);
                const uintptr_t ub = reinterpret_cast<uintptr_t>(b);
                return na > 0 && nb > 0 && ua < ub + nb && ub < ua + na;
            };
            for (int i = 0; i < 4; ++i) {
                for (int j = i + 1; j < 4; ++j)
                    MPO_REQUIRE(!overlap(out[i].p, out[i].bytes, out[j].p, out[j].bytes),
                                "the four outputs must not overlap each other");
                for (int j = 0; j < 2; ++j)
                    MPO_REQUIRE(!overlap(out[i].p, out[i].bytes, in[j].p, in[j].bytes),
                                "the outputs must not overlap the inputs");
            }
            MPO_REQUIRE(aligned_to(idx_x, 8) && aligned_to(idx_y, 8),
                        "idx_x and idx_y must be 8-byte aligned");
        }
        unsigned long long* keys_x = reinterpret_cast<unsigned long long*>(idx_x);
        unsigned long long* keys_y = reinterpret_cast<unsigned long long*>(idx_y);
        unsigned* counter = reinterpret_cast<unsigned*>(dist_x);
        if (cudaMemsetAsync(keys_x, 0xff, (size_t)B * P * 8, s) != cudaSuccess ||
            cudaMemsetAsync(keys_y, 0xff, (size_t)B * Q * 8, s) != cudaSuccess ||
            cudaMemsetAsync(counter, 0, sizeof(unsigned), s) != cudaSuccess)
            return fail(kCudaError, "mpo_chamfer_nearest_l1: reset failed");
        if (use_symd(P, Q, D)) {
            int st = launch_symd<1>(x, y, x_lengths, y_lengths, B, P, Q, D, keys_x, keys_y, s,
                                    "mpo_chamfer_nearest_l1");
            if (st) return st;
            sym::finalize_inplace_kernel<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(
                idx_x, x_lengths, y_lengths, B, P, Q, dist_x);
            st = check_launch("chamfer finalize_inplace_kernel");
            if (st) return st;
            sym::finalize_inplace_kernel<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(
                idx_y, y_lengths, x_lengths, B, Q, P, dist_y);
            return check_launch("chamfer finalize_inplace_kernel");
        }
        auto kern = sym::chamfer_sym3_kernel<MPO_SYM_DEFAULT, 1>;
        using Sh = sym::Default;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Sh::kSmem) != cudaSuccess)
            return fail(kCudaError, "mpo_chamfer_nearest_l1: shared-memory limit");
        int per_sm = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Sh::kThreads, Sh::kSmem);
        const int64_t items = B * ceil_div(P, Sh::kBM) * ceil_div(Q, Sh::kCols);
        const int64_t grid = min64(items, (int64_t)sm_count() * max64(per_sm, 1));
        kern<<<(unsigned)grid, Sh::kThreads, Sh::kSmem, s>>>(x, y, x_lengths, y_lengths, B, P, Q,
                                                             keys_x, keys_y, counter);
        int st = check_launch("chamfer_sym3_kernel<L1>");
        if (st) return st;
        sym::finalize_inplace_kernel<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(
            idx_x, x_lengths, y_lengths, B, P, Q, dist_x);
        st = check_launch("chamfer finalize_inplace_kernel");
        if (st) return st;
        sym::finalize_inplace_kernel<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(
            idx_y, y_lengths, x_lengths, B, Q, P, dist_y);
        return check_launch("chamfer finalize_inplace_kernel");
    }
    int st = nearest_l1_dir(x, y, x_lengths, y_lengths, B, P, Q, D, dist_x, idx_x, s);
    if (st || !bidirectional) return st;
    return nearest_l1_dir(y, x, y_lengths, x_lengths, B, Q, P, D, dist_y, idx_y, s);
}

}  // extern "C"

namespace mpo {
namespace {
// Scratch reset of the symmetric searches in one launch: every 64-bit key to
// all ones (nothing found yet) and the `nz` counter words that follow the
// keys to zero (the search's work-item counter, then the loss's CTA count).
// keys is 256-byte aligned (the workspace's start).
__global__ void scratch_reset_kernel(unsigned long long* __restrict__ keys, int64_t nkeys,
                                     unsigned* __restrict__ counters, int nz) {
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    ulonglong2* k2 = reinterpret_cast<ulonglong2*>(keys);
    for (int64_t e = t0; e < nkeys / 2; e += stride) k2[e] = make_ulonglong2(~0ull, ~0ull);
    if (t0 == 0 && (nkeys & 1)) keys[nkeys - 1] = ~0ull;
    if (t0 < nz) counters[t0] = 0u;
}

// The search shared by mpo_chamfer_nearest and mpo_chamfer_loss.  On the
// symmetric path it leaves 64-bit keys in the workspace (*keys_x/*keys_y set,
// dist/idx not yet written); otherwise the per-direction kernels write
// dist/idx directly (*keys_x = nullptr).
int chamfer_search(const float* x, const float* y, const int64_t* x_lengths,
                   const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                   int bidirectional, float* dist_x, int64_t* idx_x, float* dist_y,
                   int64_t* idx_y, void* workspace, size_t workspace_bytes, cudaStream_t s,
                   unsigned long long** keys_x_out, unsigned long long** keys_y_out,
                   const char* who) {
    *keys_x_out = *keys_y_out = nullptr;
    const bool symd = bidirectional && use_symd(P, Q, D);
    if (!sym::use_sym(P, Q, D) && !symd) {
        int st = nearest_dir(x, y, x_lengths, y_lengths, B, P, Q, D, dist_x, idx_x, s);
        if (st || !bidirectional) return st;
        return nearest_dir(y, x, y_lengths, x_lengths, B, Q, P, D, dist_y, idx_y, s);
    }
    const size_t need = sym::scratch_bytes(B, P, Q);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(kWorkspaceTooSmall, std::string(who) + ": workspace must hold " +
                                            std::to_string(need) + " bytes");
    unsigned long long* keys_x = reinterpret_cast<unsigned long long*>(workspace);
    unsigned long long* keys_y = keys_x + (size_t)B * P;
    unsigned* counter = reinterpret_cast<unsigned*>(keys_y + (size_t)B * Q);
    {
        const int64_t nkeys = B * (P + Q);
        const int64_t grid = max64(1, min64(ceil_div(nkeys / 2, 256), (int64_t)sm_count() * 4));
        scratch_reset_kernel<<<(unsigned)grid, 256, 0, s>>>(keys_x, nkeys, counter, 2);
        int st = check_launch("chamfer scratch_reset_kernel");
        if (st) return st;
    }
    if (symd) {
        *keys_x_out = keys_x;
        *keys_y_out = keys_y;
        return launch_symd<2>(x, y, x_lengths, y_lengths, B, P, Q, D, keys_x, keys_y, s, who);
    }
    auto kern = sym::chamfer_sym3_kernel<MPO_SYM_DEFAULT>;
    using Sh = sym::Default;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Sh::kSmem) != cudaSuccess)
        return fail(kCudaError, std::string(who) + ": shared-memory limit");
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, Sh::kThreads, Sh::kSmem);
    const int64_t items = B * ceil_div(P, Sh::kBM) * ceil_div(Q, Sh::kCols);
    const int64_t grid = min64(items, (int64_t)sm_count() * max64(per_sm, 1));
    kern<<<(unsigned)grid, Sh::kThreads, Sh::kSmem, s>>>(x, y, x_lengths, y_lengths, B, P, Q,
                                                         keys_x, keys_y, counter);
    *keys_x_out = keys_x;
    *keys_y_out = keys_y;
    return check_launch("chamfer_sym3_kernel");
}

int check_sizes(int64_t B, int64_t P, int64_t Q, int64_t D, const char* who) {
    if (!(B >= 0 && P >= 0 && Q >= 0 && D >= 1))
        return fail(kInvalidArgument, std::string(who) + ": bad sizes");
    if (B > 65535) return fail(kInvalidArgument, std::string(who) + ": batch must be at most 65535");
    if (P >= (int64_t)0x7fffffff || Q >= (int64_t)0x7fffffff)
        return fail(kInvalidArgument, std::string(who) + ": clouds must be below 2**31");
    return kOk;
}

// Loss workspace: the search scratch, then partial[B][2][kMaxRedChunks] and
// per_cloud[B].
size_t loss_extra_offset(int64_t B, int64_t P, int64_t Q, int64_t D, int bidirectional) {
    return (sym::use_sym(P, Q, D) || (bidirectional && use_symd(P, Q, D)))
               ? (sym::scratch_bytes(B, P, Q) + 255) / 256 * 256
               : 0;
}
}  // namespace
}  // namespace mpo

extern "C" {

int mpo_chamfer_nearest(const float* x, const float* y, const int64_t* x_lengths,
                        const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                        int bidirectional, float* dist_x, int64_t* idx_x, float* dist_y,
                        int64_t* idx_y, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace mpo;
    int st = check_sizes(B, P, Q, D, "mpo_chamfer_nearest");
    if (st) return st;
    MPO_REQUIRE_WORKSPACE(workspace);
    cudaStream_t s = (cudaStream_t)stream;
    if (B == 0) return kOk;
    unsigned long long *keys_x, *keys_y;
    st = chamfer_search(x, y, x_lengths, y_lengths, B, P, Q, D, bidirectional, dist_x, idx_x,
                        dist_y, idx_y, workspace, workspace_bytes, s, &keys_x, &keys_y,
                        "mpo_chamfer_nearest");
    if (st || keys_x == nullptr) return st;
    sym::finalize_kernel<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(
        keys_x, x_lengths, y_lengths, B, P, Q, dist_x, idx_x);
    st = check_launch("chamfer finalize_kernel");
    if (st || !bidirectional) return st;
    sym::finalize_kernel<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(
        keys_y, y_lengths, x_lengths, B, Q, P, dist_y, idx_y);
    return check_launch("chamfer finalize_kernel");
}

size_t mpo_chamfer_loss_workspace_bytes(int64_t B, int64_t P, int64_t Q, int64_t D,
                                        int bidirectional) {
    if (B <= 0) return 0;
    return mpo::loss_extra_offset(B, P, Q, D, bidirectional) +
           (size_t)B * (2 * mpo::kMaxRedChunks + 1) * sizeof(float);
}

int mpo_chamfer_loss(const float* x, const float* y, const int64_t* x_lengths,
                     const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                     int bidirectional, int point_mode, int batch_mode, float* dist_x,
                     int64_t* idx_x, float* dist_y, int64_t* idx_y, float* loss,
                     void* workspace, size_t workspace_bytes, void* stream) {
    using namespace mpo;
    int st = check_sizes(B, P, Q, D, "mpo_chamfer_loss");
    if (st) return st;
    MPO_REQUIRE_WORKSPACE(workspace);
    MPO_REQUIRE(point_mode == 0 || point_mode == 1, "point_mode must be 0 (sum) or 1 (mean)");
    MPO_REQUIRE(batch_mode >= 0 && batch_mode <= 2, "batch_mode must be 0, 1 or 2");
    MPO_REQUIRE(loss, "null loss pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (B == 0) {
        if (batch_mode != 0 && cudaMemsetAsync(loss, 0, sizeof(float), s) != cudaSuccess)
            return fail(kCudaError, "mpo_chamfer_loss: memset failed");
        return kOk;
    }
    const size_t need = mpo_chamfer_loss_workspace_bytes(B, P, Q, D, bidirectional);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(kWorkspaceTooSmall,
                    "mpo_chamfer_loss: workspace must hold " + std::to_string(need) + " bytes");
    unsigned long long *keys_x, *keys_y;
    st = chamfer_search(x, y, x_lengths, y_lengths, B, P, Q, D, bidirectional, dist_x, idx_x,
                        dist_y, idx_y, workspace, workspace_bytes, s, &keys_x, &keys_y,
                        "mpo_chamfer_loss");
    if (st) return st;
    float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) +
                                              loss_extra_offset(B, P, Q, D, bidirectional));
    float* per_cloud = partial + 2 * B * kMaxRedChunks;
    dim3 grid((unsigned)B, bidirectional ? 2u : 1u,
              (unsigned)red_chunks(bidirectional ? max64(P, Q) : P));
    // On the keyed (symmetric) path the scratch reset zeroed a counter after
    // the search's: the last finalize CTA computes the loss itself.
    LossArgs la{nullptr, 0, bidirectional, point_mode, batch_mode, per_cloud, loss};
    if (keys_x) {
        la.done = reinterpret_cast<unsigned*>(keys_y + (size_t)B * Q) + 1;
        la.blocks = (int)(B * (red_chunks(P) + (bidirectional ? red_chunks(Q) : 0)));
        finalize_reduce_kernel<true><<<grid, kRedThreads, 0, s>>>(
            keys_x, keys_y, x_lengths, y_lengths, B, P, Q, dist_x, idx_x, dist_y, idx_y, partial,
            la);
        return check_launch("chamfer finalize_reduce_kernel");
    }
    finalize_reduce_kernel<false><<<grid, kRedThreads, 0, s>>>(
        nullptr, nullptr, x_lengths, y_lengths, B, P, Q, dist_x, idx_x, dist_y, idx_y, partial,
        la);
    st = check_launch("chamfer finalize_reduce_kernel");
    if (st) return st;
    loss_kernel<<<1, 256, 0, s>>>(partial, x_lengths, y_lengths, B, P, Q, bidirectional,
                                  point_mode, batch_mode, per_cloud, loss);
    return check_launch("chamfer loss_kernel");
}

int mpo_chamfer_loss_backward(const float* x, const float* y, const int64_t* x_lengths,
                              const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                              int64_t D, int bidirectional, int point_mode, int batch_mode,
                              const int64_t* idx_x, const int64_t* idx_y,
                              const float* grad_loss, float* grad_x, float* grad_y,
                              void* stream) {
    using namespace mpo;
    int st = check_sizes(B, P, Q, D, "mpo_chamfer_loss_backward");
    if (st) return st;
    MPO_REQUIRE((grad_x || B * P * D == 0) && (grad_y || B * Q * D == 0), "null gradient pointer");
    cudaStream_t s = (cudaStream_t)stream;
    {
        const int64_t nz = B * (P + Q) * D;
        if (nz > 0) {
            const int64_t grid = max64(1, min64(ceil_div(nz / 4, 256), (int64_t)sm_count() * 4));
            zero2_kernel<<<(unsigned)grid, 256, 0, s>>>(grad_x, B * P * D, grad_y, B * Q * D);
            st = check_launch("chamfer zero2_kernel");
            if (st) return st;
        }
    }
    const int64_t total = B * P + (bidirectional ? B * Q : 0);
    if (total == 0) return kOk;
    MPO_REQUIRE(grad_loss && (idx_x || B * P == 0) && (idx_y || !bidirectional || B * Q == 0),
                "null pointer");
    const int pairs = (aligned_to(grad_x, 8) && aligned_to(grad_y, 8)) ? 1 : 0;
    loss_bwd_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
        x, y, x_lengths, y_lengths, B, P, Q, D, bidirectional, point_mode, batch_mode, idx_x,
        idx_y, grad_loss, grad_x, grad_y, pairs);
    return check_launch("chamfer loss_bwd_kernel");
}

int mpo_chamfer_backward(const float* x, const float* y, int64_t B, int64_t P, int64_t Q,
                         int64_t D, const int64_t* idx_x, const float* grad_dist_x,
                         const int64_t* idx_y, const float* grad_dist_y, float* grad_x,
                         float* grad_y, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && P >= 0 && Q >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE((grad_x || B * P * D == 0) && (grad_y || B * Q * D == 0), "null gradient pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (B * P * D > 0 && cudaMemsetAsync(grad_x, 0, sizeof(float) * B * P * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_backward: memset failed");
    if (B * Q * D > 0 && cudaMemsetAsync(grad_y, 0, sizeof(float) * B * Q * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_backward: memset failed");
    if (grad_dist_x && B * P > 0) {
        chamfer_bwd_kernel<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(
            x, y, B, P, Q, D, idx_x, grad_dist_x, grad_x, grad_y);
        int st = check_launch("chamfer_bwd_kernel");
        if (st) return st;
    }
    if (grad_dist_y && B * Q > 0) {
        chamfer_bwd_kernel<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(
            y, x, B, Q, P, D, idx_y, grad_dist_y, grad_y, grad_x);
        return check_launch("chamfer_bwd_kernel");
    }
    return kOk;
}

int mpo_chamfer_l1_backward(const float* x, const float* y, int64_t B, int64_t P, int64_t Q,
                            int64_t D, const int64_t* idx_x, const float* grad_dist_x,
                            const int64_t* idx_y, const float* grad_dist_y, float* grad_x,
                            float* grad_y, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && P >= 0 && Q >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE((grad_x || B * P * D == 0) && (grad_y || B * Q * D == 0), "null gradient pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (B * P * D > 0 && cudaMemsetAsync(grad_x, 0, sizeof(float) * B * P * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_l1_backward: memset failed");
    if (B * Q * D > 0 && cudaMemsetAsync(grad_y, 0, sizeof(float) * B * Q * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_l1_backward: memset failed");
    if (grad_dist_x && B * P > 0) {
        chamfer_l1_bwd_kernel<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(
            x, y, B, P, Q, D, idx_x, grad_dist_x, grad_x, grad_y);
        int st = check_launch("chamfer_l1_bwd_kernel");
        if (st) return st;
    }
    if (grad_dist_y && B * Q > 0) {
        chamfer_l1_bwd_kernel<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(
            y, x, B, Q, P, D, idx_y, grad_dist_y, grad_y, grad_x);
        return check_launch("chamfer_l1_bwd_kernel");
    }
    return kOk;
}

int mpo_chamfer_nearest_f64(const double* x, const double* y, const int64_t* x_lengths,
                            const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                            int norm, int bidirectional, double* dist_x, int64_t* idx_x,
                            double* dist_y, int64_t* idx_y, void* stream) {
    using namespace mpo;
    int st = check_sizes(B, P, Q, D, "mpo_chamfer_nearest_f64");
    if (st) return st;
    MPO_REQUIRE(norm == 1 || norm == 2, "norm must be 1 or 2");
    if (B == 0) return kOk;
    MPO_REQUIRE((x || P == 0) && (y || Q == 0), "null pointer");
    MPO_REQUIRE((dist_x && idx_x) || P == 0, "null output pointer");
    MPO_REQUIRE(!bidirectional || (dist_y && idx_y) || Q == 0, "null output pointer");
    cudaStream_t s = (cudaStream_t)stream;
    int tileN = 256;
    auto bytes = [&](int tn) {
        return ((size_t)kDThreads * (D + 1) + (size_t)tn * D) * sizeof(double);
    };
    while (bytes(tileN) > 200 * 1024 && tileN > 1) tileN /= 2;
    if (bytes(tileN) > 200 * 1024)
        return fail(kUnsupported, "mpo_chamfer_nearest_f64: coordinate dimension too large");
    const size_t smem = bytes(tileN);
    auto run = [&](auto kern, const double* q, const double* r, const int64_t* ql,
                   const int64_t* rl, int64_t M, int64_t N, double* dist, int64_t* idx) -> int {
        if (M == 0) return kOk;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return fail(kCudaError, "mpo_chamfer_nearest_f64: shared-memory limit");
        dim3 grid((unsigned)ceil_div(M, kDThreads), (unsigned)B);
        kern<<<grid, kDThreads, smem, s>>>(q, r, ql, rl, M, N, (int)D, tileN, dist, idx);
        return check_launch("nearestd_kernel<f64>");
    };
    auto kern = norm == 1 ? nearestd_kernel<1, double> : nearestd_kernel<2, double>;
    st = run(kern, x, y, x_lengths, y_lengths, P, Q, dist_x, idx_x);
    if (st || !bidirectional) return st;
    return run(kern, y, x, y_lengths, x_lengths, Q, P, dist_y, idx_y);
}

int mpo_chamfer_backward_f64(const double* x, const double* y, int64_t B, int64_t P, int64_t Q,
                             int64_t D, int norm, const int64_t* idx_x,
                             const double* grad_dist_x, const int64_t* idx_y,
                             const double* grad_dist_y, double* grad_x, double* grad_y,
                             void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && P >= 0 && Q >= 0 && D >= 1, "bad sizes");
    MPO_REQUIRE(norm == 1 || norm == 2, "norm must be 1 or 2");
    MPO_REQUIRE((grad_x || B * P * D == 0) && (grad_y || B * Q * D == 0), "null gradient pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (B * P * D > 0 && cudaMemsetAsync(grad_x, 0, sizeof(double) * B * P * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_backward_f64: memset failed");
    if (B * Q * D > 0 && cudaMemsetAsync(grad_y, 0, sizeof(double) * B * Q * D, s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_backward_f64: memset failed");
    auto kern = norm == 1 ? chamfer_l1_bwd_kernel<double> : chamfer_bwd_kernel<double>;
    if (grad_dist_x && B * P > 0) {
        MPO_REQUIRE(idx_x, "null pointer");
        kern<<<(unsigned)ceil_div(B * P, 256), 256, 0, s>>>(x, y, B, P, Q, D, idx_x, grad_dist_x,
                                                            grad_x, grad_y);
        int st = check_launch("chamfer_bwd_kernel<f64>");
        if (st) return st;
    }
    if (grad_dist_y && B * Q > 0) {
        MPO_REQUIRE(idx_y, "null pointer");
        kern<<<(unsigned)ceil_div(B * Q, 256), 256, 0, s>>>(y, x, B, Q, P, D, idx_y, grad_dist_y,
                                                            grad_y, grad_x);
        return check_launch("chamfer_bwd_kernel<f64>");
    }
    return kOk;
}

int mpo_chamfer_check_inputs(const float* x, const float* y, const int64_t* x_lengths,
                             const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                             int64_t D, int32_t* flags, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(flags, "null flag pointer");
    MPO_REQUIRE(B >= 0 && P >= 0 && Q >= 0 && D >= 1, "bad sizes");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(flags, 0, 4 * sizeof(int32_t), s) != cudaSuccess)
        return fail(kCudaError, "mpo_chamfer_check_inputs: memset failed");
    const int64_t total = max64(B * (P + Q) * D, B);
    if (total == 0) return kOk;
    // One CTA per SM at most: callers run this check on a side stream beside
    // the search, whose CTAs fill the SMs' registers, so every CTA here holds
    // back one search CTA until it ends.
    const unsigned grid = (unsigned)min64(ceil_div(total, 1024), (int64_t)sm_count());
    check_inputs_kernel<<<grid, 256, 0, s>>>(x, y, x_lengths, y_lengths, B, P, Q, D, flags);
    return check_launch("check_inputs_kernel");
}

}  // extern "C"
