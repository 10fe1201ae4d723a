// First-K radius search (ball query) on sm_100a, its pointnet2_ops padded
// form and its distance backward.
//
// Contract: gamzerA/mps-pointops mps_pointops/reference.py:83-121 -- the first
// K reference points IN INPUT ORDER with SD < r2 (strict), r2 =
// fl32(fl32(r)*fl32(r)) (mps_pointops/_ball_query_mps.py:87-119); empty slots
// are (index -1, distance 0).  A non-finite coordinate gives a NaN or +inf
// SD, which fails the strict compare, so it never matches.  Optional lengths
// follow _ball_query_mps.py:73-84.  The pointnet2_ops form
// (mps_pointops/compat.py:76-85) repeats the first hit in empty slots (all
// zeros without a hit) and writes int32.
//
// Design (B200): one warp per query scans the reference cloud in input order;
// the eight queries of a CTA (one cloud or segment) share reference tiles of
// kTile points in shared memory.  A warp step covers 128 references, four
// per lane (lane l takes points 4l .. 4l+3), evaluated as two packed f32x2
// pairs with the query duplicated in both halves, from a tile stored as
// float4s A[g] = (x0, x1, y0, y1), B[g] = (x2, x3, y2, y3), Z[g] = (z0 .. z3)
// per group of four points (a lane's three loads are consecutive across the
// warp).  One min over the lane's four distances and a ballot skip steps
// without hits.  Otherwise each lane's hit count (0..4) is spread over three
// ballots, whose popcounts below the lane give its exclusive prefix, so the
// hits land in their output slots in input order with no serial scan.  A
// warp stops as soon as K hits are found; the CTA stops loading tiles once
// all its warps have stopped.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"
#include "segments.cuh"

namespace mpo {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kTile = 2048;  // reference points per shared-memory tile (multiple of 128)

template <bool POINTNET2, bool FLAT>
__global__ void __launch_bounds__(32 * kWarpsPerCta)
ball_query_kernel(const float* __restrict__ query, const float* __restrict__ ref,
                  const int64_t* __restrict__ query_lengths,
                  const int64_t* __restrict__ ref_lengths, Layout L, int64_t K, float r2,
                  int ignore_same, float* __restrict__ dist2, int64_t* __restrict__ idx64,
                  int32_t* __restrict__ idx32) {
    __shared__ float4 tA[kTile / 4], tB[kTile / 4], tZ[kTile / 4];
    const int lane = threadIdx.x & 31;
    Span sp;
    if (!locate<FLAT>(L, kWarpsPerCta, sp)) return;  // CTA-uniform
    const int64_t q = sp.q0 + (threadIdx.x >> 5);  // global query row
    const bool in_range = q < sp.q1;
    const size_t row = (size_t)q * (size_t)K;
    int64_t nl = sp.n;
    bool live = in_range;
    if (!FLAT) {
        const int64_t b = blockIdx.y;
        if (query_lengths && in_range) live = q - b * L.M < query_lengths[b];
        if (ref_lengths) nl = max64(0, min64(ref_lengths[b], L.N));
    }
    const unsigned below = (1u << lane) - 1u;
    float qx = 0.f, qy = 0.f, qz = 0.f;
    if (live) {
        const float* qp = query + (size_t)q * 3;
        qx = qp[0];
        qy = qp[1];
        qz = qp[2];
    }
    const f32x2 X = pack2(qx, qx), Y = pack2(qy, qy), Z = pack2(qz, qz);
    // A flat search with ignore_same skips the reference whose global row
    // equals the query's (local row `self`), before the cap.
    const int64_t self = (FLAT && ignore_same) ? q - sp.obase : -1;
    const float* __restrict__ r = ref + (size_t)sp.r0 * 3;
    const int u = threadIdx.x & 3;  // tile fill: fixed place in its group
    float* const fxy = reinterpret_cast<float*>(u < 2 ? tA : tB);
    float* const fz = reinterpret_cast<float*>(tZ);

    int64_t found = 0;
    int64_t first = -1;
    bool scanning = live && K > 0;
    for (int64_t t0 = 0; t0 < nl; t0 += kTile) {
        if (!__syncthreads_or(scanning)) break;  // also guards the tile reuse
        const int tn = (int)min64(kTile, nl - t0);
        for (int p = threadIdx.x; p < tn; p += 32 * kWarpsPerCta) {
            const float* rp = r + (size_t)(t0 + p) * 3;
            const int g = p >> 2;
            fxy[4 * g + (u & 1)] = rp[0];
            fxy[4 * g + 2 + (u & 1)] = rp[1];
            fz[4 * g + u] = rp[2];
        }
        __syncthreads();
        if (!scanning) continue;
        for (int c0 = 0; c0 < tn; c0 += 128) {
            const int g = (c0 >> 2) + lane;
            const ulonglong2 a = *reinterpret_cast<const ulonglong2*>(tA + g);
            const ulonglong2 bb = *reinterpret_cast<const ulonglong2*>(tB + g);
            const ulonglong2 z = *reinterpret_cast<const ulonglong2*>(tZ + g);
            float d[4];
            unpack2(sqd3x2(X, Y, Z, a.x, a.y, z.x), d[0], d[1]);
            unpack2(sqd3x2(X, Y, Z, bb.x, bb.y, z.y), d[2], d[3]);
            // fminf ignores NaN, which never matches anyway.
            const float m = fminf(fminf(d[0], d[1]), fminf(d[2], d[3]));
            if (__ballot_sync(FULL_MASK, 4 * g < tn && m < r2) == 0u) continue;
            // Hits of this lane, in index order (points past the tile end and
            // the excluded self row never hit).
            unsigned h = 0u;
            const int64_t j0 = t0 + c0 + 4 * lane;
#pragma unroll
            for (int v = 0; v < 4; ++v)
                h |= (c0 + 4 * lane + v < tn && d[v] < r2 && j0 + v != self) ? (1u << v) : 0u;
            const int c = __popc(h);
            const unsigned b0 = __ballot_sync(FULL_MASK, c & 1);
            const unsigned b1 = __ballot_sync(FULL_MASK, c & 2);
            const unsigned b2 = __ballot_sync(FULL_MASK, c & 4);
            const int total = __popc(b0) + 2 * __popc(b1) + 4 * __popc(b2);
            if (total == 0) continue;
            if (POINTNET2 && first < 0) {
                const int src = __ffs(__ballot_sync(FULL_MASK, h != 0u)) - 1;
                first = t0 + c0 + 4 * src + (__ffs(__shfl_sync(FULL_MASK, h, src)) - 1);
            }
            int64_t slot = found + __popc(b0 & below) + 2 * __popc(b1 & below) +
                           4 * __popc(b2 & below);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                if ((h >> v) & 1u) {
                    if (slot < K) {
                        if (POINTNET2) {
                            idx32[row + slot] = (int32_t)(j0 + v);
                        } else {
                            idx64[row + slot] = sp.obase + j0 + v;
                            if (dist2) dist2[row + slot] = d[v];
                        }
                    }
                    ++slot;
                }
            }
            found += total;
            if (found >= K) {
                scanning = false;
                break;
            }
        }
    }
    if (!in_range) return;
    // Padding.
    const int64_t filled = min64(found, K);
    for (int64_t s = filled + lane; s < K; s += 32) {
        if (POINTNET2) {
            idx32[row + s] = first < 0 ? 0 : (int32_t)first;
        } else {
            idx64[row + s] = -1;
            if (dist2) dist2[row + s] = 0.f;
        }
    }
}

// Backward: one thread per (b, m, slot).  grad_query accumulates over the K
// slots of its row; grad_ref receives -2 g (q - x) at the selected point.
__global__ void ball_query_grad_query_kernel(const float* __restrict__ g,
                                             const float* __restrict__ query,
                                             const float* __restrict__ ref,
                                             const int64_t* __restrict__ idx, int64_t B,
                                             int64_t M, int64_t N, int64_t K,
                                             float* __restrict__ grad_query) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (b, m)
    if (row >= B * M) return;
    const int64_t b = row / M;
    const float qx = query[3 * row], qy = query[3 * row + 1], qz = query[3 * row + 2];
    float ax = 0.f, ay = 0.f, az = 0.f;
    for (int64_t s = 0; s < K; ++s) {
        const int64_t j = idx[row * K + s];
        if (j < 0) continue;
        const float c = 2.0f * g[row * K + s];
        const float* x = ref + (b * N + j) * 3;
        ax = __fadd_rn(ax, __fmul_rn(c, __fsub_rn(qx, x[0])));
        ay = __fadd_rn(ay, __fmul_rn(c, __fsub_rn(qy, x[1])));
        az = __fadd_rn(az, __fmul_rn(c, __fsub_rn(qz, x[2])));
    }
    grad_query[3 * row] = ax;
    grad_query[3 * row + 1] = ay;
    grad_query[3 * row + 2] = az;
}

__global__ void ball_query_grad_ref_kernel(const float* __restrict__ g,
                                           const float* __restrict__ query,
                                           const float* __restrict__ ref,
                                           const int64_t* __restrict__ idx, int64_t B, int64_t M,
                                           int64_t N, int64_t K, float* __restrict__ grad_ref) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (b, m, s)
    if (e >= B * M * K) return;
    const int64_t j = idx[e];
    if (j < 0) return;
    const int64_t row = e / K;
    const int64_t b = row / M;
    const float c = 2.0f * g[e];
    const float* x = ref + (b * N + j) * 3;
    float* gr = grad_ref + (b * N + j) * 3;
    atomicAdd(gr + 0, -__fmul_rn(c, __fsub_rn(query[3 * row + 0], x[0])));
    atomicAdd(gr + 1, -__fmul_rn(c, __fsub_rn(query[3 * row + 1], x[1])));
    atomicAdd(gr + 2, -__fmul_rn(c, __fsub_rn(query[3 * row + 2], x[2])));
}

}  // namespace
}  // namespace mpo

extern "C" {

int mpo_ball_query(const float* query, const float* ref, const int64_t* query_lengths,
                   const int64_t* ref_lengths, int64_t B, int64_t M, int64_t N, int64_t K,
                   float radius_sq, float* dist2, int64_t* idx, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && M >= 0 && N >= 0 && K >= 0, "negative size");
    if (B == 0 || M == 0 || K == 0) return kOk;
    MPO_REQUIRE(query && dist2 && idx && (ref || N == 0), "null pointer");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    dim3 grid((unsigned)ceil_div(M, kWarpsPerCta), (unsigned)B);
    ball_query_kernel<false, false><<<grid, 32 * kWarpsPerCta, 0, (cudaStream_t)stream>>>(
        query, ref, query_lengths, ref_lengths, dense_layout(M, N), K, radius_sq, 0, dist2, idx,
        nullptr);
    return check_launch("ball_query_kernel");
}

int mpo_flat_radius(const float* x, const float* y, const int64_t* ptr_x, const int64_t* ptr_y,
                    int64_t segments, int64_t nx, int64_t ny, float radius_sq,
                    int64_t max_neighbors, int ignore_same_index, int64_t* out, int32_t* status,
                    void* stream) {
    using namespace mpo;
    MPO_REQUIRE(segments >= 0 && nx >= 0 && ny >= 0 && max_neighbors >= 0, "negative size");
    MPO_REQUIRE(status != nullptr, "status must not be null");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(status, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(kCudaError, "mpo_flat_radius: status reset failed");
    if (ny == 0 || max_neighbors == 0) return kOk;
    MPO_REQUIRE(segments >= 1, "a nonempty query set needs at least one segment");
    MPO_REQUIRE(y && ptr_x && ptr_y && out && (x || nx == 0), "null pointer");
    int st = flat_offsets_check(ptr_y, ptr_x, segments, ny, nx, status, s);
    if (st) return st;
    Layout L{ny, nx, ptr_y, ptr_x, segments, status};
    const dim3 grid((unsigned)flat_tiles(ny, segments, kWarpsPerCta));
    ball_query_kernel<false, true><<<grid, 32 * kWarpsPerCta, 0, s>>>(
        y, x, nullptr, nullptr, L, max_neighbors, radius_sq, ignore_same_index ? 1 : 0, nullptr,
        out, nullptr);
    return check_launch("ball_query_kernel<flat>");
}

int mpo_ball_query_pointnet2(const float* xyz, const float* new_xyz, int64_t B, int64_t N,
                             int64_t npoint, int64_t nsample, float radius_sq, int32_t* idx,
                             void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && npoint >= 0 && nsample >= 0, "negative size");
    if (B == 0 || npoint == 0 || nsample == 0) return kOk;
    MPO_REQUIRE(new_xyz && idx && (xyz || N == 0), "null pointer");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    dim3 grid((unsigned)ceil_div(npoint, kWarpsPerCta), (unsigned)B);
    ball_query_kernel<true, false><<<grid, 32 * kWarpsPerCta, 0, (cudaStream_t)stream>>>(
        new_xyz, xyz, nullptr, nullptr, dense_layout(npoint, N), nsample, radius_sq, 0, nullptr,
        nullptr, idx);
    return check_launch("ball_query_kernel<pointnet2>");
}

int mpo_ball_query_backward(const float* grad_dist2, const float* query, const float* ref,
                            const int64_t* idx, int64_t B, int64_t M, int64_t N, int64_t K,
                            float* grad_query, float* grad_ref, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && M >= 0 && N >= 0 && K >= 0, "negative size");
    cudaStream_t s = (cudaStream_t)stream;
    if (grad_ref && B * N > 0) {
        if (cudaMemsetAsync(grad_ref, 0, sizeof(float) * 3 * B * N, s) != cudaSuccess)
            return fail(kCudaError, "mpo_ball_query_backward: memset failed");
    }
    if (grad_query && B * M > 0) {
        if (K == 0) {
            if (cudaMemsetAsync(grad_query, 0, sizeof(float) * 3 * B * M, s) != cudaSuccess)
                return fail(kCudaError, "mpo_ball_query_backward: memset failed");
        } else {
            ball_query_grad_query_kernel<<<(unsigned)ceil_div(B * M, 256), 256, 0, s>>>(
                grad_dist2, query, ref, idx, B, M, N, K, grad_query);
            int st = check_launch("ball_query_grad_query_kernel");
            if (st) return st;
        }
    }
    if (grad_ref && B * M * K > 0) {
        ball_query_grad_ref_kernel<<<(unsigned)ceil_div(B * M * K, 256), 256, 0, s>>>(
            grad_dist2, query, ref, idx, B, M, N, K, grad_ref);
        return check_launch("ball_query_grad_ref_kernel");
    }
    return kOk;
}

}  // extern "C"
