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
// Design (B200): one warp per query scans the reference cloud in input order,
// 128 points per step (four independent 32-point chunks, so the loads of a
// step overlap).  Each lane evaluates one point; __ballot_sync gives
// the hit mask and __popc(mask & lanes_below) the rank of each hit, so the
// hits land in their output slots in order with no serial scan.  The warp
// stops as soon as K hits are found (on uniform clouds that is a small
// prefix of the cloud), then writes the padding.  Eight queries per CTA.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"
#include "segments.cuh"

namespace mpo {
namespace {

constexpr int kWarpsPerCta = 8;

template <bool POINTNET2, bool FLAT>
__global__ void __launch_bounds__(32 * kWarpsPerCta)
ball_query_kernel(const float* __restrict__ query, const float* __restrict__ ref,
                  const int64_t* __restrict__ query_lengths,
                  const int64_t* __restrict__ ref_lengths, Layout L, int64_t K, float r2,
                  int ignore_same, float* __restrict__ dist2, int64_t* __restrict__ idx64,
                  int32_t* __restrict__ idx32) {
    const int lane = threadIdx.x & 31;
    Span sp;
    if (!locate<FLAT>(L, kWarpsPerCta, sp)) return;
    const int64_t q = sp.q0 + (threadIdx.x >> 5);  // global query row
    if (q >= sp.q1) return;
    const size_t row = (size_t)q * (size_t)K;
    int64_t nl = sp.n;
    bool live = true;
    if (!FLAT) {
        const int64_t b = blockIdx.y;
        if (query_lengths) live = q - b * L.M < query_lengths[b];
        if (ref_lengths) nl = min64(ref_lengths[b], L.N);
    }
    const unsigned below = (1u << lane) - 1u;

    int64_t found = 0;
    int64_t first = -1;
    if (live) {
        const float* qp = query + (size_t)q * 3;
        const float qx = qp[0], qy = qp[1], qz = qp[2];
        const float* __restrict__ r = ref + (size_t)sp.r0 * 3;
        // A flat search with ignore_same skips the reference whose global row
        // equals the query's (local row `self`), before the cap.
        const int64_t self = (FLAT && ignore_same) ? q - sp.obase : -1;
        // Four 32-point chunks per iteration: their loads are independent,
        // so a lane has 12 loads in flight; hits are still ranked in input
        // order chunk by chunk.
        constexpr int kU = 4;
        for (int64_t j0 = 0; j0 < nl && found < K; j0 += 32 * kU) {
            float d[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t j = j0 + u * 32 + lane;
                d[u] = INFINITY;
                if (j < nl) d[u] = sqd3(qx, qy, qz, r[3 * j], r[3 * j + 1], r[3 * j + 2]);
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t j = j0 + u * 32 + lane;
                const bool hit = j < nl && d[u] < r2 && j != self;
                const unsigned mask = __ballot_sync(FULL_MASK, hit);
                if (mask == 0u) continue;
                if (first < 0) first = j0 + u * 32 + (__ffs(mask) - 1);
                const int64_t slot = found + __popc(mask & below);
                if (hit && slot < K) {
                    if (POINTNET2) {
                        idx32[row + slot] = (int32_t)j;
                    } else {
                        idx64[row + slot] = sp.obase + j;
                        if (dist2) dist2[row + slot] = d[u];
                    }
                }
                found += __popc(mask);
            }
        }
    }
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
