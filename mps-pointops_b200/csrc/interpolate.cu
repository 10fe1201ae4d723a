// PointNet++ three_interpolate forward / backward on sm_100a.
//
// Contract: gamzerA/mps-pointops mps_pointops/pointnet2.py:135-188 --
//   out[b,c,n] = ((F[b,c,I0]*W0 + F[b,c,I1]*W1) + F[b,c,I2]*W2), each
//   product and sum rounded on its own (the reference's CPU path multiplies,
//   then sums the length-3 axis in order);
//   grad_F[b,c,m] = sum over (n,t) with I[b,n,t] == m of g[b,c,n]*W[b,n,t].
//
// Design (B200): both directions are bandwidth-bound gathers.
//   * Forward: a thread owns one (b, n) and a slice of channels; it loads its
//     three indices and weights once and walks the channels, so the (B,C,N)
//     output is written coalesced along n and each feature row (M floats,
//     4 KB at M = 1024) stays hot in L1.
//   * Indices outside [0, M) contribute nothing (the forward sums the valid
//     terms, the backward skips them): callers check bounds with
//     mpo_index_check and raise afterwards, without a host round trip before
//     the launch, so the kernels must stay memory-safe on such input.
//   * Backward: a CTA owns one (b, c) feature row; it scatters into a
//     shared-memory copy of that row with shared atomics, then writes the row
//     once -- no global atomics and no separate zero fill when the row fits
//     in shared memory (M <= 48K); otherwise global atomics on a zeroed row.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

// Channels per forward thread: the three indices and weights of a point are
// loaded once for this many channels (config 1 forward: 3.9 -> 2.8 us with
// 32 instead of 8).
constexpr int kChanPerThread = 32;


__global__ void __launch_bounds__(256)
interp_fwd_kernel(const float* __restrict__ features, const int32_t* __restrict__ idx,
                  const float* __restrict__ weights, int64_t C, int64_t M, int64_t N,
                  float* __restrict__ out) {
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t b = blockIdx.z;
    const int64_t c0 = (int64_t)blockIdx.y * kChanPerThread;
    if (n >= N) return;
    const int32_t* I = idx + (b * N + n) * 3;
    const float* W = weights + (b * N + n) * 3;
    const int32_t i0 = I[0], i1 = I[1], i2 = I[2];
    const float w0 = W[0], w1 = W[1], w2 = W[2];
    const bool v0 = i0 >= 0 && i0 < M, v1 = i1 >= 0 && i1 < M, v2 = i2 >= 0 && i2 < M;
    const int64_t c1 = min64(C, c0 + kChanPerThread);
    for (int64_t c = c0; c < c1; ++c) {
        const float* F = features + (b * C + c) * M;
        const float p0 = v0 ? __fmul_rn(__ldg(F + i0), w0) : 0.f;
        const float p1 = v1 ? __fmul_rn(__ldg(F + i1), w1) : 0.f;
        const float p2 = v2 ? __fmul_rn(__ldg(F + i2), w2) : 0.f;
        out[(b * C + c) * N + n] = __fadd_rn(__fadd_rn(p0, p1), p2);
    }
}

__global__ void __launch_bounds__(512)
interp_bwd_smem_kernel(const float* __restrict__ grad_out, const int32_t* __restrict__ idx,
                       const float* __restrict__ weights, int64_t C, int64_t M, int64_t N,
                       float* __restrict__ grad_features) {
    extern __shared__ float row[];
    const int64_t c = blockIdx.x;
    const int64_t b = blockIdx.y;
    for (int64_t m = threadIdx.x; m < M; m += blockDim.x) row[m] = 0.f;
    __syncthreads();
    const float* g = grad_out + (b * C + c) * N;
    const int32_t* I = idx + b * N * 3;
    const float* W = weights + b * N * 3;
    for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
        const float gv = g[n];
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const int32_t m = I[3 * n + t];
            if (m >= 0 && m < M) atomicAdd(&row[m], __fmul_rn(gv, W[3 * n + t]));
        }
    }
    __syncthreads();
    float* dst = grad_features + (b * C + c) * M;
    for (int64_t m = threadIdx.x; m < M; m += blockDim.x) dst[m] = row[m];
}

__global__ void __launch_bounds__(256)
interp_bwd_global_kernel(const float* __restrict__ grad_out, const int32_t* __restrict__ idx,
                         const float* __restrict__ weights, int64_t C, int64_t M, int64_t N,
                         float* __restrict__ grad_features) {
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t b = blockIdx.z;
    const int64_t c0 = (int64_t)blockIdx.y * kChanPerThread;
    if (n >= N) return;
    const int32_t* I = idx + (b * N + n) * 3;
    const float* W = weights + (b * N + n) * 3;
    const int64_t c1 = min64(C, c0 + kChanPerThread);
    for (int64_t c = c0; c < c1; ++c) {
        const float gv = grad_out[(b * C + c) * N + n];
        float* dst = grad_features + (b * C + c) * M;
#pragma unroll
        for (int t = 0; t < 3; ++t)
            if (I[t] >= 0 && I[t] < M) atomicAdd(dst + I[t], __fmul_rn(gv, W[t]));
    }
}

// flag = 1 if any of the n indices lies outside [0, upper).
template <typename T>
__global__ void index_check_kernel(const T* __restrict__ idx, int64_t n, int64_t upper,
                                   int32_t* __restrict__ flag) {
    bool bad = false;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = (int64_t)idx[e];
        bad |= v < 0 || v >= upper;
    }
    if (__any_sync(FULL_MASK, bad) && (threadIdx.x & 31) == 0) *flag = 1;
}

}  // namespace
}  // namespace mpo

extern "C" {

int mpo_index_check(const void* idx, int idx_is_int64, int64_t n, int64_t upper, int32_t* flag,
                    void* stream) {
    using namespace mpo;
    MPO_REQUIRE(n >= 0, "negative size");
    MPO_REQUIRE(flag, "null flag pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(flag, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(kCudaError, "mpo_index_check: memset failed");
    if (n == 0) return kOk;
    MPO_REQUIRE(idx, "null pointer");
    const unsigned grid = (unsigned)min64(ceil_div(n, 256), (int64_t)sm_count() * 8);
    if (idx_is_int64)
        index_check_kernel<int64_t><<<grid, 256, 0, s>>>(static_cast<const int64_t*>(idx), n,
                                                         upper, flag);
    else
        index_check_kernel<int32_t><<<grid, 256, 0, s>>>(static_cast<const int32_t*>(idx), n,
                                                         upper, flag);
    return check_launch("index_check_kernel");
}

int mpo_three_interpolate(const float* features, const int32_t* idx, const float* weights,
                          int64_t B, int64_t C, int64_t M, int64_t N, float* out, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && M >= 0 && N >= 0, "negative size");
    if (B == 0 || C == 0 || N == 0) return kOk;
    MPO_REQUIRE(M >= 1, "nonempty interpolation requires at least one source point");
    MPO_REQUIRE(features && idx && weights && out, "null pointer");
    MPO_REQUIRE(B <= 65535 && ceil_div(C, kChanPerThread) <= 65535, "batch or channels too large");
    dim3 grid((unsigned)ceil_div(N, 256), (unsigned)ceil_div(C, kChanPerThread), (unsigned)B);
    interp_fwd_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(features, idx, weights, C, M, N, out);
    return check_launch("interp_fwd_kernel");
}

int mpo_three_interpolate_backward(const float* grad_out, const int32_t* idx,
                                   const float* weights, int64_t B, int64_t C, int64_t M,
                                   int64_t N, float* grad_features, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && M >= 0 && N >= 0, "negative size");
    if (B == 0 || C == 0 || M == 0) return kOk;
    MPO_REQUIRE(grad_features, "null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    if (N == 0) {
        if (cudaMemsetAsync(grad_features, 0, sizeof(float) * B * C * M, s) != cudaSuccess)
            return fail(kCudaError, "mpo_three_interpolate_backward: memset failed");
        return kOk;
    }
    MPO_REQUIRE(grad_out && idx && weights, "null pointer");
    const size_t smem = (size_t)M * sizeof(float);
    if (smem <= 192 * 1024 && C <= 2147483647 && B <= 65535) {
        if (cudaFuncSetAttribute(interp_bwd_smem_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return fail(kCudaError, "three_interpolate_backward: shared-memory limit");
        dim3 grid((unsigned)C, (unsigned)B);
        interp_bwd_smem_kernel<<<grid, 512, smem, s>>>(grad_out, idx, weights, C, M, N,
                                                       grad_features);
        return check_launch("interp_bwd_smem_kernel");
    }
    if (cudaMemsetAsync(grad_features, 0, sizeof(float) * B * C * M, s) != cudaSuccess)
        return fail(kCudaError, "mpo_three_interpolate_backward: memset failed");
    dim3 grid((unsigned)ceil_div(N, 256), (unsigned)ceil_div(C, kChanPerThread), (unsigned)B);
    interp_bwd_global_kernel<<<grid, 256, 0, s>>>(grad_out, idx, weights, C, M, N, grad_features);
    return check_launch("interp_bwd_global_kernel");
}

}  // extern "C"
