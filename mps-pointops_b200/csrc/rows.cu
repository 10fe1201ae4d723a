// Row gathers with -1 padding and the flat inverse-distance interpolation, on
// sm_100a: the neighbour gathers of the PyTorch3D ball-query adapter
// (gamzerA/mps-pointops mps_pointops/pytorch3d.py:26-38) and of Pointcept's
// `grouping` (pointcept.py:168-203), and Pointcept's `interpolation`
// (pointcept.py:219-243), with their backwards.
//
// Layout: row-major float rows in HBM.  The gathers run one thread per output
// element (consecutive threads read consecutive columns of one source row and
// write consecutive output words), so a warp moves whole rows with coalesced
// accesses; indices outside [0, N) give zero rows (memory-safe on any input).
// The interpolation runs one warp per query row: the lanes compute the row's
// weights redundantly, in the reference's order, then each lane produces
// columns c = lane, lane + 32, ... as the sequential sum over the k
// neighbours of rounded products.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ int64_t load_index(const void* idx, int idx_int32, int64_t e) {
    return idx_int32 ? (int64_t)static_cast<const int32_t*>(idx)[e]
                     : static_cast<const int64_t*>(idx)[e];
}

// out[(b R + r) * stride + offset + w] = src[(b N + i) W + w] (- centers[...])
// for i = idx[b R + r] in [0, N), else 0.
__global__ void __launch_bounds__(kRowThreads)
gather_rows_kernel(const float* __restrict__ src, int64_t B, int64_t N, int64_t W,
                   const void* __restrict__ idx, int idx_int32, int64_t R,
                   const float* __restrict__ centers, int64_t K, float* __restrict__ out,
                   int64_t stride, int64_t offset) {
    const int64_t total = B * R * W;
    for (int64_t e = (int64_t)blockIdx.x * kRowThreads + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * kRowThreads) {
        const int64_t row = e / W, w = e - row * W;
        const int64_t b = row / R;
        const int64_t i = load_index(idx, idx_int32, row);
        float v = 0.f;
        if (i >= 0 && i < N) {
            v = src[(b * N + i) * W + w];
            if (centers) v = __fsub_rn(v, centers[(row / K) * W + w]);
        }
        out[row * stride + offset + w] = v;
    }
}

// grad_src[(b N + i) W + w] += g; grad_centers[(row / K) W + w] -= g.
__global__ void __launch_bounds__(kRowThreads)
gather_rows_bwd_kernel(const float* __restrict__ grad_out, int64_t stride, int64_t offset,
                       int64_t B, int64_t N, int64_t W, const void* __restrict__ idx,
                       int idx_int32, int64_t R, int64_t K, float* __restrict__ grad_src,
                       float* __restrict__ grad_centers) {
    const int64_t total = B * R * W;
    for (int64_t e = (int64_t)blockIdx.x * kRowThreads + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * kRowThreads) {
        const int64_t row = e / W, w = e - row * W;
        const int64_t b = row / R;
        const int64_t i = load_index(idx, idx_int32, row);
        if (i < 0 || i >= N) continue;
        const float g = grad_out[row * stride + offset + w];
        if (grad_src) atomicAdd(grad_src + (b * N + i) * W + w, g);
        if (grad_centers) atomicAdd(grad_centers + (row / K) * W + w, -g);
    }
}

// Weight of neighbour t of a query row (pointcept.py:232-236):
// r_t = 1 / (d_t + 1e-8) for a valid neighbour, else 0; w_t = r_t / max(sum r, 1e-20).
__device__ __forceinline__ float interp_recip(int32_t i, float d, int64_t N) {
    return (i >= 0 && i < N) ? __fdiv_rn(1.0f, __fadd_rn(d, 1e-8f)) : 0.f;
}

__global__ void __launch_bounds__(kRowThreads)
flat_interp_kernel(const float* __restrict__ feat, int64_t N, int64_t C,
                   const int32_t* __restrict__ idx, const float* __restrict__ dist, int64_t M,
                   int k, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kRowThreads / 32);
    for (int64_t m = (int64_t)blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5); m < M;
         m += warps) {
        const int32_t* ir = idx + m * k;
        const float* dr = dist + m * k;
        float norm = 0.f;
        for (int t = 0; t < k; ++t) norm = __fadd_rn(norm, interp_recip(ir[t], dr[t], N));
        const float den = fmaxf(norm, 1e-20f);
        for (int64_t c = lane; c < C; c += 32) {
            float acc = 0.f;
            for (int t = 0; t < k; ++t) {
                const int32_t i = ir[t];
                const float wt = __fdiv_rn(interp_recip(i, dr[t], N), den);
                const float f = (i >= 0 && i < N) ? feat[(int64_t)i * C + c] : 0.f;
                acc = __fadd_rn(acc, __fmul_rn(f, wt));
            }
            out[m * C + c] = acc;
        }
    }
}

// grad_feat[i_t, c] += w_t * grad_out[m, c] (the weights carry no gradient).
__global__ void __launch_bounds__(kRowThreads)
flat_interp_bwd_kernel(const float* __restrict__ grad_out, const int32_t* __restrict__ idx,
                       const float* __restrict__ dist, int64_t M, int k, int64_t N, int64_t C,
                       float* __restrict__ grad_feat) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kRowThreads / 32);
    for (int64_t m = (int64_t)blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5); m < M;
         m += warps) {
        const int32_t* ir = idx + m * k;
        const float* dr = dist + m * k;
        float norm = 0.f;
        for (int t = 0; t < k; ++t) norm = __fadd_rn(norm, interp_recip(ir[t], dr[t], N));
        const float den = fmaxf(norm, 1e-20f);
        for (int t = 0; t < k; ++t) {
            const int32_t i = ir[t];
            if (i < 0 || i >= N) continue;
            const float wt = __fdiv_rn(interp_recip(i, dr[t], N), den);
            for (int64_t c = lane; c < C; c += 32)
                atomicAdd(grad_feat + (int64_t)i * C + c, __fmul_rn(grad_out[m * C + c], wt));
        }
    }
}

unsigned grid_for(int64_t work, int per_block) {
    const int64_t blocks = ceil_div(work, per_block);
    return (unsigned)min64(max64(blocks, 1), (int64_t)sm_count() * 16);
}

}  // namespace
}  // namespace mpo

extern "C" {

int mpo_gather_rows(const float* src, int64_t B, int64_t N, int64_t W, const void* idx,
                    int idx_int32, int64_t R, const float* centers, int64_t K, float* out,
                    int64_t out_stride, int64_t out_offset, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && W >= 1 && R >= 0, "bad sizes");
    MPO_REQUIRE(out_offset >= 0 && out_stride >= out_offset + W, "bad output stride");
    MPO_REQUIRE(!centers || (K >= 1 && R % K == 0), "K must divide R when centers are given");
    const int64_t total = B * R * W;
    if (total == 0) return kOk;
    MPO_REQUIRE(idx && out && (src || N == 0), "null pointer");
    gather_rows_kernel<<<grid_for(total, kRowThreads), kRowThreads, 0, (cudaStream_t)stream>>>(
        src, B, N, W, idx, idx_int32 ? 1 : 0, R, centers, centers ? K : 1, out, out_stride,
        out_offset);
    return check_launch("gather_rows_kernel");
}

int mpo_gather_rows_backward(const float* grad_out, int64_t out_stride, int64_t out_offset,
                             int64_t B, int64_t N, int64_t W, const void* idx, int idx_int32,
                             int64_t R, int64_t K, float* grad_src, float* grad_centers,
                             void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && W >= 1 && R >= 0, "bad sizes");
    MPO_REQUIRE(out_offset >= 0 && out_stride >= out_offset + W, "bad output stride");
    MPO_REQUIRE(!grad_centers || (K >= 1 && R % K == 0),
                "K must divide R when grad_centers is given");
    const int64_t total = B * R * W;
    if (total == 0 || (!grad_src && !grad_centers)) return kOk;
    MPO_REQUIRE(idx && grad_out, "null pointer");
    gather_rows_bwd_kernel<<<grid_for(total, kRowThreads), kRowThreads, 0,
                             (cudaStream_t)stream>>>(grad_out, out_stride, out_offset, B, N, W,
                                                     idx, idx_int32 ? 1 : 0, R,
                                                     grad_centers ? K : 1, grad_src,
                                                     grad_centers);
    return check_launch("gather_rows_bwd_kernel");
}

int mpo_flat_interpolate(const float* feat, int64_t N, int64_t C, const int32_t* idx,
                         const float* dist, int64_t M, int64_t k, float* out, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(N >= 0 && C >= 0 && M >= 0 && k >= 1 && k <= 0x7fffffff, "bad sizes");
    if (M == 0 || C == 0) return kOk;
    MPO_REQUIRE(idx && dist && out && (feat || N == 0), "null pointer");
    flat_interp_kernel<<<grid_for(M, kRowThreads / 32), kRowThreads, 0, (cudaStream_t)stream>>>(
        feat, N, C, idx, dist, M, (int)k, out);
    return check_launch("flat_interp_kernel");
}

int mpo_flat_interpolate_backward(const float* grad_out, const int32_t* idx, const float* dist,
                                  int64_t M, int64_t k, int64_t N, int64_t C, float* grad_feat,
                                  void* stream) {
    using namespace mpo;
    MPO_REQUIRE(N >= 0 && C >= 0 && M >= 0 && k >= 1 && k <= 0x7fffffff, "bad sizes");
    cudaStream_t s = (cudaStream_t)stream;
    if (N * C > 0) {
        MPO_REQUIRE(grad_feat, "null pointer");
        if (cudaMemsetAsync(grad_feat, 0, sizeof(float) * N * C, s) != cudaSuccess)
            return fail(kCudaError, "mpo_flat_interpolate_backward: memset failed");
    }
    if (M == 0 || C == 0 || N == 0) return kOk;
    MPO_REQUIRE(idx && dist && grad_out, "null pointer");
    flat_interp_bwd_kernel<<<grid_for(M, kRowThreads / 32), kRowThreads, 0, s>>>(
        grad_out, idx, dist, M, (int)k, N, C, grad_feat);
    return check_launch("flat_interp_bwd_kernel");
}

}  // extern "C"
