// PointNet++ set-abstraction grouping on sm_100a: gather_operation,
// grouping_operation and the fused ball-query grouping (QueryAndGroup), with
// their backward passes.
//
// Contracts (gamzerA/mps-pointops):
//   gather_operation    mps_pointops/compat.py:62-65  out[b,c,p]   = F[b,c,I[b,p]]
//   grouping_operation  mps_pointops/compat.py:68-73  out[b,c,p,s] = F[b,c,I[b,p,s]]
//   query-and-group     tests/test_pointnet2_e2e.py:40-44: ball query (pointnet2 form),
//                       grouped xyz minus the centre, grouped features, concatenated
//                       along channels: out[b, 0:3, p, s] = xyz[b, I, :] - new_xyz[b, p, :]
//                       (one rounded subtraction), out[b, 3 + c, p, s] = F[b, c, I].
// The forward passes are exact copies (and one subtraction), so they are
// bit-identical to torch's gather.  The backward passes scatter-add the
// gradient into the sources with float atomics (the order of the additions
// into one source element is not fixed, as with torch's scatter_add on CUDA).
//
// Design (B200): HBM-bound gathers.  A thread owns one (b, p, s) slot and a
// slice of channels: it loads its index once and walks the channels, so the
// (B, C, P, S) output is written coalesced along (p, s) and each source row
// stays hot in L1/L2.  The fused form writes the concatenated (B, 3 + C, P, S)
// tensor once -- no (B, 3, P, S) and (B, C, P, S) temporaries, no subtraction
// pass, no concatenation copy, and no int32 -> int64 index cast.  Indices
// outside [0, N) read as zero in the forward and are skipped by the backward,
// so the kernels stay memory-safe on input that the caller's index check
// (mpo_index_check) rejects afterwards.
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kThreads = 256;
constexpr int kChan = 8;  // channels per thread

template <typename IDX>
__global__ void __launch_bounds__(kThreads)
group_fwd_kernel(const float* __restrict__ features, const IDX* __restrict__ idx, int64_t C,
                 int64_t N, int64_t PS, float* __restrict__ out) {
    const int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (e >= PS) return;
    const int64_t b = blockIdx.z;
    const int64_t c0 = (int64_t)blockIdx.y * kChan;
    const int64_t j = (int64_t)idx[b * PS + e];
    const bool ok = j >= 0 && j < N;
    const int64_t c1 = min64(C, c0 + kChan);
    for (int64_t c = c0; c < c1; ++c)
        out[(b * C + c) * PS + e] = ok ? __ldg(features + (b * C + c) * N + j) : 0.f;
}

template <typename IDX>
__global__ void __launch_bounds__(kThreads)
group_bwd_kernel(const float* __restrict__ grad, const IDX* __restrict__ idx, int64_t C,
                 int64_t N, int64_t PS, float* __restrict__ grad_features) {
    const int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (e >= PS) return;
    const int64_t b = blockIdx.z;
    const int64_t c0 = (int64_t)blockIdx.y * kChan;
    const int64_t j = (int64_t)idx[b * PS + e];
    if (j < 0 || j >= N) return;
    const int64_t c1 = min64(C, c0 + kChan);
    for (int64_t c = c0; c < c1; ++c)
        atomicAdd(grad_features + (b * C + c) * N + j, grad[(b * C + c) * PS + e]);
}

// Fused grouping: output channels [0, 3) (when use_xyz) are the centred
// coordinates, the rest the grouped features.
__global__ void __launch_bounds__(kThreads)
query_group_fwd_kernel(const float* __restrict__ xyz, const float* __restrict__ new_xyz,
                       const float* __restrict__ features, const int32_t* __restrict__ idx,
                       int64_t N, int64_t P, int64_t S, int64_t C, int use_xyz,
                       float* __restrict__ out) {
    const int64_t PS = P * S;
    const int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (e >= PS) return;
    const int64_t b = blockIdx.z;
    const int64_t X = use_xyz ? 3 : 0;
    const int64_t Cout = X + C;
    const int64_t c0 = (int64_t)blockIdx.y * kChan;
    const int64_t c1 = min64(Cout, c0 + kChan);
    const int64_t j = idx[b * PS + e];
    const bool ok = j >= 0 && j < N;
    const int64_t p = e / S;
    for (int64_t c = c0; c < c1; ++c) {
        float v = 0.f;
        if (c < X) {
            if (ok) v = __fsub_rn(__ldg(xyz + (b * N + j) * 3 + c), __ldg(new_xyz + (b * P + p) * 3 + c));
        } else if (ok) {
            v = __ldg(features + (b * C + (c - X)) * N + j);
        }
        out[(b * Cout + c) * PS + e] = v;
    }
}

__global__ void __launch_bounds__(kThreads)
query_group_bwd_kernel(const float* __restrict__ grad, const int32_t* __restrict__ idx,
                       int64_t N, int64_t P, int64_t S, int64_t C, int use_xyz,
                       float* __restrict__ grad_xyz, float* __restrict__ grad_features) {
    const int64_t PS = P * S;
    const int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (e >= PS) return;
    const int64_t b = blockIdx.z;
    const int64_t X = use_xyz ? 3 : 0;
    const int64_t Cout = X + C;
    const int64_t c0 = (int64_t)blockIdx.y * kChan;
    const int64_t c1 = min64(Cout, c0 + kChan);
    const int64_t j = idx[b * PS + e];
    if (j < 0 || j >= N) return;
    for (int64_t c = c0; c < c1; ++c) {
        const float g = grad[(b * Cout + c) * PS + e];
        if (c < X) {
            if (grad_xyz) atomicAdd(grad_xyz + (b * N + j) * 3 + c, g);
        } else if (grad_features) {
            atomicAdd(grad_features + (b * C + (c - X)) * N + j, g);
        }
    }
}

// Gradient of the centre subtraction: grad_new_xyz[b,p,k] = -(sum over s of
// grad[b,k,p,s]), summed in slot order.
__global__ void __launch_bounds__(kThreads)
centre_grad_kernel(const float* __restrict__ grad, int64_t B, int64_t P, int64_t S,
                   int64_t Cout, float* __restrict__ grad_new_xyz) {
    const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;  // (b, p, k)
    if (t >= B * P * 3) return;
    const int64_t k = t % 3, p = (t / 3) % P, b = t / (3 * P);
    const float* g = grad + ((b * Cout + k) * P + p) * S;
    float acc = 0.f;
    for (int64_t s = 0; s < S; ++s) acc = __fadd_rn(acc, g[s]);
    grad_new_xyz[t] = -acc;
}

dim3 slot_grid(int64_t B, int64_t PS, int64_t channels) {
    return dim3((unsigned)ceil_div(PS, kThreads), (unsigned)ceil_div(channels, kChan), (unsigned)B);
}

}  // namespace
}  // namespace mpo

extern "C" {

int mpo_group_points(const float* features, const void* idx, int idx_is_int64, int64_t B,
                     int64_t C, int64_t N, int64_t P, int64_t S, float* out, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && N >= 0 && P >= 0 && S >= 0, "negative size");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    MPO_REQUIRE(ceil_div(C, kChan) <= 65535, "too many channels");
    if (B == 0 || C == 0 || P == 0 || S == 0) return kOk;
    MPO_REQUIRE(idx && out && (features || N == 0), "null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t PS = P * S;
    if (idx_is_int64)
        group_fwd_kernel<int64_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            features, static_cast<const int64_t*>(idx), C, N, PS, out);
    else
        group_fwd_kernel<int32_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            features, static_cast<const int32_t*>(idx), C, N, PS, out);
    return check_launch("group_fwd_kernel");
}

int mpo_group_points_backward(const float* grad_out, const void* idx, int idx_is_int64,
                              int64_t B, int64_t C, int64_t N, int64_t P, int64_t S,
                              float* grad_features, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && N >= 0 && P >= 0 && S >= 0, "negative size");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    MPO_REQUIRE(ceil_div(C, kChan) <= 65535, "too many channels");
    cudaStream_t s = (cudaStream_t)stream;
    if (B * C * N > 0) {
        MPO_REQUIRE(grad_features, "null pointer");
        if (cudaMemsetAsync(grad_features, 0, sizeof(float) * B * C * N, s) != cudaSuccess)
            return fail(kCudaError, "mpo_group_points_backward: memset failed");
    }
    if (B == 0 || C == 0 || N == 0 || P == 0 || S == 0) return kOk;
    MPO_REQUIRE(idx && grad_out, "null pointer");
    const int64_t PS = P * S;
    if (idx_is_int64)
        group_bwd_kernel<int64_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            grad_out, static_cast<const int64_t*>(idx), C, N, PS, grad_features);
    else
        group_bwd_kernel<int32_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            grad_out, static_cast<const int32_t*>(idx), C, N, PS, grad_features);
    return check_launch("group_bwd_kernel");
}

int mpo_query_and_group(const float* xyz, const float* new_xyz, const float* features,
                        int64_t B, int64_t N, int64_t P, int64_t S, int64_t C, float radius_sq,
                        int use_xyz, int32_t* idx, float* out, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && P >= 0 && S >= 0 && C >= 0, "negative size");
    MPO_REQUIRE(use_xyz || C > 0, "use_xyz = 0 needs features");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    const int64_t Cout = (use_xyz ? 3 : 0) + C;
    MPO_REQUIRE(ceil_div(Cout, kChan) <= 65535, "too many channels");
    if (B == 0 || P == 0 || S == 0) return kOk;
    MPO_REQUIRE(new_xyz && idx && out && (xyz || N == 0) && (features || C == 0 || N == 0),
                "null pointer");
    int st = mpo_ball_query_pointnet2(xyz, new_xyz, B, N, P, S, radius_sq, idx, stream);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    query_group_fwd_kernel<<<slot_grid(B, P * S, Cout), kThreads, 0, s>>>(
        xyz, new_xyz, features, idx, N, P, S, C, use_xyz ? 1 : 0, out);
    return check_launch("query_group_fwd_kernel");
}

int mpo_query_and_group_backward(const float* grad_out, const int32_t* idx, int64_t B, int64_t N,
                                 int64_t P, int64_t S, int64_t C, int use_xyz, float* grad_xyz,
                                 float* grad_new_xyz, float* grad_features, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && P >= 0 && S >= 0 && C >= 0, "negative size");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    const int X = use_xyz ? 3 : 0;
    const int64_t Cout = X + C;
    MPO_REQUIRE(ceil_div(Cout, kChan) <= 65535, "too many channels");
    cudaStream_t s = (cudaStream_t)stream;
    if (grad_xyz && B * N > 0) {
        if (cudaMemsetAsync(grad_xyz, 0, sizeof(float) * B * N * 3, s) != cudaSuccess)
            return fail(kCudaError, "mpo_query_and_group_backward: memset failed");
    }
    if (grad_features && B * C * N > 0) {
        if (cudaMemsetAsync(grad_features, 0, sizeof(float) * B * C * N, s) != cudaSuccess)
            return fail(kCudaError, "mpo_query_and_group_backward: memset failed");
    }
    if (grad_new_xyz && B * P > 0) {
        if (!X || S == 0) {
            if (cudaMemsetAsync(grad_new_xyz, 0, sizeof(float) * B * P * 3, s) != cudaSuccess)
                return fail(kCudaError, "mpo_query_and_group_backward: memset failed");
        } else {
            MPO_REQUIRE(grad_out, "null pointer");
            centre_grad_kernel<<<(unsigned)ceil_div(B * P * 3, kThreads), kThreads, 0, s>>>(
                grad_out, B, P, S, Cout, grad_new_xyz);
            int st = check_launch("centre_grad_kernel");
            if (st) return st;
        }
    }
    if (B == 0 || N == 0 || P == 0 || S == 0 || (!grad_xyz && !grad_features)) return kOk;
    MPO_REQUIRE(idx && grad_out, "null pointer");
    query_group_bwd_kernel<<<slot_grid(B, P * S, Cout), kThreads, 0, s>>>(
        grad_out, idx, N, P, S, C, X, grad_xyz, grad_features);
    return check_launch("query_group_bwd_kernel");
}

}  // extern "C"
