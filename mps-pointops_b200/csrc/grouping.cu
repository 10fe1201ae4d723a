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
// Design (B200): bandwidth-bound gathers.  A thread owns one (b, p, s) slot and
// a slice of eight channels: it loads its index once, issues the channel
// loads together, then writes them, so the (B, C, P, S) output is written
// coalesced along (p, s).  Gathering straight from the (B, C, N) features
// reads one 32-byte sector per 4-byte value (the slots of a warp hit random
// points), so when every point is gathered several times (P * S >= N) the
// features are first transposed to (B, N, C) in a caller workspace and
// gathered through shared-memory tiles (group_tile_kernel) with coalesced
// reads and writes.  The fused form writes the concatenated (B, 3 + C, P, S)
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
    // All loads of the slot first (independent, in flight together), then the
    // coalesced stores.
    float v[kChan];
#pragma unroll
    for (int u = 0; u < kChan; ++u)
        v[u] = (ok && c0 + u < c1) ? __ldg(features + (b * C + c0 + u) * N + j) : 0.f;
#pragma unroll
    for (int u = 0; u < kChan; ++u)
        if (c0 + u < c1) out[(b * C + c0 + u) * PS + e] = v[u];
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

// (B, C, N) -> (B, N, C) through 32 x 33 shared-memory tiles.
__global__ void __launch_bounds__(1024)
transpose_cn_kernel(const float* __restrict__ in, int64_t C, int64_t N, float* __restrict__ out) {
    __shared__ float tile[32][33];
    const int64_t b = blockIdx.z;
    const int64_t n0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;
    if (c0 + ty < C && n0 + tx < N) tile[ty][tx] = in[(b * C + c0 + ty) * N + n0 + tx];
    __syncthreads();
    if (n0 + ty < N && c0 + tx < C) out[(b * N + n0 + ty) * C + c0 + tx] = tile[tx][ty];
}

// Gather from transposed (B, N, C) features through a shared-memory tile, so
// that both global phases are coalesced: a CTA owns 32 slots x 64 channels;
// each warp reads whole channel runs of its slots' points (consecutive floats
// of one row), the tile is stored transposed, and each warp writes whole
// 32-slot runs of output rows.  (A thread-per-slot gather touches one cache
// line per lane on every load: 32 L1 wavefronts per instruction.)  With
// X = 3 (the fused grouping) the CTAs of channel block 0 also write the three
// centred coordinate rows, and the features go to output rows 3 .. 3 + C.
constexpr int kTileSlots = 32, kTileChans = 64;

template <typename IDX>
__global__ void __launch_bounds__(kThreads)
group_tile_kernel(const float* __restrict__ ft, const IDX* __restrict__ idx,
                  const float* __restrict__ xyz, const float* __restrict__ new_xyz, int64_t N,
                  int64_t P, int64_t S, int64_t C, int X, float* __restrict__ out) {
    __shared__ float tile[kTileChans][kTileSlots + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t PS = P * S;
    const int64_t b = blockIdx.z;
    const int64_t e0 = (int64_t)blockIdx.x * kTileSlots;
    const int64_t c0 = (int64_t)blockIdx.y * kTileChans;
    const int64_t Cout = X + C;
#pragma unroll
    for (int r = 0; r < kTileSlots / 8; ++r) {
        const int sl = warp + 8 * r;
        const int64_t e = e0 + sl;
        int64_t j = -1;
        if (e < PS) j = (int64_t)idx[b * PS + e];
        const bool ok = j >= 0 && j < N;
#pragma unroll
        for (int h = 0; h < kTileChans / 32; ++h) {
            const int64_t c = c0 + 32 * h + lane;
            tile[32 * h + lane][sl] = (ok && c < C) ? __ldg(ft + (b * N + j) * C + c) : 0.f;
        }
    }
    __syncthreads();
    const int64_t e = e0 + lane;
    if (e >= PS) return;
#pragma unroll
    for (int r = 0; r < kTileChans / 8; ++r) {
        const int cc = warp + 8 * r;
        if (c0 + cc < C) out[(b * Cout + X + c0 + cc) * PS + e] = tile[cc][lane];
    }
    if (X && blockIdx.y == 0 && warp < 3) {
        const int64_t j = (int64_t)idx[b * PS + e];
        const int64_t p = e / S;
        const bool ok = j >= 0 && j < N;
        out[(b * Cout + warp) * PS + e] =
            ok ? __fsub_rn(__ldg(xyz + (b * N + j) * 3 + warp), __ldg(new_xyz + (b * P + p) * 3 + warp))
               : 0.f;
    }
}

// Backward through the same tiles: the gradient rows are read coalesced
// (32 slots of one channel per warp instruction) into a transposed tile, and
// each warp then adds a slot's channel run into its point's row of the
// transposed (B, N, C) gradient -- consecutive addresses, so a warp's atomic
// adds hit one or two cache lines instead of 32.  With X = 3 the CTAs of
// channel block 0 also add the coordinate rows into grad_xyz.
template <typename IDX>
__global__ void __launch_bounds__(kThreads)
group_tile_bwd_kernel(const float* __restrict__ grad, const IDX* __restrict__ idx, int64_t N,
                      int64_t PS, int64_t C, int X, float* __restrict__ gt,
                      float* __restrict__ grad_xyz) {
    __shared__ float tile[kTileChans][kTileSlots + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.z;
    const int64_t e0 = (int64_t)blockIdx.x * kTileSlots;
    const int64_t c0 = (int64_t)blockIdx.y * kTileChans;
    const int64_t Cout = X + C;
    const int64_t e = e0 + lane;
#pragma unroll
    for (int r = 0; r < kTileChans / 8; ++r) {
        const int cc = warp + 8 * r;
        tile[cc][lane] = (c0 + cc < C && e < PS) ? grad[(b * Cout + X + c0 + cc) * PS + e] : 0.f;
    }
    if (X && grad_xyz && blockIdx.y == 0 && warp < 3 && e < PS) {
        const int64_t j = (int64_t)idx[b * PS + e];
        if (j >= 0 && j < N)
            atomicAdd(grad_xyz + (b * N + j) * 3 + warp, grad[(b * Cout + warp) * PS + e]);
    }
    if (!gt) return;  // no feature gradient wanted (CTA-uniform)
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kTileSlots / 8; ++r) {
        const int sl = warp + 8 * r;
        const int64_t es = e0 + sl;
        if (es >= PS) continue;
        const int64_t j = (int64_t)idx[b * PS + es];
        if (j < 0 || j >= N) continue;
#pragma unroll
        for (int h = 0; h < kTileChans / 32; ++h) {
            const int64_t c = c0 + 32 * h + lane;
            if (c < C) atomicAdd(gt + (b * N + j) * C + c, tile[32 * h + lane][sl]);
        }
    }
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
    float v[kChan];
#pragma unroll
    for (int u = 0; u < kChan; ++u) {
        const int64_t c = c0 + u;
        v[u] = 0.f;
        if (ok && c < c1) {
            if (c < X)
                v[u] = __fsub_rn(__ldg(xyz + (b * N + j) * 3 + c),
                                 __ldg(new_xyz + (b * P + p) * 3 + c));
            else
                v[u] = __ldg(features + (b * C + (c - X)) * N + j);
        }
    }
#pragma unroll
    for (int u = 0; u < kChan; ++u)
        if (c0 + u < c1) out[(b * Cout + c0 + u) * PS + e] = v[u];
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

// Gradient of the fused FPS gather: grad_xyz[b, idx[b,p], k] += grad[b, p, k].
__global__ void __launch_bounds__(kThreads)
gather_points_bwd_kernel(const float* __restrict__ grad, const int32_t* __restrict__ idx,
                         int64_t BP, int64_t N, int64_t P, float* __restrict__ grad_xyz) {
    const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;  // (b, p)
    if (t >= BP) return;
    const int64_t j = idx[t];
    if (j < 0 || j >= N) return;
    float* dst = grad_xyz + ((t / P) * N + j) * 3;
#pragma unroll
    for (int k = 0; k < 3; ++k) atomicAdd(dst + k, grad[t * 3 + k]);
}

dim3 slot_grid(int64_t B, int64_t PS, int64_t channels) {
    return dim3((unsigned)ceil_div(PS, kThreads), (unsigned)ceil_div(channels, kChan), (unsigned)B);
}

// Transposed-feature path: worth its extra pass when every point is gathered
// several times; needs B*N*C floats of workspace.
size_t transposed_bytes(int64_t B, int64_t C, int64_t N, int64_t P, int64_t S) {
    if (B <= 0 || C < 4 || N <= 0 || P * S < N) return 0;
    return (size_t)B * (size_t)N * (size_t)C * sizeof(float);
}

int transpose_features(const float* features, int64_t B, int64_t C, int64_t N, float* ft,
                       cudaStream_t s) {
    const dim3 grid((unsigned)ceil_div(N, 32), (unsigned)ceil_div(C, 32), (unsigned)B);
    transpose_cn_kernel<<<grid, dim3(32, 32), 0, s>>>(features, C, N, ft);
    return check_launch("transpose_cn_kernel");
}

bool use_workspace(void* ws, size_t ws_bytes, size_t need) {
    return need > 0 && ws != nullptr && ws_bytes >= need &&
           (reinterpret_cast<uintptr_t>(ws) & 15u) == 0;
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_group_points_workspace_bytes(int64_t B, int64_t C, int64_t N, int64_t P, int64_t S) {
    return mpo::transposed_bytes(B, C, N, P, S);
}

int mpo_group_points(const float* features, const void* idx, int idx_is_int64, int64_t B,
                     int64_t C, int64_t N, int64_t P, int64_t S, float* out, void* workspace,
                     size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && N >= 0 && P >= 0 && S >= 0, "negative size");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    MPO_REQUIRE(ceil_div(C, kChan) <= 65535 && ceil_div(C, 32) <= 65535, "too many channels");
    if (B == 0 || C == 0 || P == 0 || S == 0) return kOk;
    MPO_REQUIRE(idx && out && (features || N == 0), "null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t PS = P * S;
    if (use_workspace(workspace, workspace_bytes, transposed_bytes(B, C, N, P, S))) {
        float* ft = static_cast<float*>(workspace);
        int st = transpose_features(features, B, C, N, ft, s);
        if (st) return st;
        const dim3 grid((unsigned)ceil_div(PS, kTileSlots), (unsigned)ceil_div(C, kTileChans),
                        (unsigned)B);
        if (idx_is_int64)
            group_tile_kernel<int64_t><<<grid, kThreads, 0, s>>>(
                ft, static_cast<const int64_t*>(idx), nullptr, nullptr, N, PS, 1, C, 0, out);
        else
            group_tile_kernel<int32_t><<<grid, kThreads, 0, s>>>(
                ft, static_cast<const int32_t*>(idx), nullptr, nullptr, N, PS, 1, C, 0, out);
        return check_launch("group_tile_kernel");
    }
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
                              float* grad_features, void* workspace, size_t workspace_bytes,
                              void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && C >= 0 && N >= 0 && P >= 0 && S >= 0, "negative size");
    MPO_REQUIRE(B <= 65535, "batch must be at most 65535");
    MPO_REQUIRE(ceil_div(C, kChan) <= 65535 && N <= (int64_t)65535 * 32, "sizes too large");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t PS = P * S;
    const size_t need = transposed_bytes(B, C, N, P, S);
    if (PS > 0 && use_workspace(workspace, workspace_bytes, need)) {
        MPO_REQUIRE(idx && grad_out && grad_features, "null pointer");
        float* gt = static_cast<float*>(workspace);
        if (cudaMemsetAsync(gt, 0, need, s) != cudaSuccess)
            return fail(kCudaError, "mpo_group_points_backward: memset failed");
        const dim3 grid((unsigned)ceil_div(PS, kTileSlots), (unsigned)ceil_div(C, kTileChans),
                        (unsigned)B);
        if (idx_is_int64)
            group_tile_bwd_kernel<int64_t><<<grid, kThreads, 0, s>>>(
                grad_out, static_cast<const int64_t*>(idx), N, PS, C, 0, gt, nullptr);
        else
            group_tile_bwd_kernel<int32_t><<<grid, kThreads, 0, s>>>(
                grad_out, static_cast<const int32_t*>(idx), N, PS, C, 0, gt, nullptr);
        int st = check_launch("group_tile_bwd_kernel");
        if (st) return st;
        return transpose_features(gt, B, N, C, grad_features, s);  // (B,N,C) -> (B,C,N)
    }
    if (B * C * N > 0) {
        MPO_REQUIRE(grad_features, "null pointer");
        if (cudaMemsetAsync(grad_features, 0, sizeof(float) * B * C * N, s) != cudaSuccess)
            return fail(kCudaError, "mpo_group_points_backward: memset failed");
    }
    if (B == 0 || C == 0 || N == 0 || P == 0 || S == 0) return kOk;
    MPO_REQUIRE(idx && grad_out, "null pointer");
    if (idx_is_int64)
        group_bwd_kernel<int64_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            grad_out, static_cast<const int64_t*>(idx), C, N, PS, grad_features);
    else
        group_bwd_kernel<int32_t><<<slot_grid(B, PS, C), kThreads, 0, s>>>(
            grad_out, static_cast<const int32_t*>(idx), C, N, PS, grad_features);
    return check_launch("group_bwd_kernel");
}

size_t mpo_query_and_group_workspace_bytes(int64_t B, int64_t N, int64_t P, int64_t S,
                                           int64_t C) {
    return mpo::transposed_bytes(B, C, N, P, S);
}

int mpo_query_and_group(const float* xyz, const float* new_xyz, const float* features,
                        int64_t B, int64_t N, int64_t P, int64_t S, int64_t C, float radius_sq,
                        int use_xyz, int32_t* idx, float* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
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
    if (use_workspace(workspace, workspace_bytes, transposed_bytes(B, C, N, P, S))) {
        float* ft = static_cast<float*>(workspace);
        st = transpose_features(features, B, C, N, ft, s);
        if (st) return st;
        const dim3 grid((unsigned)ceil_div(P * S, kTileSlots), (unsigned)ceil_div(C, kTileChans),
                        (unsigned)B);
        group_tile_kernel<int32_t><<<grid, kThreads, 0, s>>>(ft, idx, xyz, new_xyz, N, P, S, C,
                                                             use_xyz ? 3 : 0, out);
        return check_launch("group_tile_kernel");
    }
    query_group_fwd_kernel<<<slot_grid(B, P * S, Cout), kThreads, 0, s>>>(
        xyz, new_xyz, features, idx, N, P, S, C, use_xyz ? 1 : 0, out);
    return check_launch("query_group_fwd_kernel");
}

int mpo_query_and_group_backward(const float* grad_out, const int32_t* idx, int64_t B, int64_t N,
                                 int64_t P, int64_t S, int64_t C, int use_xyz, float* grad_xyz,
                                 float* grad_new_xyz, float* grad_features, void* workspace,
                                 size_t workspace_bytes, void* stream) {
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
    const size_t need = transposed_bytes(B, C, N, P, S);
    if (grad_features && use_workspace(workspace, workspace_bytes, need) &&
        N <= (int64_t)65535 * 32) {
        float* gt = static_cast<float*>(workspace);
        if (cudaMemsetAsync(gt, 0, need, s) != cudaSuccess)
            return fail(kCudaError, "mpo_query_and_group_backward: memset failed");
        const dim3 grid((unsigned)ceil_div(P * S, kTileSlots), (unsigned)ceil_div(C, kTileChans),
                        (unsigned)B);
        group_tile_bwd_kernel<int32_t><<<grid, kThreads, 0, s>>>(grad_out, idx, N, P * S, C, X, gt,
                                                                 grad_xyz);
        int st = check_launch("group_tile_bwd_kernel");
        if (st) return st;
        return transpose_features(gt, B, N, C, grad_features, s);  // (B,N,C) -> (B,C,N)
    }
    query_group_bwd_kernel<<<slot_grid(B, P * S, Cout), kThreads, 0, s>>>(
        grad_out, idx, N, P, S, C, X, grad_xyz, grad_features);
    return check_launch("query_group_bwd_kernel");
}

int mpo_gather_points_backward(const float* grad, const int32_t* idx, int64_t B, int64_t N,
                               int64_t P, float* grad_xyz, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && P >= 0, "negative size");
    cudaStream_t s = (cudaStream_t)stream;
    if (B * N > 0) {
        MPO_REQUIRE(grad_xyz, "null pointer");
        if (cudaMemsetAsync(grad_xyz, 0, sizeof(float) * B * N * 3, s) != cudaSuccess)
            return fail(kCudaError, "mpo_gather_points_backward: memset failed");
    }
    if (B * N == 0 || P == 0) return kOk;
    MPO_REQUIRE(grad && idx, "null pointer");
    gather_points_bwd_kernel<<<(unsigned)ceil_div(B * P, kThreads), kThreads, 0, s>>>(
        grad, idx, B * P, N, P, grad_xyz);
    return check_launch("gather_points_bwd_kernel");
}

}  // extern "C"
