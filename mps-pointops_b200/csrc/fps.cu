// Farthest point sampling on sm_100a.
//
// Contract: gamzerA/mps-pointops mps_pointops/reference.py:27-58 --
//   out[0] = start_idx; min_d2 = min(min_d2, SD(x, x[out[i]])) with NaN
//   propagating (torch.minimum); out[i+1] = first index of the maximum of
//   min_d2, NaN ranking above every number (torch.argmax).  skip_near_origin
//   starts points with ((x*x + y*y) + z*z) < fl32(1e-3) at -inf
//   (reference.py:46-50).
//
// Design (B200): the whole npoint-step loop runs inside ONE launch.
//   * A cloud is owned by a group of G CTAs of up to 1024 threads; each
//     thread keeps P <= 8 points (x, y, z, min_d2) in registers for the whole
//     run, so a step touches no memory except the argmax exchange.
//   * Argmax per step: each thread scans its points, then a warp reduces
//     (ordered key, index) pairs with two redux.sync instructions (max key,
//     then min index among the lanes holding it), and every warp redundantly
//     reduces the per-warp results from shared memory -- one __syncthreads()
//     per step.
//   * G == 1 (clouds up to 8192 points): the cloud's xyz is also staged in
//     shared memory so the next centroid is a shared-memory load.
//   * G > 1 (large clouds: 2^20 points on 128 SMs): a
//     cooperative launch makes the group co-resident; each CTA publishes its
//     best as a 64-bit key (ordered distance << 32 | ~index) with one
//     atomicMax into a rotating slot and arrives on a counter; thread 0 then
//     spins with ld.acquire on the counter.  The spin is bounded
//     (kSpinLimit); on expiry the CTA records status 1 and returns.
#include <cooperative_groups.h>

#include <mutex>
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kMaxThreads = 1024;
constexpr int kMaxP = 8;
constexpr int64_t kPointsPerCta = (int64_t)kMaxThreads * kMaxP;  // 8192
constexpr unsigned kSpinLimit = 1u << 26;

// Cross-CTA exchange state of one cloud (lives in the caller's workspace,
// zeroed before each launch).
struct GroupSync {
    unsigned long long slot[3];
    unsigned count;
    unsigned error;
};

template <int P, bool GROUP>
__global__ void __launch_bounds__(kMaxThreads, 1)
fps_kernel(const float* __restrict__ xyz, int64_t N, int64_t npoint, int64_t start_idx,
           int skip, int out_int32, void* __restrict__ out, int G, int64_t per_cta,
           int cloud_offset, GroupSync* __restrict__ sync, int32_t* __restrict__ status) {
    extern __shared__ float s_xyz[];  // G == 1 only: the cloud, 3 floats per point
    __shared__ uint32_t s_key[2][32];
    __shared__ uint32_t s_idx[2][32];
    __shared__ uint32_t s_far;
    __shared__ int s_abort;

    const int b = cloud_offset + blockIdx.x / G;
    const int g = blockIdx.x % G;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const int nthr = blockDim.x;
    const float* __restrict__ p = xyz + (size_t)b * (size_t)N * 3;
    const int64_t lo = (int64_t)g * per_cta;
    const int64_t hi = min(N, lo + per_cta);
    GroupSync* gs = GROUP ? sync + b : nullptr;

    float px[P], py[P], pz[P], md[P];
#pragma unroll
    for (int s = 0; s < P; ++s) {
        const int64_t j = lo + tid + (int64_t)s * nthr;
        if (j < hi) {
            px[s] = p[3 * j + 0];
            py[s] = p[3 * j + 1];
            pz[s] = p[3 * j + 2];
            float init = INFINITY;
            if (skip && sqd3(px[s], py[s], pz[s], 0.f, 0.f, 0.f) < 1e-3f) init = -INFINITY;
            md[s] = init;
        } else {
            px[s] = py[s] = pz[s] = 0.f;
            md[s] = -INFINITY;
        }
    }
    if (!GROUP) {
        for (int64_t e = tid; e < 3 * N; e += nthr) s_xyz[e] = p[e];
    }
    if (tid == 0) s_abort = 0;
    bool mine_nonfinite = false;
#pragma unroll
    for (int s = 0; s < P; ++s)
        mine_nonfinite |= !(isfinite(px[s]) && isfinite(py[s]) && isfinite(pz[s]));
    bool nan_mode = __syncthreads_or(mine_nonfinite) != 0;

    uint32_t far = (uint32_t)start_idx;
    float cx, cy, cz;
    if (!GROUP) {
        cx = s_xyz[3 * far + 0];
        cy = s_xyz[3 * far + 1];
        cz = s_xyz[3 * far + 2];
    } else {
        cx = p[3 * (size_t)far + 0];
        cy = p[3 * (size_t)far + 1];
        cz = p[3 * (size_t)far + 2];
    }
    int64_t* out64 = reinterpret_cast<int64_t*>(out) + (size_t)b * npoint;
    int32_t* out32 = reinterpret_cast<int32_t*>(out) + (size_t)b * npoint;

    for (int64_t i = 0; i < npoint; ++i) {
        if (tid == 0 && g == 0) {
            if (out_int32) out32[i] = (int32_t)far;
            else out64[i] = (int64_t)far;
        }
        if (i + 1 == npoint) break;

        // NaN can only enter min_d2 through a non-finite coordinate of this
        // CTA's points or of a centroid; from then on (sticky) the keys must
        // rank NaN above every number, like torch.argmax.
        nan_mode = nan_mode || !(isfinite(cx) && isfinite(cy) && isfinite(cz));
        uint32_t bkey = 0u, bidx = 0xffffffffu;
        if (!nan_mode) {
#pragma unroll
            for (int s = 0; s < P; ++s) {
                const int64_t j = lo + tid + (int64_t)s * nthr;
                const bool valid = j < hi;
                const float d = sqd3(px[s], py[s], pz[s], cx, cy, cz);
                const float m = fminf(md[s], d);
                md[s] = valid ? m : md[s];
                const uint32_t k = valid ? ordered_key(m) : 0u;
                if (k > bkey) {
                    bkey = k;
                    bidx = (uint32_t)j;
                }
            }
        } else {
#pragma unroll
            for (int s = 0; s < P; ++s) {
                const int64_t j = lo + tid + (int64_t)s * nthr;
                const bool valid = j < hi;
                const float d = sqd3(px[s], py[s], pz[s], cx, cy, cz);
                const float m = fmin_nan(md[s], d);
                md[s] = valid ? m : md[s];
                const uint32_t k = !valid ? 0u : (isnan(m) ? 0xffffffffu : ordered_key(m));
                if (k > bkey) {
                    bkey = k;
                    bidx = (uint32_t)j;
                }
            }
        }
        const uint32_t wmax = __reduce_max_sync(FULL_MASK, bkey);
        const uint32_t widx = __reduce_min_sync(FULL_MASK, bkey == wmax ? bidx : 0xffffffffu);
        const int buf = (int)(i & 1);
        if (lane == 0) {
            s_key[buf][warp] = wmax;
            s_idx[buf][warp] = widx;
        }
        __syncthreads();
        const uint32_t k2 = lane < nwarps ? s_key[buf][lane] : 0u;
        const uint32_t i2 = lane < nwarps ? s_idx[buf][lane] : 0xffffffffu;
        const uint32_t cmax = __reduce_max_sync(FULL_MASK, k2);
        const uint32_t cidx = __reduce_min_sync(FULL_MASK, k2 == cmax ? i2 : 0xffffffffu);

        if (!GROUP) {
            far = cidx;
            cx = s_xyz[3 * far + 0];
            cy = s_xyz[3 * far + 1];
            cz = s_xyz[3 * far + 2];
        } else {
            if (tid == 0) {
                const int slot = (int)(i % 3);
                const unsigned long long packed =
                    ((unsigned long long)cmax << 32) | (unsigned long long)(0xffffffffu - cidx);
                atomicMax(&gs->slot[slot], packed);
                __threadfence();
                atomicAdd(&gs->count, 1u);
                const unsigned target = (unsigned)(i + 1) * (unsigned)G;
                unsigned spins = 0;
                while (ld_acquire_u32(&gs->count) < target) {
                    if (++spins > kSpinLimit || ld_acquire_u32(&gs->error) != 0u) {
                        atomicExch(&gs->error, 1u);
                        if (status) atomicExch(status, 1);
                        s_abort = 1;
                        break;
                    }
                }
                const unsigned long long win = ld_relaxed_u64(&gs->slot[slot]);
                s_far = 0xffffffffu - (uint32_t)(win & 0xffffffffull);
                // Step i+2 reuses slot (i+2)%3 == (i-1)%3, which every CTA has
                // finished reading once it arrived for step i.
                if (g == 0) gs->slot[(i + 2) % 3] = 0ull;
            }
            __syncthreads();
            if (s_abort) return;
            far = s_far;
            cx = p[3 * (size_t)far + 0];
            cy = p[3 * (size_t)far + 1];
            cz = p[3 * (size_t)far + 2];
        }
    }
}

template <int P, bool GROUP>
int launch_fps(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
               int skip, int out_int32, void* out, int G, int64_t per_cta, int threads,
               GroupSync* sync, int32_t* status, cudaStream_t stream) {
    auto kern = fps_kernel<P, GROUP>;
    const size_t smem = GROUP ? 0 : (size_t)N * 3 * sizeof(float);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
        return fail(kCudaError, "mpo_fps: cannot set the shared-memory limit");
    }
    if (!GROUP) {
        kern<<<(unsigned)B, threads, smem, stream>>>(xyz, N, npoint, start_idx, skip, out_int32,
                                                     out, 1, per_cta, 0, sync, status);
        return check_launch("mpo_fps");
    }
    // Co-residency of each group is guaranteed by cooperative launch; clouds
    // are processed in waves that fit on the device at one CTA per SM.
    const int sms = sm_count();
    const int clouds_per_wave = sms / G;
    if (clouds_per_wave < 1) return fail(kUnsupported, "mpo_fps: cloud too large for one wave");
    for (int64_t c0 = 0; c0 < B; c0 += clouds_per_wave) {
        const int nc = (int)min64(clouds_per_wave, B - c0);
        int cloud_offset = (int)c0;
        void* args[] = {(void*)&xyz,  (void*)&N,      (void*)&npoint, (void*)&start_idx,
                        (void*)&skip, (void*)&out_int32, (void*)&out,  (void*)&G,
                        (void*)&per_cta, (void*)&cloud_offset, (void*)&sync, (void*)&status};
        cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, dim3(nc * G),
                                                    dim3(threads), args, 0, stream);
        if (e != cudaSuccess) {
            return fail(kCudaError, std::string("mpo_fps: cooperative launch: ") +
                                        cudaGetErrorString(e));
        }
        count_launches(1);
    }
    return kOk;
}

int pick_p(int64_t per_cta) {
    if (per_cta <= 1024) return 1;
    if (per_cta <= 2048) return 2;
    if (per_cta <= 4096) return 4;
    return 8;
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_fps_workspace_bytes(int64_t B, int64_t N, int64_t npoint, int strategy) {
    (void)npoint;
    if (strategy != MPO_FPS_GROUP && N <= mpo::kPointsPerCta) return 0;
    return (size_t)(B > 0 ? B : 1) * sizeof(mpo::GroupSync);
}

int mpo_fps(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
            int skip_near_origin, int out_int32, int strategy, void* out, int32_t* status_out,
            void* workspace, size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && npoint >= 0, "negative size");
    MPO_REQUIRE(strategy == MPO_FPS_AUTO || strategy == MPO_FPS_SINGLE ||
                    strategy == MPO_FPS_GROUP,
                "unknown strategy");
    cudaStream_t s = (cudaStream_t)stream;
    if (status_out) {
        if (cudaMemsetAsync(status_out, 0, sizeof(int32_t), s) != cudaSuccess)
            return fail(kCudaError, "mpo_fps: status reset failed");
    }
    if (B == 0 || npoint == 0) return kOk;
    MPO_REQUIRE(N >= 1, "cannot sample from an empty point cloud");
    MPO_REQUIRE(start_idx >= 0 && start_idx < N, "start_idx out of range");
    MPO_REQUIRE(N < (int64_t)0x7fffffff, "N must be below 2**31");
    MPO_REQUIRE(xyz != nullptr && out != nullptr, "null pointer");
    const int skip = skip_near_origin ? 1 : 0;
    const int o32 = out_int32 ? 1 : 0;

    if (strategy != MPO_FPS_GROUP && N <= kPointsPerCta) {
        const int P = pick_p(N);
        const int threads = (int)min64(kMaxThreads, ((ceil_div(N, P) + 31) / 32) * 32);
        switch (P) {
            case 1: return launch_fps<1, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            case 2: return launch_fps<2, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            case 4: return launch_fps<4, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            default: return launch_fps<8, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
        }
    }
    if (strategy == MPO_FPS_SINGLE) {
        return fail(kUnsupported, "mpo_fps: the single-CTA strategy holds at most " +
                                      std::to_string((long long)kPointsPerCta) + " points");
    }
    const int sms = sm_count();
    // Forced group on a small cloud still uses at least two CTAs (when the
    // cloud has two points) so the cross-CTA exchange is exercised.
    int64_t G = ceil_div(N, kPointsPerCta);
    if (strategy == MPO_FPS_GROUP) G = min64(max64(G, 2), N);
    if (G > sms) {
        return fail(kUnsupported, "mpo_fps: clouds above " +
                                      std::to_string((long long)kPointsPerCta * sms) +
                                      " points are not supported on this device");
    }
    const size_t need = mpo_fps_workspace_bytes(B, N, npoint, strategy);
    if (workspace == nullptr || workspace_bytes < need) {
        return fail(kWorkspaceTooSmall, "mpo_fps: workspace must hold " + std::to_string(need) +
                                            " bytes");
    }
    if (cudaMemsetAsync(workspace, 0, need, s) != cudaSuccess)
        return fail(kCudaError, "mpo_fps: workspace reset failed");
    const int64_t per_cta = ceil_div(N, G);
    const int threads = (int)min64(kMaxThreads, ((ceil_div(per_cta, kMaxP) + 31) / 32) * 32);
    return launch_fps<8, true>(xyz, B, N, npoint, start_idx, skip, o32, out, (int)G, per_cta,
                               threads, reinterpret_cast<GroupSync*>(workspace), status_out, s);
}

}  // extern "C"

// --------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at all: a plugin that its host
// application hands nothing but input and output buffers, or a loop whose
// rules forbid any allocation once it is running.  mpo_fps_noalloc serves
// them: the cross-CTA step slots of the CTA-group path live in the
// file-scope array below instead of a caller workspace.
//   * Capacity: kNoAllocMaxClouds clouds per call on the group path
//     (32 bytes each, 32 KiB per device, held by every device that loads
//     this library until the process exits).  The one-CTA-per-cloud path
//     needs no scratch and has no such limit.
//   * In host code the array's name is only a host-side stand-in; the
//     device address is looked up once per device with cudaGetSymbolAddress
//     (device current) on the first call that needs it, so that first call
//     should happen before any stream capture begins.
//   * Every call shares the array.  It is cleared on the caller's stream at
//     the start of each call, so calls whose GPU work overlaps (different
//     streams, or different host threads) race on it and must be serialised
//     by the caller.
namespace mpo {
namespace {
constexpr int64_t kNoAllocMaxClouds = 1024;
static __device__ __align__(256) GroupSync g_fps_noalloc_scratch[kNoAllocMaxClouds];

int noalloc_scratch(GroupSync** out) {
    static std::mutex mu;
    static GroupSync* addr[64] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return fail(kUnsupported, "mpo_fps_noalloc: device index above 63");
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_fps_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return fail(kCudaError, std::string("mpo_fps_noalloc: cudaGetSymbolAddress: ") +
                                        cudaGetErrorString(e));
        }
        addr[dev] = reinterpret_cast<GroupSync*>(p);
    }
    *out = addr[dev];
    return kOk;
}
}  // namespace
}  // namespace mpo

extern "C" {

int mpo_fps_noalloc(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                    int skip_near_origin, int out_int32, int strategy, void* out,
                    int32_t* status_out, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(B >= 0 && N >= 0 && npoint >= 0, "negative size");
    MPO_REQUIRE(strategy == MPO_FPS_AUTO || strategy == MPO_FPS_SINGLE ||
                    strategy == MPO_FPS_GROUP,
                "unknown strategy");
    cudaStream_t s = (cudaStream_t)stream;
    if (status_out) {
        if (cudaMemsetAsync(status_out, 0, sizeof(int32_t), s) != cudaSuccess)
            return fail(kCudaError, "mpo_fps_noalloc: status reset failed");
    }
    if (B == 0 || npoint == 0) return kOk;
    MPO_REQUIRE(N >= 1, "cannot sample from an empty point cloud");
    MPO_REQUIRE(start_idx >= 0 && start_idx < N, "start_idx out of range");
    MPO_REQUIRE(N < (int64_t)0x7fffffff, "N must be below 2**31");
    MPO_REQUIRE(xyz != nullptr && out != nullptr, "null pointer");
    const int skip = skip_near_origin ? 1 : 0;
    const int o32 = out_int32 ? 1 : 0;
    if (strategy != MPO_FPS_GROUP && N <= kPointsPerCta) {
        const int P = pick_p(N);
        const int threads = (int)min64(kMaxThreads, ((ceil_div(N, P) + 31) / 32) * 32);
        switch (P) {
            case 1: return launch_fps<1, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            case 2: return launch_fps<2, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            case 4: return launch_fps<4, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
            default: return launch_fps<8, false>(xyz, B, N, npoint, start_idx, skip, o32, out, 1, N, threads, nullptr, status_out, s);
        }
    }
    if (strategy == MPO_FPS_SINGLE) {
        return fail(kUnsupported, "mpo_fps_noalloc: the single-CTA strategy holds at most " +
                                      std::to_string((long long)kPointsPerCta) + " points");
    }
    if (B > kNoAllocMaxClouds) {
        return fail(kInvalidArgument,
                    "mpo_fps_noalloc: the CTA-group path holds at most " +
                        std::to_string((long long)kNoAllocMaxClouds) +
                        " clouds per call in its fixed scratch; got " +
                        std::to_string((long long)B) + " (use mpo_fps with a workspace)");
    }
    const int sms = sm_count();
    int64_t G = ceil_div(N, kPointsPerCta);
    if (strategy == MPO_FPS_GROUP) G = min64(max64(G, 2), N);
    if (G > sms) {
        return fail(kUnsupported, "mpo_fps_noalloc: clouds above " +
                                      std::to_string((long long)kPointsPerCta * sms) +
                                      " points are not supported on this device");
    }
    GroupSync* scratch = nullptr;
    int st = noalloc_scratch(&scratch);
    if (st) return st;
    if (cudaMemsetAsync(scratch, 0, (size_t)B * sizeof(GroupSync), s) != cudaSuccess)
        return fail(kCudaError, "mpo_fps_noalloc: scratch reset failed");
    const int64_t per_cta = ceil_div(N, G);
    const int threads = (int)min64(kMaxThreads, ((ceil_div(per_cta, kMaxP) + 31) / 32) * 32);
    return launch_fps<8, true>(xyz, B, N, npoint, start_idx, skip, o32, out, (int)G, per_cta,
                               threads, scratch, status_out, s);
}

}  // extern "C"
