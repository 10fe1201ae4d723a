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
//   * A cloud is owned by a group of G CTAs of up to 256 threads; each thread
//     keeps P <= 32 points (x, y, z, min_d2) in registers for the whole run,
//     so a step touches no memory except the argmax exchange.  Few warps with
//     many points each keep the per-step reduction overhead small.
//   * Argmax per step: each thread scans its points (float compare on the
//     finite fast path), then a warp reduces (ordered key, index) pairs with
//     two redux.sync instructions (max key, then min index among the lanes
//     holding it), and every warp redundantly reduces the per-warp results
//     from shared memory -- one __syncthreads() per step.
//   * G == 1 (clouds up to 8192 points): the cloud's xyz is also staged in
//     shared memory so the next centroid is a shared-memory load.
//   * G > 1 (large clouds: 2^20 points on 128 SMs): a
//     cooperative launch makes the group co-resident.  Each CTA publishes its
//     best as one 64-bit word (ordered distance key << 32 | 8-bit step
//     sequence << 24 | index local to the CTA) into its slot of a
//     double-buffered slot array (buffer = step parity), and one warp of
//     every CTA polls the G slots with ld.relaxed.gpu until all carry the
//     current step's sequence, then reduces them itself -- no atomics and one
//     cross-SM round trip per step.  The poll is bounded in time
//     (kSpinLimitNs of %globaltimer); on expiry the CTA records status 1,
//     raises the group's error word and returns.
//   * Clouds above 8192 points per SM (more than 1,212,416 points on a
//     148-SM B200) use every SM; a CTA keeps its first 8192 points in
//     registers and the rest as float4 (x, y, z, min_d2) records, first in
//     shared memory (up to kSmemTierPoints, 224 KiB) and beyond that in the
//     caller's workspace (L2-resident for clouds of a few million points),
//     streamed once per step.  Any N below 2^31 is accepted.
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kMaxThreads = 256;
constexpr int kMaxP = 32;
constexpr int64_t kPointsPerCta = (int64_t)kMaxThreads * kMaxP;  // 8192
constexpr unsigned long long kSpinLimitNs = 2000000000ull;  // 2 s per step
// Step word of the group path: ordered key (32) | step sequence (8) | index
// of the point within its CTA's range (24).  The reader adds c * per_cta.
// Two steps apart differ in the sequence, which is all the double buffer
// needs; 24 local bits cover per_cta < 2^24 (every N < 2^31 on >= 128 SMs).
constexpr int kLocalBits = 24;
constexpr unsigned long long kLocalMask = (1ull << kLocalBits) - 1;
constexpr unsigned long long kSeqMask = 0xffull;
// Slots one polling lane reads: G <= 32 * kSlotsPerLane CTAs per cloud.
constexpr int kSlotsPerLane = 5;
// Overflow tier in shared memory: float4 (x, y, z, min_d2) per point.
constexpr int kSmemTierPoints = 14336;  // 224 KiB

// Cross-CTA exchange state of the clouds of one cooperative wave, in the
// caller's workspace (zeroed before each wave):
//   slots[cloud_in_wave][parity][G]  one u64 per 128-byte line, so the G
//                                    readers of a step spread over G lines
//   error[cloud_in_wave]             u32
// followed, 256-byte aligned, by the overflow tier in global memory:
//   ovf[cloud_in_wave][G][global_pts] float4 (written by the kernel itself)
constexpr int kSlotStride = 16;  // u64 words per slot (128 bytes)
inline size_t group_bytes(int64_t clouds, int64_t G) {
    return (size_t)clouds * 2 * (size_t)G * 8 * kSlotStride + (size_t)clouds * 8;
}
inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }
inline size_t group_total_bytes(int64_t clouds, int64_t G, int64_t global_pts) {
    const size_t slots = group_bytes(clouds, G);
    if (global_pts <= 0) return slots;
    return align256(slots) + (size_t)clouds * (size_t)G * (size_t)global_pts * sizeof(float4);
}

// One overflow tier of a CTA (records t[e0 .. e1) of index jbase + e), the
// thread taking e = tid, tid + nthr, ... from `e` on; min_d2 is updated in
// place (stored only when it changes) and the thread's first maximum is
// tracked as in the register tier: a float compare on the finite path, the
// NaN-ranking key otherwise.
template <bool NANM>
__device__ __forceinline__ void ovf_scan(float4* __restrict__ t, int& e, int e1, int nthr,
                                         uint32_t jbase, float cx, float cy, float cz,
                                         float& bv, uint32_t& bj, uint32_t& bkey,
                                         uint32_t& bidx) {
    for (; e < e1; e += nthr) {
        const float4 v = t[e];
        const float d = sqd3(v.x, v.y, v.z, cx, cy, cz);
        if (!NANM) {
            const float m = fminf(v.w, d);
            if (m < v.w) t[e].w = m;
            if (m > bv) {
                bv = m;
                bj = jbase + (uint32_t)e;
            }
        } else {
            const float m = fmin_nan(v.w, d);
            if (__float_as_uint(m) != __float_as_uint(v.w)) t[e].w = m;
            const uint32_t kk = isnan(m) ? 0xffffffffu : ordered_key(m);
            if (kk > bkey) {
                bkey = kk;
                bidx = jbase + (uint32_t)e;
            }
        }
    }
}

// Flat (ragged) batches of the torch_cluster API: cloud b is the rows
// [ptr[b], ptr[b+1]) of xyz, its samples go to out[out_ptr[b] .. out_ptr[b+1])
// as global row numbers, starting from the local index starts[b].
struct FlatFps {
    const int64_t* ptr;
    const int64_t* out_ptr;
    const int64_t* starts;
    int64_t total_n, total_out, max_len;
};

template <int P, bool GROUP, bool FLAT>
__global__ void __launch_bounds__(kMaxThreads, 1)
fps_kernel(const float* __restrict__ xyz, int64_t N, int64_t npoint, int64_t start_idx,
           int skip, int out_int32, void* __restrict__ out, int G, int64_t per_cta,
           int cloud_offset, unsigned long long* __restrict__ slots,
           unsigned* __restrict__ errors, int32_t* __restrict__ status, FlatFps flat,
           float* __restrict__ out_xyz, int smem_pts, float4* __restrict__ ovf_global,
           int64_t global_pts) {
    // G == 1: the cloud, 3 floats per point.  GROUP: the shared-memory
    // overflow tier, smem_pts float4 records.
    extern __shared__ __align__(16) float s_xyz[];
    __shared__ uint32_t s_key[2][32];
    __shared__ uint32_t s_idx[2][32];
    __shared__ uint32_t s_far;
    __shared__ float s_cxyz[3];
    __shared__ int s_abort;

    const int wave_cloud = blockIdx.x / G;
    const int b = cloud_offset + wave_cloud;
    const int g = blockIdx.x % G;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const int nthr = blockDim.x;
    // Rows of this cloud, its sample count and first sample, where its
    // samples go, and the value added to a local index on output.
    int64_t base = (int64_t)b * N, n = N, np = npoint, start = start_idx;
    int64_t obase = (int64_t)b * npoint, vbase = 0;
    if (FLAT) {
        base = flat.ptr[b];
        n = flat.ptr[b + 1] - base;
        obase = flat.out_ptr[b];
        np = flat.out_ptr[b + 1] - obase;
        start = flat.starts[b];
        vbase = base;
        if (np == 0) return;  // the same decision in every CTA of the cloud
        if (!(base >= 0 && n >= 1 && n <= flat.max_len && base + n <= flat.total_n &&
              obase >= 0 && np > 0 && obase + np <= flat.total_out && start >= 0 && start < n)) {
            if (tid == 0 && g == 0 && status) atomicExch(status, 2);
            return;
        }
    }
    const float* __restrict__ p = xyz + (size_t)base * 3;
    const int64_t lo = (int64_t)g * per_cta;
    const int64_t hi = min64(n, lo + per_cta);
    unsigned long long* my_slots =
        GROUP ? slots + (size_t)wave_cloud * 2 * G * kSlotStride : nullptr;
    unsigned* my_error = GROUP ? errors + wave_cloud : nullptr;

    // Points in packed pairs (slot s = 2 h + l is lane l of pair h), so one
    // f32x2 pass computes two squared distances with the same per-lane
    // rounding as sqd3.  P = 1 uses one pair with an empty second slot.
    constexpr int PP = (P + 1) / 2;
    constexpr int PS = 2 * PP;
    f32x2 PX[PP], PY[PP], PZ[PP];
    float md[PS];
#pragma unroll
    for (int h = 0; h < PP; ++h) {
        float c[6];
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            const int s = 2 * h + l;
            const int64_t j = lo + tid + (int64_t)s * nthr;
            if (s < P && j < hi) {
                c[3 * l + 0] = p[3 * j + 0];
                c[3 * l + 1] = p[3 * j + 1];
                c[3 * l + 2] = p[3 * j + 2];
                float init = INFINITY;
                if (skip && sqd3(c[3 * l], c[3 * l + 1], c[3 * l + 2], 0.f, 0.f, 0.f) < 1e-3f)
                    init = -INFINITY;
                md[s] = init;
            } else {
                c[3 * l + 0] = c[3 * l + 1] = c[3 * l + 2] = 0.f;
                md[s] = -INFINITY;
            }
        }
        PX[h] = pack2(c[0], c[3]);
        PY[h] = pack2(c[1], c[4]);
        PZ[h] = pack2(c[2], c[5]);
    }
    if (!GROUP) {
        for (int64_t e = tid; e < 3 * n; e += nthr) s_xyz[e] = p[e];
    }
    if (tid == 0) s_abort = 0;
    bool mine_nonfinite = false;
    // Overflow (GROUP, more than P * nthr points per CTA): points
    // [ob, hi) as float4 records, the first sc in shared memory, the rest in
    // this CTA's part of the global tier.
    const int64_t ob = lo + (int64_t)P * nthr;
    const int oc = GROUP ? (int)max64(0, hi - ob) : 0;
    const int sc = min(oc, smem_pts);
    float4* s_ovf = reinterpret_cast<float4*>(s_xyz);
    float4* g_ovf = (GROUP && oc > sc)
                        ? ovf_global + ((size_t)wave_cloud * G + g) * (size_t)global_pts - sc
                        : nullptr;
    for (int e = tid; e < oc; e += nthr) {
        const int64_t j = ob + e;
        const float x = p[3 * j + 0], y = p[3 * j + 1], z = p[3 * j + 2];
        mine_nonfinite |= !(isfinite(x) && isfinite(y) && isfinite(z));
        const float init = (skip && sqd3(x, y, z, 0.f, 0.f, 0.f) < 1e-3f) ? -INFINITY : INFINITY;
        const float4 v = make_float4(x, y, z, init);
        if (e < sc) s_ovf[e] = v;
        else g_ovf[e] = v;
    }
#pragma unroll
    for (int h = 0; h < PP; ++h) {
        float a0, a1, b0, b1, c0, c1;
        unpack2(PX[h], a0, a1);
        unpack2(PY[h], b0, b1);
        unpack2(PZ[h], c0, c1);
        mine_nonfinite |= !(isfinite(a0) && isfinite(b0) && isfinite(c0) && isfinite(a1) &&
                            isfinite(b1) && isfinite(c1));
    }
    bool nan_mode = __syncthreads_or(mine_nonfinite) != 0;

    uint32_t far = (uint32_t)start;
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
    int64_t* out64 = reinterpret_cast<int64_t*>(out) + (size_t)obase;
    int32_t* out32 = reinterpret_cast<int32_t*>(out) + (size_t)obase;

    for (int64_t i = 0; i < np; ++i) {
        if (tid == 0 && g == 0) {
            if (out_int32) out32[i] = (int32_t)far;
            else out64[i] = vbase + (int64_t)far;
            // Fused gather of the sample's coordinates (dense layout only).
            if (out_xyz) {
                float* o = out_xyz + ((size_t)obase + (size_t)i) * 3;
                o[0] = cx;
                o[1] = cy;
                o[2] = cz;
            }
        }
        if (i + 1 == np) break;

        // NaN can only enter min_d2 through a non-finite coordinate of this
        // CTA's points or of a centroid; from then on (sticky) the keys must
        // rank NaN above every number, like torch.argmax.
        nan_mode = nan_mode || !(isfinite(cx) && isfinite(cy) && isfinite(cz));
        uint32_t bkey = 0u, bidx = 0xffffffffu;
        if (!nan_mode) {
            // Finite fast path: min_d2 is -inf (skipped or unused slot, kept
            // there by min) or in [0, +inf]; a float compare finds the
            // thread's first maximum and the ordered key is formed once.
            float bv = -INFINITY;
            uint32_t bj = 0xffffffffu;
            const f32x2 CX = pack2(cx, cx), CY = pack2(cy, cy), CZ = pack2(cz, cz);
#pragma unroll
            for (int h = 0; h < PP; ++h) {
                float d[2];
                unpack2(sqd3x2(PX[h], PY[h], PZ[h], CX, CY, CZ), d[0], d[1]);
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    const int s = 2 * h + l;
                    if (s >= P) break;
                    md[s] = fminf(md[s], d[l]);
                    if (md[s] > bv) {
                        bv = md[s];
                        bj = (uint32_t)(lo + tid + (int64_t)s * nthr);
                    }
                }
            }
            if (GROUP && oc > 0) {
                int e = tid;
                uint32_t k0 = 0u, i0 = 0u;
                ovf_scan<false>(s_ovf, e, sc, nthr, (uint32_t)ob, cx, cy, cz, bv, bj, k0, i0);
                ovf_scan<false>(g_ovf, e, oc, nthr, (uint32_t)ob, cx, cy, cz, bv, bj, k0, i0);
            }
            // A lane whose points are all -inf offers its first valid point
            // (the lowest index among equal keys).
            if (bj == 0xffffffffu && lo + tid < hi) bj = (uint32_t)(lo + tid);
            bidx = bj;
            bkey = bj == 0xffffffffu ? 0u : ordered_key(bv);
        } else {
#pragma unroll
            for (int s = 0; s < P; ++s) {
                const int64_t j = lo + tid + (int64_t)s * nthr;
                const bool valid = j < hi;
                float x0, x1, y0, y1, z0, z1;
                unpack2(PX[s / 2], x0, x1);
                unpack2(PY[s / 2], y0, y1);
                unpack2(PZ[s / 2], z0, z1);
                const float d = (s & 1) ? sqd3(x1, y1, z1, cx, cy, cz) : sqd3(x0, y0, z0, cx, cy, cz);
                const float m = fmin_nan(md[s], d);
                md[s] = valid ? m : md[s];
                const uint32_t k = !valid ? 0u : (isnan(m) ? 0xffffffffu : ordered_key(m));
                if (k > bkey) {
                    bkey = k;
                    bidx = (uint32_t)j;
                }
            }
            if (GROUP && oc > 0) {
                int e = tid;
                float v0 = 0.f;
                uint32_t j0 = 0u;
                ovf_scan<true>(s_ovf, e, sc, nthr, (uint32_t)ob, cx, cy, cz, v0, j0, bkey, bidx);
                ovf_scan<true>(g_ovf, e, oc, nthr, (uint32_t)ob, cx, cy, cz, v0, j0, bkey, bidx);
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
            // Publish this CTA's best into slots[parity][g], then warp 0 waits
            // for all G slots of this step and reduces them.  A CTA can be at
            // most one step ahead of the slowest reader, so two buffers suffice.
            unsigned long long* cur = my_slots + (size_t)buf * G * kSlotStride;
            const unsigned long long seq = (unsigned long long)(i + 1) & kSeqMask;
            if (warp == 0) {
                if (lane == 0) {
                    const unsigned long long word =
                        ((unsigned long long)cmax << 32) | (seq << kLocalBits) |
                        ((unsigned long long)(uint32_t)(cidx - (uint32_t)lo) & kLocalMask);
                    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(cur + g * kSlotStride),
                                 "l"(word)
                                 : "memory");
                }
                // Each lane polls its slots c = lane + 32 m until every one
                // carries this step's sequence, re-reading only the slots not
                // yet seen.  When a slot is seen, the lane starts loading its
                // candidate's coordinates from the (read-only) cloud, so the
                // winner's centroid is in registers when the reduction ends
                // instead of costing another round trip after the barrier.
                uint32_t sk[kSlotsPerLane], si[kSlotsPerLane];
                float sx[kSlotsPerLane], sy[kSlotsPerLane], sz[kSlotsPerLane];
                unsigned need = 0u, seen = 0u;
#pragma unroll
                for (int m = 0; m < kSlotsPerLane; ++m) {
                    sk[m] = 0u;
                    si[m] = 0xffffffffu;
                    sx[m] = sy[m] = sz[m] = 0.f;
                    if (lane + 32 * m < G) need |= 1u << m;
                }
                // Two sets of poll results alternate: a round's loads are
                // issued before the previous round's results are examined, so
                // a slot that lands is seen about one L2 round trip later
                // instead of one and a half.
                unsigned long long va[kSlotsPerLane], vb[kSlotsPerLane];
                auto issue = [&](unsigned long long (&v)[kSlotsPerLane]) {
#pragma unroll
                    for (int m = 0; m < kSlotsPerLane; ++m)
                        v[m] = (((need & ~seen) >> m) & 1u)
                                   ? ld_relaxed_u64(cur + (lane + 32 * m) * kSlotStride)
                                   : 0ull;
                };
                auto examine = [&](const unsigned long long (&v)[kSlotsPerLane]) {
#pragma unroll
                    for (int m = 0; m < kSlotsPerLane; ++m) {
                        if ((((need & ~seen) >> m) & 1u) &&
                            ((v[m] >> kLocalBits) & kSeqMask) == seq) {
                            const int c = lane + 32 * m;
                            seen |= 1u << m;
                            sk[m] = (uint32_t)(v[m] >> 32);
                            si[m] = (uint32_t)c * (uint32_t)per_cta + (uint32_t)(v[m] & kLocalMask);
                            // A key of 0 marks a CTA without valid points
                            // (it never wins): nothing to load.
                            if (sk[m] != 0u && si[m] < (uint32_t)n) {
                                sx[m] = p[3 * (size_t)si[m] + 0];
                                sy[m] = p[3 * (size_t)si[m] + 1];
                                sz[m] = p[3 * (size_t)si[m] + 2];
                            }
                        }
                    }
                };
                const unsigned long long t0 = globaltimer_ns();
                bool abort = false;
                issue(va);
                for (unsigned round = 1;; ++round) {
                    issue(vb);
                    examine(va);
                    if (__all_sync(FULL_MASK, seen == need)) break;
                    issue(va);
                    examine(vb);
                    if (__all_sync(FULL_MASK, seen == need)) break;
                    if ((round & 31u) == 0u &&
                        (globaltimer_ns() - t0 > kSpinLimitNs || ld_acquire_u32(my_error) != 0u)) {
                        abort = true;
                        break;
                    }
                }
                abort = __any_sync(FULL_MASK, abort);
                if (abort) {
                    if (lane == 0) {
                        atomicExch(my_error, 1u);
                        if (status) atomicExch(status, 1);
                        s_abort = 1;
                    }
                } else {
                    uint32_t bk = 0u, bi = 0xffffffffu;
                    float bx = 0.f, by = 0.f, bz = 0.f;
#pragma unroll
                    for (int m = 0; m < kSlotsPerLane; ++m) {
                        if (((need >> m) & 1u) && (sk[m] > bk || (sk[m] == bk && si[m] < bi))) {
                            bk = sk[m];
                            bi = si[m];
                            bx = sx[m];
                            by = sy[m];
                            bz = sz[m];
                        }
                    }
                    const uint32_t gk = __reduce_max_sync(FULL_MASK, bk);
                    const uint32_t gi = __reduce_min_sync(FULL_MASK, bk == gk ? bi : 0xffffffffu);
                    if (bk == gk && bi == gi) {  // the one lane holding the winner
                        s_far = gi;
                        s_cxyz[0] = bx;
                        s_cxyz[1] = by;
                        s_cxyz[2] = bz;
                    }
                }
            }
            __syncthreads();
            if (s_abort) return;
            far = s_far;
            cx = s_cxyz[0];
            cy = s_cxyz[1];
            cz = s_cxyz[2];
        }
    }
}

// ---------------------------------------------------------------------------
// One CTA per cloud (clouds of up to 8192 points), the path of mpo_fps,
// mpo_fps_gather and mpo_flat_fps.  The cloud is staged in shared memory (the
// centroid load); thread t owns the contiguous points [t P, t P + P), so its
// slots are in index order and a strict > keeps its first maximum.  Per step:
// the packed distance update and the thread's argmax, two redux.sync per
// warp, one barrier, and a redundant cross-warp reduce in every warp.
// Contiguous ownership measured faster than the strided one of fps_kernel
// (8 clouds x 8192 -> 2048 samples: 1.48 -> 1.26 ms; 32 x 2048 -> 512:
// 0.178 -> 0.163 ms; 8 x 4096 -> 1024: 0.421 -> 0.416 ms).  Sorting the points by Morton code so that a thread could skip
// steps whose centroid is provably too far from its points' bounding box
// (bit-exact) was slower at every size: a step's time is dominated by the
// reduce-and-barrier chain (about 0.3 us of the 0.4 us step at 4096 points),
// which skipping does not shorten.
template <int P, bool FLAT>
__global__ void __launch_bounds__(kMaxThreads, 1)
fps_cta_kernel(const float* __restrict__ xyz, int64_t N, int64_t npoint, int64_t start_idx,
               int skip, int out_int32, void* __restrict__ out, int32_t* __restrict__ status,
               FlatFps flat, float* __restrict__ out_xyz) {
    extern __shared__ float s_xyz[];  // [3 n]
    __shared__ uint32_t s_key[2][32];
    __shared__ uint32_t s_idx[2][32];

    const int b = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5, nthr = blockDim.x;
    int64_t base = (int64_t)b * N, n = N, np = npoint, start = start_idx;
    int64_t obase = (int64_t)b * npoint, vbase = 0;
    if (FLAT) {
        base = flat.ptr[b];
        n = flat.ptr[b + 1] - base;
        obase = flat.out_ptr[b];
        np = flat.out_ptr[b + 1] - obase;
        start = flat.starts[b];
        vbase = base;
        if (np == 0) return;
        if (!(base >= 0 && n >= 1 && n <= flat.max_len && base + n <= flat.total_n &&
              obase >= 0 && np > 0 && obase + np <= flat.total_out && start >= 0 && start < n)) {
            if (tid == 0 && status) atomicExch(status, 2);
            return;
        }
    }
    const float* __restrict__ p = xyz + (size_t)base * 3;
    const int nn = (int)n;
    for (int e = tid; e < 3 * nn; e += nthr) s_xyz[e] = p[e];
    __syncthreads();

    // This thread's points: slot u -> index tid P + u (none past n).
    constexpr int PP = (P + 1) / 2;
    constexpr int PS = 2 * PP;
    uint32_t jdx[PS];
#pragma unroll
    for (int u = 0; u < PS; ++u) {
        const int j = tid * P + u;
        jdx[u] = (u < P && j < nn) ? (uint32_t)j : 0xffffffffu;
    }
    f32x2 PX[PP], PY[PP], PZ[PP];
    float md[PS];
    bool bad = false;
#pragma unroll
    for (int h = 0; h < PP; ++h) {
        float c[6];
#pragma unroll
        for (int l = 0; l < 2; ++l) {
            const int u = 2 * h + l;
            const uint32_t j = jdx[u];
            if (j != 0xffffffffu) {
                c[3 * l + 0] = s_xyz[3 * j + 0];
                c[3 * l + 1] = s_xyz[3 * j + 1];
                c[3 * l + 2] = s_xyz[3 * j + 2];
                bad |= !(isfinite(c[3 * l]) && isfinite(c[3 * l + 1]) && isfinite(c[3 * l + 2]));
                float init = INFINITY;
                if (skip && sqd3(c[3 * l], c[3 * l + 1], c[3 * l + 2], 0.f, 0.f, 0.f) < 1e-3f)
                    init = -INFINITY;
                md[u] = init;
            } else {
                c[3 * l + 0] = c[3 * l + 1] = c[3 * l + 2] = 0.f;
                md[u] = -INFINITY;
            }
        }
        PX[h] = pack2(c[0], c[3]);
        PY[h] = pack2(c[1], c[4]);
        PZ[h] = pack2(c[2], c[5]);
    }
    // NaN can only enter min_d2 through a non-finite coordinate; then (for
    // the whole run) the keys rank NaN above every number, like torch.argmax.
    const bool nan_mode = __syncthreads_or(bad) != 0;

    uint32_t far = (uint32_t)start;
    float cx = s_xyz[3 * far + 0], cy = s_xyz[3 * far + 1], cz = s_xyz[3 * far + 2];
    int64_t* out64 = reinterpret_cast<int64_t*>(out) + (size_t)obase;
    int32_t* out32 = reinterpret_cast<int32_t*>(out) + (size_t)obase;

    for (int64_t i = 0; i < np; ++i) {
        if (tid == 0) {
            if (out_int32) out32[i] = (int32_t)far;
            else out64[i] = vbase + (int64_t)far;
            if (out_xyz) {
                float* o = out_xyz + ((size_t)obase + (size_t)i) * 3;
                o[0] = cx;
                o[1] = cy;
                o[2] = cz;
            }
        }
        if (i + 1 == np) break;
        uint32_t bkey = 0u, bidx = 0xffffffffu;
        if (!nan_mode) {
            // Finite fast path: min_d2 is -inf (skipped or unused slot, kept
            // there by min) or in [0, +inf]; a float compare finds the
            // thread's first maximum and the ordered key is formed once.
            const f32x2 CX = pack2(cx, cx), CY = pack2(cy, cy), CZ = pack2(cz, cz);
            float bv = -INFINITY;
            uint32_t bj = 0xffffffffu;
#pragma unroll
            for (int h = 0; h < PP; ++h) {
                float d[2];
                unpack2(sqd3x2(PX[h], PY[h], PZ[h], CX, CY, CZ), d[0], d[1]);
#pragma unroll
                for (int l = 0; l < 2; ++l) {
                    const int u = 2 * h + l;
                    if (u >= P) break;
                    md[u] = fminf(md[u], d[l]);
                    if (md[u] > bv) {
                        bv = md[u];
                        bj = jdx[u];
                    }
                }
            }
            // A thread whose points are all -inf offers its first point (the
            // lowest index among equal keys).
            if (bj == 0xffffffffu) bj = jdx[0];
            bidx = bj;
            bkey = bj == 0xffffffffu ? 0u : ordered_key(bv);
        } else {
#pragma unroll
            for (int u = 0; u < P; ++u) {
                const uint32_t j = jdx[u];
                const bool valid = j != 0xffffffffu;
                float x0, x1, y0, y1, z0, z1;
                unpack2(PX[u / 2], x0, x1);
                unpack2(PY[u / 2], y0, y1);
                unpack2(PZ[u / 2], z0, z1);
                const float d = (u & 1) ? sqd3(x1, y1, z1, cx, cy, cz) : sqd3(x0, y0, z0, cx, cy, cz);
                const float m = fmin_nan(md[u], d);
                md[u] = valid ? m : md[u];
                const uint32_t kk = !valid ? 0u : (isnan(m) ? 0xffffffffu : ordered_key(m));
                if (kk > bkey) {
                    bkey = kk;
                    bidx = j;
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
        far = __reduce_min_sync(FULL_MASK, k2 == cmax ? i2 : 0xffffffffu);
        cx = s_xyz[3 * far + 0];
        cy = s_xyz[3 * far + 1];
        cz = s_xyz[3 * far + 2];
    }
}

// Points per thread for a CTA that owns `per_cta` points with <= 256 threads.
int pick_p(int64_t per_cta) {
    if (per_cta <= 256) return 1;
    if (per_cta <= 512) return 2;
    if (per_cta <= 1024) return 4;
    if (per_cta <= 2048) return 8;
    if (per_cta <= 4096) return 16;
    return 32;
}

int threads_for(int64_t per_cta, int P) {
    return (int)min64(kMaxThreads, ((ceil_div(per_cta, P) + 31) / 32) * 32);
}

// fps_cta_kernel launch: N is the cloud size (dense) or the longest segment
// (flat); it sets P, the CTA size and the shared-memory stage.
template <int P, bool FLAT>
int launch_cta(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
               int skip, int out_int32, void* out, int32_t* status, const FlatFps& flat,
               float* out_xyz, cudaStream_t stream) {
    auto kern = fps_cta_kernel<P, FLAT>;
    const size_t smem = (size_t)N * 3 * sizeof(float);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return fail(kCudaError, "mpo_fps: cannot set the shared-memory limit");
    kern<<<(unsigned)B, threads_for(N, P), smem, stream>>>(xyz, N, npoint, start_idx, skip,
                                                           out_int32, out, status, flat, out_xyz);
    return check_launch("mpo_fps");
}

// N is the cloud size (dense) or the longest segment (flat); it sets P, the
// CTA size and the shared-memory stage.
template <int P, bool FLAT>
int launch_single(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                  int skip, int out_int32, void* out, int32_t* status, const FlatFps& flat,
                  float* out_xyz, cudaStream_t stream) {
    auto kern = fps_kernel<P, false, FLAT>;
    const size_t smem = (size_t)N * 3 * sizeof(float);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return fail(kCudaError, "mpo_fps: cannot set the shared-memory limit");
    kern<<<(unsigned)B, threads_for(N, P), smem, stream>>>(xyz, N, npoint, start_idx, skip,
                                                           out_int32, out, 1, N, 0, nullptr,
                                                           nullptr, status, flat, out_xyz, 0,
                                                           nullptr, 0);
    return check_launch("mpo_fps");
}

// cta: take fps_cta_kernel (mpo_fps, mpo_fps_gather, mpo_flat_fps) instead of
// the one-CTA form of fps_kernel (kept for mpo_fps_noalloc).
template <bool FLAT>
int launch_single_any(const float* xyz, int64_t B, int64_t N, int64_t npoint,
                      int64_t start_idx, int skip, int o32, void* out, int32_t* status,
                      const FlatFps& f, cudaStream_t s, float* oxyz = nullptr,
                      bool cta = false) {
    if (cta) {
        switch (pick_p(N)) {
            case 1: return launch_cta<1, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
            case 2: return launch_cta<2, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
            case 4: return launch_cta<4, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
            case 8: return launch_cta<8, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
            case 16: return launch_cta<16, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
            default: return launch_cta<32, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        }
    }
    switch (pick_p(N)) {
        case 1: return launch_single<1, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        case 2: return launch_single<2, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        case 4: return launch_single<4, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        case 8: return launch_single<8, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        case 16: return launch_single<16, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
        default: return launch_single<32, FLAT>(xyz, B, N, npoint, start_idx, skip, o32, out, status, f, oxyz, s);
    }
}

// Group plan for one call: CTAs per cloud, clouds per cooperative wave, and
// the overflow tiers of a CTA owning more than kPointsPerCta points.
struct GroupPlan {
    int64_t G = 0, per_cta = 0, clouds_per_wave = 0;
    int64_t smem_pts = 0, global_pts = 0;  // per CTA
};

int plan_group(int64_t B, int64_t N, int strategy, GroupPlan* plan, const char* who) {
    const int sms = sm_count();
    if (sms < 1) return fail(kCudaError, std::string(who) + ": no SM count for this device");
    int64_t G = ceil_div(N, kPointsPerCta);
    // A forced group on a small cloud still uses at least two CTAs (when the
    // cloud has two points) so the cross-CTA exchange is exercised.
    if (strategy == MPO_FPS_GROUP) G = min64(max64(G, 2), N);
    // Above 8192 points per SM every SM takes part and the CTAs' extra points
    // go to the overflow tiers.
    G = min64(G, min64(sms, 32 * kSlotsPerLane));
    const int64_t per_cta = ceil_div(N, G);
    if (per_cta > (int64_t)kLocalMask) {
        return fail(kUnsupported, std::string(who) + ": clouds above " +
                                      std::to_string((long long)kLocalMask * G) +
                                      " points are not supported on this device");
    }
    const int64_t over = max64(0, per_cta - kPointsPerCta);
    plan->G = G;
    plan->per_cta = per_cta;
    plan->clouds_per_wave = min64(B, sms / G);
    plan->smem_pts = min64(over, kSmemTierPoints);
    plan->global_pts = over - plan->smem_pts;
    return kOk;
}

inline size_t plan_bytes(const GroupPlan& plan) {
    return group_total_bytes(plan.clouds_per_wave, plan.G, plan.global_pts);
}

// Runs the group path in cooperative waves; `scratch` holds group_bytes()
// for one wave and is zeroed on the stream before each wave.
template <bool FLAT>
int launch_group(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                 int skip, int out_int32, void* out, const GroupPlan& plan, void* scratch,
                 int32_t* status, const FlatFps& flat_in, cudaStream_t stream, const char* who,
                 float* out_xyz = nullptr) {
    auto kern = fps_kernel<kMaxP, true, FLAT>;
    FlatFps flat = flat_in;
    int G = (int)plan.G;
    int64_t per_cta = plan.per_cta;
    const int threads = threads_for(per_cta, kMaxP);
    unsigned long long* slots = reinterpret_cast<unsigned long long*>(scratch);
    unsigned* errors =
        reinterpret_cast<unsigned*>(slots + (size_t)plan.clouds_per_wave * 2 * G * kSlotStride);
    const size_t bytes = group_bytes(plan.clouds_per_wave, G);
    int smem_pts = (int)plan.smem_pts;
    int64_t global_pts = plan.global_pts;
    float4* ovf_global =
        global_pts > 0
            ? reinterpret_cast<float4*>(static_cast<unsigned char*>(scratch) + align256(bytes))
            : nullptr;
    const size_t smem = (size_t)smem_pts * sizeof(float4);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return fail(kCudaError, std::string(who) + ": cannot set the shared-memory limit");
    for (int64_t c0 = 0; c0 < B; c0 += plan.clouds_per_wave) {
        const int nc = (int)min64(plan.clouds_per_wave, B - c0);
        if (cudaMemsetAsync(scratch, 0, bytes, stream) != cudaSuccess)
            return fail(kCudaError, std::string(who) + ": scratch reset failed");
        int cloud_offset = (int)c0;
        void* args[] = {(void*)&xyz,      (void*)&N,         (void*)&npoint, (void*)&start_idx,
                        (void*)&skip,     (void*)&out_int32, (void*)&out,    (void*)&G,
                        (void*)&per_cta,  (void*)&cloud_offset, (void*)&slots, (void*)&errors,
                        (void*)&status,   (void*)&flat,      (void*)&out_xyz,
                        (void*)&smem_pts, (void*)&ovf_global, (void*)&global_pts};
        cudaError_t e = cudaLaunchCooperativeKernel((const void*)kern, dim3(nc * G),
                                                    dim3(threads), args, smem, stream);
        if (e != cudaSuccess) {
            return fail(kCudaError, std::string(who) + ": cooperative launch: " +
                                        cudaGetErrorString(e));
        }
        count_launches(1);
    }
    return kOk;
}

int check_fps_args(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                   int strategy, void* out, int32_t* status_out, cudaStream_t s,
                   const char* who, bool* nothing_to_do) {
    const std::string w(who);
    *nothing_to_do = false;
    if (!(B >= 0 && N >= 0 && npoint >= 0)) return fail(kInvalidArgument, w + ": negative size");
    if (!(strategy == MPO_FPS_AUTO || strategy == MPO_FPS_SINGLE || strategy == MPO_FPS_GROUP))
        return fail(kInvalidArgument, w + ": unknown strategy");
    if (status_out) {
        if (cudaMemsetAsync(status_out, 0, sizeof(int32_t), s) != cudaSuccess)
            return fail(kCudaError, w + ": status reset failed");
    }
    if (B == 0 || npoint == 0) {
        *nothing_to_do = true;
        return kOk;
    }
    if (N < 1) return fail(kInvalidArgument, w + ": cannot sample from an empty point cloud");
    if (!(start_idx >= 0 && start_idx < N))
        return fail(kInvalidArgument, w + ": start_idx out of range");
    if (N >= (int64_t)0x7fffffff) return fail(kInvalidArgument, w + ": N must be below 2**31");
    if (xyz == nullptr || out == nullptr) return fail(kInvalidArgument, w + ": null pointer");
    if (strategy == MPO_FPS_SINGLE && N > kPointsPerCta) {
        return fail(kUnsupported, w + ": the single-CTA strategy holds at most " +
                                      std::to_string((long long)kPointsPerCta) + " points");
    }
    return kOk;
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_fps_workspace_bytes(int64_t B, int64_t N, int64_t npoint, int strategy) {
    (void)npoint;
    if (B <= 0 || N <= 0 || (strategy != MPO_FPS_GROUP && N <= mpo::kPointsPerCta)) return 0;
    mpo::GroupPlan plan;
    if (mpo::plan_group(B, N, strategy, &plan, "mpo_fps_workspace_bytes") != mpo::kOk) return 0;
    return mpo::plan_bytes(plan);
}

int mpo_fps(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
            int skip_near_origin, int out_int32, int strategy, void* out, int32_t* status_out,
            void* workspace, size_t workspace_bytes, void* stream) {
    return mpo_fps_gather(xyz, B, N, npoint, start_idx, skip_near_origin, out_int32, strategy,
                          out, nullptr, status_out, workspace, workspace_bytes, stream);
}

int mpo_fps_gather(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                   int skip_near_origin, int out_int32, int strategy, void* out, float* out_xyz,
                   int32_t* status_out, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE_WORKSPACE(workspace);
    cudaStream_t s = (cudaStream_t)stream;
    bool done = false;
    int st = check_fps_args(xyz, B, N, npoint, start_idx, strategy, out, status_out, s, "mpo_fps",
                            &done);
    if (st || done) return st;
    const int skip = skip_near_origin ? 1 : 0;
    const int o32 = out_int32 ? 1 : 0;
    if (strategy != MPO_FPS_GROUP && N <= kPointsPerCta)
        return launch_single_any<false>(xyz, B, N, npoint, start_idx, skip, o32, out, status_out,
                                        FlatFps{}, s, out_xyz, /*cta=*/true);
    GroupPlan plan;
    st = plan_group(B, N, strategy, &plan, "mpo_fps");
    if (st) return st;
    const size_t need = plan_bytes(plan);
    if (workspace == nullptr || workspace_bytes < need) {
        return fail(kWorkspaceTooSmall, "mpo_fps: workspace must hold " + std::to_string(need) +
                                            " bytes");
    }
    return launch_group<false>(xyz, B, N, npoint, start_idx, skip, o32, out, plan, workspace,
                               status_out, FlatFps{}, s, "mpo_fps", out_xyz);
}

size_t mpo_flat_fps_workspace_bytes(int64_t segments, int64_t max_len) {
    if (segments <= 0 || max_len <= mpo::kPointsPerCta) return 0;
    mpo::GroupPlan plan;
    if (mpo::plan_group(segments, max_len, MPO_FPS_AUTO, &plan, "mpo_flat_fps_workspace_bytes") !=
        mpo::kOk)
        return 0;
    return mpo::plan_bytes(plan);
}

int mpo_flat_fps(const float* x, const int64_t* ptr, const int64_t* out_ptr,
                 const int64_t* starts, int64_t segments, int64_t total_n, int64_t total_out,
                 int64_t max_len, int64_t* out, int32_t* status, void* workspace,
                 size_t workspace_bytes, void* stream) {
    using namespace mpo;
    MPO_REQUIRE(segments >= 0 && total_n >= 0 && total_out >= 0 && max_len >= 0,
                "negative size");
    MPO_REQUIRE(status != nullptr, "status must not be null");
    MPO_REQUIRE_WORKSPACE(workspace);
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(status, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(kCudaError, "mpo_flat_fps: status reset failed");
    if (segments == 0 || total_out == 0) return kOk;
    MPO_REQUIRE(max_len >= 1 && max_len <= total_n, "max_len must be in [1, total_n]");
    MPO_REQUIRE(max_len < (int64_t)0x7fffffff, "segments must be below 2**31 points");
    MPO_REQUIRE(x && ptr && out_ptr && starts && out, "null pointer");
    const FlatFps flat{ptr, out_ptr, starts, total_n, total_out, max_len};
    if (max_len <= kPointsPerCta)
        return launch_single_any<true>(x, segments, max_len, 0, 0, 0, 0, out, status, flat, s,
                                       nullptr, /*cta=*/true);
    GroupPlan plan;
    int st = plan_group(segments, max_len, MPO_FPS_AUTO, &plan, "mpo_flat_fps");
    if (st) return st;
    const size_t need = plan_bytes(plan);
    if (workspace == nullptr || workspace_bytes < need) {
        return fail(kWorkspaceTooSmall, "mpo_flat_fps: workspace must hold " +
                                            std::to_string(need) + " bytes");
    }
    return launch_group<true>(x, segments, max_len, 0, 0, 0, 0, out, plan, workspace, status,
                              flat, s, "mpo_flat_fps");
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
//   * Capacity: kNoAllocScratchBytes (40 KiB per device, held by every device
//     that loads this library until the process exits).  The group path
//     needs 256 bytes per CTA of one cooperative wave plus 8 per cloud (under
//     38 KiB on a 148-SM B200) whatever the batch size, because waves reuse
//     the slots; a configuration needing more is rejected, and so is a cloud
//     too large for registers plus shared memory (above 22,528 points per SM,
//     3,334,144 on a 148-SM B200), whose extra points would need workspace.
//     The one-CTA-per-cloud path needs no scratch.
//   * In host code the array's name is only a host-side stand-in; the
//     device address is looked up with cudaGetSymbolAddress (device current)
//     on the first call that needs it on a device, so that first call should
//     happen before any stream capture begins.  The address is cached with
//     the ID of the CUDA context it belongs to; a call in a newer context of
//     the device (after cudaDeviceReset) looks it up again.
//   * Every call shares the array.  It is cleared on the caller's stream
//     before each wave, so calls whose GPU work overlaps (different streams,
//     or different host threads) race on it and must be serialised by the
//     caller.
namespace mpo {
namespace {
constexpr size_t kNoAllocScratchBytes = 40960;
static __device__ __align__(256) unsigned char g_fps_noalloc_scratch[kNoAllocScratchBytes];

// Unique ID of the calling thread's current CUDA context (IDs are never
// reused within a process), through the driver entry points the runtime
// exposes; 0 if unavailable.
unsigned long long current_context_id() {
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != 0 || ctx == nullptr ||
        get_id(ctx, &id) != 0)
        return 0;
    return id;
}

int noalloc_scratch(void** out) {
    struct Entry {
        unsigned long long ctx = 0;
        void* addr = nullptr;
    };
    static std::mutex mu;
    static std::map<int, Entry> cache;
    const int dev = current_device();
    if (dev < 0) return fail(kCudaError, "mpo_fps_noalloc: no current device");
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    Entry& e = cache[dev];
    if (e.addr == nullptr || e.ctx != ctx || ctx == 0) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_fps_noalloc_scratch);
        if (err != cudaSuccess || p == nullptr) {
            e = Entry{};
            return fail(kCudaError, std::string("mpo_fps_noalloc: cudaGetSymbolAddress: ") +
                                        cudaGetErrorString(err));
        }
        e.addr = p;
        e.ctx = ctx;
    }
    *out = e.addr;
    return kOk;
}
}  // namespace
}  // namespace mpo

extern "C" {

int mpo_fps_noalloc(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                    int skip_near_origin, int out_int32, int strategy, void* out,
                    int32_t* status_out, void* stream) {
    using namespace mpo;
    cudaStream_t s = (cudaStream_t)stream;
    bool done = false;
    int st = check_fps_args(xyz, B, N, npoint, start_idx, strategy, out, status_out, s,
                            "mpo_fps_noalloc", &done);
    if (st || done) return st;
    const int skip = skip_near_origin ? 1 : 0;
    const int o32 = out_int32 ? 1 : 0;
    if (strategy != MPO_FPS_GROUP && N <= kPointsPerCta)
        return launch_single_any<false>(xyz, B, N, npoint, start_idx, skip, o32, out, status_out,
                                        FlatFps{}, s);
    GroupPlan plan;
    st = plan_group(B, N, strategy, &plan, "mpo_fps_noalloc");
    if (st) return st;
    if (plan.global_pts > 0) {
        return fail(kInvalidArgument,
                    "mpo_fps_noalloc: clouds above " +
                        std::to_string((long long)(kPointsPerCta + kSmemTierPoints) * plan.G) +
                        " points need workspace (use mpo_fps with a workspace)");
    }
    const size_t need = group_bytes(plan.clouds_per_wave, plan.G);
    if (need > kNoAllocScratchBytes) {
        return fail(kInvalidArgument,
                    "mpo_fps_noalloc: this launch needs " + std::to_string(need) +
                        " bytes of exchange scratch, above the fixed " +
                        std::to_string(kNoAllocScratchBytes) +
                        " bytes (use mpo_fps with a workspace)");
    }
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st) return st;
    return launch_group<false>(xyz, B, N, npoint, start_idx, skip, o32, out, plan, scratch,
                               status_out, FlatFps{}, s, "mpo_fps_noalloc");
}

}  // extern "C"
