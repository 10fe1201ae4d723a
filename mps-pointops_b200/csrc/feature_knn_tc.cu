// Feature-space kNN (D != 3) on the 5th-generation tensor cores of sm_100a,
// with an exact fp32 re-rank.
//
// Contract: gamzerA/mps-pointops mps_pointops/ops.py:144-205 with the exact
// order of tests/test_feature_knn.py:16-35 and docs/feature-knn.md:16-47: for
// every query the k references with the smallest (SD, index), where SD is the
// sequential fp32 sum s = d0*d0; s = s + dt*dt (d = q - r, every op rounded),
// non-finite SD discarded, unfilled slots (inf, -1), Euclidean distance =
// sqrt(SD) taken after selection.
//
// The tensor cores only PROPOSE candidates; every reported distance and every
// ranking decision comes from the exact fp32 SD.  Design:
//
//  1. Norms (fknn_norms_kernel): n(p) = sum of p_t^2 in fp32 for queries and
//     references; per cloud the largest reference norm and a flag for
//     non-finite or huge norms (such clouds skip the tensor path).
//  2. Approximate scores on tcgen05 (fknn_tc_kernel): for a CTA's 128 queries
//     and a 256-reference tile, dot(q, r) comes from kind::f16 MMAs with bf16
//     operands split as p = hi + lo (hi = bf16(p), lo = bf16(p - hi)):
//     dot ~= hi.hi' + hi.lo' + lo.hi' accumulated in fp32 in tensor memory
//     (TMEM, 128 lanes x 256 columns).  The epilogue thread of a query row
//     reads its accumulator row with tcgen05.ld and forms the score
//     s_j = n(r_j) - 2 dot'_j, so SD'_j = n(q) + s_j approximates SD_j with
//     |SD'_j - SD_j| <= eps(q) = C_K (n(q) + max_j n(r_j)) (bound below).
//       pass 1: the minimum of s over each group of 32 consecutive columns;
//               the k-th smallest group minimum U is an upper bound on the
//               k-th smallest s (k groups -> k distinct columns).
//       pass 2: every column with s_j <= U + 2 eps(q) is appended to the
//               query's candidate list (capacity kCap).
//     The k nearest by exact SD are all candidates: F_k <= n(q) + U + eps
//     (k columns have SD' <= n(q) + U), and a needed column has
//     SD' <= F_k + eps.
//  3. Exact re-rank (fknn_rerank_kernel): exact fp32 SD of every candidate,
//     sorted by (SD, index).  A query whose list overflowed, or whose cloud
//     was flagged, is scanned exactly over all references instead.
//
// Error bound C_K (per unit of n(q) + n(r), K = D padded to 16): the dropped
// lo.lo' term and the residual of lo are each below 2^-16 |q_t||r_t|; fp32
// accumulation inside the tensor core, the norms, the score FMA and the
// reference's own rounding add the rest.  C_K = 2 * (2^-13 + 3K 2^-21 +
// (3D + 16) 2^-24) is about twice the sum of those terms.
//
// Work per (query tile, reference tile): 3 * 2 * 128 * 256 * K flops on the
// tensor pipe; the synchronous loop below (stage tile -> MMA -> epilogue)
// relies on two resident CTAs per SM to overlap the phases.
#include <cuda_bf16.h>

#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"
#include "knn_select.cuh"

namespace mpo {
namespace {

constexpr int kTM = 128;          // queries per CTA (TMEM lanes)
constexpr int kTN = 256;          // references per tile (TMEM columns)
constexpr int kKC = 64;           // features per staged K chunk
constexpr int kThreadsTC = 256;   // 8 warps: 2 per TMEM lane quarter
constexpr int kCap = 64;          // candidates kept per query
constexpr int kMaxK = 32;         // largest k served by this path
constexpr unsigned long long kWaitNs = 2000000000ull;

// Shared-memory layout (bytes), K-major core-matrix ("interleaved", no
// swizzle) layout for both operands: element (row, t) of a 64-feature chunk
// sits at (row / 8) * kSBO + (t / 8) * 128 + (row % 8) * 16 + (t % 8) * 2.
constexpr int kSBO = (kKC / 8) * 128;                  // 1024 B per 8-row group
constexpr int kABytes = kTM * kKC * 2;                 // 16 KB per bf16 part
constexpr int kBBytes = kTN * kKC * 2;                 // 32 KB per bf16 part
constexpr int kOffAhi = 0;
constexpr int kOffAlo = kOffAhi + kABytes;
constexpr int kOffBhi = kOffAlo + kABytes;
constexpr int kOffBlo = kOffBhi + kBBytes;
constexpr int kOffNy = kOffBlo + kBBytes;              // float[kTN]
constexpr int kOffCount = kOffNy + kTN * 4;            // u32[kTM] (pass 2)
// Pass 1 merges the two column halves' lists in the (then idle) B region.
static_assert(2 * kTM * kMaxK * 4 <= 2 * kBBytes, "merge buffer must fit");
constexpr int kOffMisc = kOffCount + kTM * 4;          // mbarrier (8) + tmem slot (4)
constexpr int kSmemTC = kOffMisc + 64;
// 2 CTAs per SM fit (TMEM: 2 x 256 columns = all 512).
static_assert(2 * kSmemTC <= 227 * 1024, "two CTAs per SM must fit");

// ---- PTX wrappers (tcgen05, mbarrier, proxies) ---------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false if the barrier did not complete within kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitNs) return false;
    }
    return true;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// Shared-memory matrix descriptor: K-major, no swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor: kind::f16, A = B = bf16 (K-major), D = f32, M = 128,
// N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t bf16_bits(float x) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}
// hi/lo split of 8 floats into two 16-byte rows of 8 bf16.
__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& lo) {
    uint32_t h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        h[i] = bf16_bits(x[i]);
        const float hf = __uint_as_float(h[i] << 16);
        l[i] = bf16_bits(__fsub_rn(x[i], hf));
    }
    hi = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    lo = make_uint4(l[0] | (l[1] << 16), l[2] | (l[3] << 16), l[4] | (l[5] << 16), l[6] | (l[7] << 16));
}

// Stage rows [row0, row0 + rows) x features [t0, t0 + kKC) of a (n, D) fp32
// matrix as hi/lo bf16 in the core-matrix layout; rows >= n and features
// >= D are zero.
__device__ __forceinline__ void stage_rows(const float* __restrict__ p, int64_t n, int D,
                                           int64_t row0, int rows, int t0, unsigned char* hi_base,
                                           unsigned char* lo_base, int tid, int nthreads) {
    const int chunks = rows * (kKC / 8);
    for (int c = tid; c < chunks; c += nthreads) {
        const int row = c / (kKC / 8);
        const int kc = c % (kKC / 8);
        const int64_t gr = row0 + row;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int t = t0 + kc * 8 + i;
            x[i] = (gr < n && t < D) ? p[gr * D + t] : 0.f;
        }
        uint4 h, l;
        split8(x, h, l);
        const int off = (row >> 3) * kSBO + kc * 128 + (row & 7) * 16;
        *reinterpret_cast<uint4*>(hi_base + off) = h;
        *reinterpret_cast<uint4*>(lo_base + off) = l;
    }
}

__device__ __forceinline__ float eps_coef(int D) {
    const int K = (D + 15) / 16 * 16;
    return 2.f * (1.220703125e-4f /* 2^-13 */ + 3.f * (float)K * 4.76837158203125e-7f /* 2^-21 */ +
                  (3.f * (float)D + 16.f) * 5.9604644775390625e-8f /* 2^-24 */);
}

// ---- 1. norms ---------------------------------------------------------------
// One warp per point; nmax = largest reference norm (bit order of non-negative
// floats), bad = some norm is not finite or above 2^100 (scores could lose
// all precision), which sends the cloud to the exact path.
__global__ void fknn_norms_kernel(const float* __restrict__ q, const float* __restrict__ r,
                                  int64_t B, int64_t M, int64_t N, int D, float* __restrict__ nq,
                                  float* __restrict__ nr, unsigned* __restrict__ nmax,
                                  int* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t total = B * (M + N);
    if (w >= total) return;
    const bool is_q = w < B * M;
    const int64_t row = is_q ? w : w - B * M;
    const float* p = (is_q ? q : r) + row * D;
    float s = 0.f;
    for (int t = lane; t < D; t += 32) s = __fadd_rn(s, __fmul_rn(p[t], p[t]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(FULL_MASK, s, o));
    if (lane != 0) return;
    const int64_t b = is_q ? row / M : row / N;
    const bool ok = isfinite(s) && s <= 1.2676506e30f;  // 2^100
    if (!ok) bad[b] = 1;
    if (is_q) {
        nq[row] = s;
    } else {
        nr[row] = s;
        if (ok) atomicMax(&nmax[b], __float_as_uint(s));
    }
}

// ---- 2. approximate scores on the tensor cores ------------------------------
// KCAP >= k: capacity of the pass-1 list of group minima, right-aligned so
// that the k-th smallest sits in the static slot KCAP - 1 (leading slots hold
// -inf sentinels).
template <int PASS, int KCAP>
__global__ void __launch_bounds__(kThreadsTC, 1)
fknn_tc_kernel(const float* __restrict__ q, const float* __restrict__ r, int64_t M, int64_t N,
               int D, int k, const float* __restrict__ nq, const float* __restrict__ nr,
               const unsigned* __restrict__ nmax, const int* __restrict__ bad,
               float* __restrict__ ubound, unsigned* __restrict__ counts, uint2* __restrict__ cand,
               int* __restrict__ status) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.y;
    const int64_t m0 = (int64_t)blockIdx.x * kTM;
    if (bad[b]) return;  // uniform: the cloud goes to the exact path

    float* s_ny = reinterpret_cast<float*>(smem + kOffNy);
    float* s_list = reinterpret_cast<float*>(smem + kOffBhi);  // pass 1, after the loop
    unsigned* s_count = reinterpret_cast<unsigned*>(smem + kOffCount);
    const uint32_t bar = smem_u32(smem + kOffMisc);
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kOffMisc + 8);
    const float* qb = q + (int64_t)b * M * D;
    const float* rb = r + (int64_t)b * N * D;

    if (warp == 0) tmem_alloc(smem_u32(s_tmem), kTN);
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    if (PASS == 2 && tid < kTM) s_count[tid] = 0u;

    // This thread's query row and column half.
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;
    const int64_t gq = m0 + row;
    const bool qvalid = gq < M;
    const float nqi = qvalid ? nq[(int64_t)b * M + gq] : 0.f;
    const float eps = eps_coef(D) * (nqi + __uint_as_float(nmax[b]));
    float thr = -INFINITY;  // pass 2: s_j <= thr makes j a candidate
    if (PASS == 2 && qvalid) thr = ubound[(int64_t)b * M + gq] + 2.f * eps;
    // Pass 1: the k smallest group minima of this thread's columns, sorted.
    float lst[KCAP];
#pragma unroll
    for (int i = 0; i < KCAP; ++i) lst[i] = i < KCAP - k ? -INFINITY : INFINITY;

    const int nkc = (D + kKC - 1) / kKC;
    const bool a_resident = nkc == 1;
    if (a_resident)
        stage_rows(qb, M, D, m0, kTM, 0, smem + kOffAhi, smem + kOffAlo, tid, kThreadsTC);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    uint32_t phase = 0;
    bool ok = true;

    for (int64_t n0 = 0; n0 < N && ok; n0 += kTN) {
        for (int kc = 0; kc < nkc && ok; ++kc) {
            if (!a_resident)
                stage_rows(qb, M, D, m0, kTM, kc * kKC, smem + kOffAhi, smem + kOffAlo, tid,
                           kThreadsTC);
            stage_rows(rb, N, D, n0, kTN, kc * kKC, smem + kOffBhi, smem + kOffBlo, tid,
                       kThreadsTC);
            if (kc == 0) {
                for (int j = tid; j < kTN; j += kThreadsTC)
                    s_ny[j] = (n0 + j < N) ? nr[(int64_t)b * N + n0 + j] : INFINITY;
            }
            fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const int ksteps = min(kKC, ((D - kc * kKC) + 15) / 16 * 16) / 16;
                for (int s = 0; s < ksteps; ++s) {
                    const uint32_t koff = (uint32_t)s * 256u;
                    const uint64_t ahi = smem_desc(smem_u32(smem + kOffAhi) + koff, 128, kSBO);
                    const uint64_t alo = smem_desc(smem_u32(smem + kOffAlo) + koff, 128, kSBO);
                    const uint64_t bhi = smem_desc(smem_u32(smem + kOffBhi) + koff, 128, kSBO);
                    const uint64_t blo = smem_desc(smem_u32(smem + kOffBlo) + koff, 128, kSBO);
                    const uint32_t first = (kc == 0 && s == 0) ? 0u : 1u;
                    mma_bf16(tmem, ahi, bhi, first);
                    mma_bf16(tmem, ahi, blo, 1u);
                    mma_bf16(tmem, alo, bhi, 1u);
                }
                mma_commit(bar);
            }
            const bool done = mbar_wait(bar, phase);
            ok = __syncthreads_and(done) != 0;  // every thread takes the same path
            if (!ok && tid == 0) atomicExch(status, 1);
            phase ^= 1u;
            tc_fence_after();
        }
        if (!ok) break;
        // Epilogue: this thread's row, columns [half * 128, half * 128 + 128).
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            const int col0 = half * 128 + c * 32;
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0, v);
            if (PASS == 1) {
                float g = INFINITY;
#pragma unroll
                for (int i = 0; i < 32; ++i) g = fminf(g, fmaf(-2.f, v[i], s_ny[col0 + i]));
                if (g < lst[KCAP - 1]) {
                    // Insert g, dropping the largest; sentinels never move.
#pragma unroll
                    for (int i = KCAP - 1; i >= 1; --i) {
                        const float lo = lst[i - 1];
                        lst[i] = (g < lo) ? lo : ((g < lst[i]) ? g : lst[i]);
                    }
                    lst[0] = fminf(lst[0], g);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float sj = fmaf(-2.f, v[i], s_ny[col0 + i]);
                    if (sj <= thr) {
                        const unsigned slot = atomicAdd(&s_count[row], 1u);
                        if (slot < (unsigned)kCap && qvalid)
                            cand[((int64_t)b * M + gq) * kCap + slot] =
                                make_uint2((unsigned)(n0 + col0 + i), __float_as_uint(sj));
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();  // TMEM and the B tile are free again
    }

    if (PASS == 1) {
        // k-th smallest group minimum over both halves of the row: each half
        // writes its k entries, half 0 merges.
        __syncthreads();  // the B region is idle now
#pragma unroll
        for (int i = 0; i < KCAP; ++i)
            if (i >= KCAP - k) s_list[(half * kTM + row) * kMaxK + (i - (KCAP - k))] = lst[i];
        __syncthreads();
        if (half == 0 && qvalid) {
            const float* la = s_list + row * kMaxK;
            const float* lb = s_list + (kTM + row) * kMaxK;
            int ia = 0, ib = 0;
            float kth = INFINITY;
            for (int t = 0; t < k; ++t) {
                const float a = la[ia], bb = lb[ib];
                if (a <= bb) {
                    kth = a;
                    ++ia;
                } else {
                    kth = bb;
                    ++ib;
                }
            }
            ubound[(int64_t)b * M + gq] = ok ? kth : INFINITY;
        }
    } else {
        __syncthreads();
        if (half == 0 && qvalid) counts[(int64_t)b * M + gq] = ok ? s_count[row] : 0xffffffffu;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTN);
    }
}

// ---- 3. exact re-rank --------------------------------------------------------
// Thread per query: the exact sequential-fp32 SD of every candidate (or of
// every reference when the candidate list overflowed or the cloud was
// flagged), selected in (SD, index) order with non-finite SD dropped.
template <int KCAP>
__global__ void __launch_bounds__(128)
fknn_rerank_kernel(const float* __restrict__ q, const float* __restrict__ r, int64_t B, int64_t M,
                   int64_t N, int D, int k, const int* __restrict__ bad,
                   const unsigned* __restrict__ counts, const uint2* __restrict__ cand,
                   float* __restrict__ dist, int64_t* __restrict__ idx64,
                   float* __restrict__ sqdist) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= B * M) return;
    const int64_t b = row / M;
    const float* qp = q + row * D;
    const float* rb = r + b * N * D;
    TopK<KCAP, kDropNonFinite> top;
    top.init(k);
    const unsigned cnt = bad[b] ? 0xffffffffu : counts[row];
    if (cnt > (unsigned)kCap) {
        for (int64_t j = 0; j < N; ++j) top.offer(sqd_seq(qp, rb + j * D, D), (uint32_t)j);
    } else {
        for (unsigned c = 0; c < cnt; ++c) {
            const uint32_t j = cand[row * kCap + c].x;
            top.offer(sqd_seq(qp, rb + (int64_t)j * D, D), j);
        }
    }
    const int64_t o = row * k;
#pragma unroll
    for (int s = 0; s < KCAP; ++s) {
        const int l = s - top.base;
        if (l >= 0) {
            const bool filled = l < top.cnt;
            const float d = filled ? top.d[s] : INFINITY;
            dist[o + l] = sqrtf(d);
            if (sqdist) sqdist[o + l] = d;
            idx64[o + l] = filled ? (int64_t)top.i[s] : -1;
        }
    }
}

struct Scratch {
    float* nq;
    float* nr;
    float* ubound;
    unsigned* counts;
    uint2* cand;
    unsigned* nmax;
    int* bad;
    int* status;
    size_t bytes;
};

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

inline Scratch carve(void* base, int64_t B, int64_t M, int64_t N) {
    Scratch s{};
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t at = off;
        off += align256(n);
        return base ? static_cast<unsigned char*>(base) + at : nullptr;
    };
    s.nq = reinterpret_cast<float*>(take(sizeof(float) * B * M));
    s.nr = reinterpret_cast<float*>(take(sizeof(float) * B * N));
    s.ubound = reinterpret_cast<float*>(take(sizeof(float) * B * M));
    s.counts = reinterpret_cast<unsigned*>(take(sizeof(unsigned) * B * M));
    s.cand = reinterpret_cast<uint2*>(take(sizeof(uint2) * B * M * kCap));
    // nmax, bad and status are contiguous so one memset clears them.
    unsigned char* flags = take(sizeof(unsigned) * B + sizeof(int) * B + sizeof(int));
    s.nmax = reinterpret_cast<unsigned*>(flags);
    s.bad = flags ? reinterpret_cast<int*>(flags + sizeof(unsigned) * B) : nullptr;
    s.status = flags ? reinterpret_cast<int*>(flags + (sizeof(unsigned) + sizeof(int)) * B) : nullptr;
    s.bytes = off;
    return s;
}

template <int KCAP>
int run_tc(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int D, int k,
           float* dist, int64_t* idx, float* sqdist, const Scratch& w, cudaStream_t s) {
    if (cudaMemsetAsync(w.nmax, 0, sizeof(unsigned) * B + sizeof(int) * B + sizeof(int), s) !=
        cudaSuccess)
        return fail(kCudaError, "knn: scratch reset failed");
    const int64_t warps = B * (M + N);
    fknn_norms_kernel<<<(unsigned)ceil_div(warps * 32, 256), 256, 0, s>>>(
        query, ref, B, M, N, D, w.nq, w.nr, w.nmax, w.bad);
    int st = check_launch("fknn_norms_kernel");
    if (st) return st;
    auto k1 = fknn_tc_kernel<1, KCAP>;
    auto k2 = fknn_tc_kernel<2, KCAP>;
    if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTC) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTC) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    dim3 grid((unsigned)ceil_div(M, kTM), (unsigned)B);
    k1<<<grid, kThreadsTC, kSmemTC, s>>>(query, ref, M, N, D, k, w.nq, w.nr, w.nmax, w.bad,
                                         w.ubound, w.counts, w.cand, w.status);
    st = check_launch("fknn_tc_kernel<1>");
    if (st) return st;
    k2<<<grid, kThreadsTC, kSmemTC, s>>>(query, ref, M, N, D, k, w.nq, w.nr, w.nmax, w.bad,
                                         w.ubound, w.counts, w.cand, w.status);
    st = check_launch("fknn_tc_kernel<2>");
    if (st) return st;
    fknn_rerank_kernel<KCAP><<<(unsigned)ceil_div(B * M, 128), 128, 0, s>>>(
        query, ref, B, M, N, D, k, w.bad, w.counts, w.cand, dist, idx, sqdist);
    return check_launch("fknn_rerank_kernel");
}

}  // namespace

// The tensor path serves D != 3 with 16 <= D <= 1024, k <= 32 and reference
// clouds of at least 2048 points (smaller problems are cheap exactly).
bool fknn_tc_eligible(int64_t M, int64_t N, int64_t D, int64_t k) {
    return D != 3 && D >= 16 && D <= 1024 && k >= 1 && k <= kMaxK && N >= 2048 && M >= 1 &&
           N <= 0x7fffffffLL;
}

size_t fknn_tc_workspace_bytes(int64_t B, int64_t M, int64_t N) {
    return carve(nullptr, B, M, N).bytes;
}

int fknn_tc_run(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int64_t D,
                int64_t k, float* dist, int64_t* idx, float* sqdist, void* workspace,
                size_t workspace_bytes, cudaStream_t s) {
    const Scratch w = carve(workspace, B, M, N);
    if (workspace == nullptr || workspace_bytes < w.bytes)
        return fail(kWorkspaceTooSmall,
                    "knn: workspace must hold " + std::to_string(w.bytes) + " bytes");
    if (B > 65535) return fail(kInvalidArgument, "knn: batch must be at most 65535");
    const int kk = (int)k, DD = (int)D;
    if (kk <= 8) return run_tc<8>(query, ref, B, M, N, DD, kk, dist, idx, sqdist, w, s);
    if (kk <= 16) return run_tc<16>(query, ref, B, M, N, DD, kk, dist, idx, sqdist, w, s);
    return run_tc<32>(query, ref, B, M, N, DD, kk, dist, idx, sqdist, w, s);
}

}  // namespace mpo
