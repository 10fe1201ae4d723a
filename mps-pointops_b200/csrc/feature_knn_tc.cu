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
//  1. Pack (fknn_prep_kernel): queries and references are rounded to tf32
//     (cvt.rna: 11 significant bits) and written once in the operand layout
//     of the MMA (per 128-row tile, K-major core matrices), so a tile reaches
//     shared memory with one bulk copy.  After the Kpad feature columns every
//     row has an 8-column norm block: a reference row carries tf32(-n(r)/2)
//     (n(p) = sum of p_t^2 in fp32; -2^100 for padding rows past N).  The
//     same pass writes the query norms, per cloud the largest reference norm,
//     and a flag for non-finite or huge norms (such clouds skip the tensor
//     path).  When the queries are the references (the same array), one pack
//     serves both operands.
//  2. Approximate scores (fknn_tc_kernel): a CTA owns 128 queries; warp 0
//     streams 128-reference tiles into a shared-memory ring with
//     cp.async.bulk, warp 1 issues tcgen05.mma kind::tf32 (tf32 x tf32 -> fp32,
//     M = 128, N = 128, K = 8) over the feature columns and one more MMA that
//     pairs the references' norm block with a constant block of ones in
//     shared memory, into one of two TMEM accumulators (128 lanes x 128
//     columns each), so the accumulator holds
//         t_j = tf32(q) . tf32(r_j) + tf32(-n(r_j) / 2),   s_j := -2 t_j,
//     and SD'_j = n(q) + s_j approximates SD_j with |SD'_j - SD_j| <= eps(q) =
//     C_K (n(q) + max n(r)).  Eight epilogue warps (two groups of four, one
//     thread per query) read the accumulators with tcgen05.ld:
//       pass 1: the maximum of t in each of 64 column buckets; the k-th
//               smallest bucket minimum U of s = -2 t bounds the k-th
//               smallest s from above (k buckets -> k distinct columns);
//       pass 2: every column with s_j <= U + 2 eps(q), i.e. t_j >=
//               -(U + 2 eps(q)) / 2, is appended to the query's candidate
//               list (capacity kCap).
//     The k nearest by exact SD are all candidates: F_k <= n(q) + U + eps
//     (k columns have SD' <= n(q) + U), and a needed column has
//     SD' <= F_k + eps.
//  3. Exact re-rank (fknn_rerank_half_kernel for 16-byte rows,
//     fknn_rerank_kernel otherwise): exact fp32 SD of every candidate,
//     ranked by (SD, index).  A query whose list overflowed, or whose cloud
//     was flagged, is scanned exactly over all references instead
//     (fknn_exact_rows_kernel).
//
// Error bound C_K (per unit of n(q) + n(r), K = Kpad): rounding to tf32
// moves each coordinate by at most u|p| with u = 2^-11, so a product
// q_t r_t moves by at most (2u + u^2)|q_t||r_t| (the tf32 products are exact
// in fp32), the dot product by (2u + u^2)(n(q) + n(r)) / 2 and s by twice
// that; rounding -n(r)/2 to tf32 moves s by at most u n(r); the fp32
// accumulation of K + 8 terms inside the tensor core, the norms and the
// reference's own rounding add the rest.  C_K = 2 * (2^-10 + 2^-11 + 2^-22 +
// (K + 8) 2^-21 + (3D + 16) 2^-24) is about twice the sum of those terms.
// (Three bf16 products hi.hi' + hi.lo' + lo.hi' give a bound about 10x
// tighter for 3x the MMA work; on the config-4 shapes the tf32 bound adds a
// few candidates per query, which the re-rank absorbs.)
//
// Every wait on an mbarrier is bounded (kWaitNs of %globaltimer); on expiry
// the CTA records status 1, the waiting role stops, the rows of the CTA are
// sent to the exact path, and the TMEM is freed before the CTA exits.
#include <string>

#include "../../include/mpo_b200.h"
#include "knn_select.cuh"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kTM = 128;         // queries per CTA (TMEM lanes)
constexpr int kTN = 128;         // references per tile (accumulator columns)
constexpr int kMaxD = 96;        // widest feature vector of the tensor path (shared memory)
constexpr int kCap = 64;         // candidates kept per query
constexpr int kMaxK = 32;        // largest k served by this path
constexpr int kQT = 1;           // 128-query tiles per CTA (share every reference tile)
constexpr int kRows = kQT * kTM;  // queries per CTA
// Warp 0 producer, warp 1 MMA, 8 kQT epilogue warps.  One 128-query tile per
// CTA and two CTAs per SM: a second CTA fills the gaps of the first one's MMA
// issue and epilogue (config 4: 0.370 -> 0.345 ms against two query tiles per
// CTA and one CTA per SM).
constexpr int kThreadsTC = 64 + 256 * kQT;
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr float kHuge = 1.15292150e18f;  // 2^60: larger norms go to the exact path

// Operand layout of one 128-row tile of tf32 values, K-major core matrices
// (8 rows x 16 bytes) without swizzle: element (row, t) sits at
//   (row / 8) * SBO + (t / 4) * 128 + (row % 8) * 16 + (t % 4) * 4,
// SBO = W / 4 * 128, W = the tile's width in tf32 values.  A packed row holds
// Kpad feature columns (D padded to 16) and one 8-column norm block: column
// Kpad holds tf32(-n(p) / 2) for a reference (-2^100 for a padding row past
// N), the rest zeros.  The norm block of a query row is never read: the MMAs
// pair the references' norm block with a constant block of ones (column 0 =
// 1.0) held in shared memory, so the accumulator receives
//   t_j = tf32(q) . tf32(r_j) + tf32(-n(r_j) / 2)  =  -s_j / 2
// directly, and the epilogue needs no per-column arithmetic.
__host__ __device__ constexpr int kpad_of(int D) { return (D + 15) / 16 * 16; }
__host__ __device__ constexpr int width_of(int D) { return kpad_of(D) + 8; }
__host__ __device__ constexpr int part_bytes(int W) { return 128 * W * 4; }
constexpr int kOnesBytes = 128 * 8 * 4;  // the constant ones block (128 rows x 8 tf32)
constexpr float kPadNorm = 1.26765060e30f;  // 2^100: t = -2^100 for padding columns

// Shared memory: A (kQT tiles) | nst stages x B (also the epilogue's handoff
// area once the tiles are done) | the ones block | barriers.
constexpr int kMaxStages = 4;
// Barrier indices: full[kMaxStages] | empty[kMaxStages] | accf[2] | acce[2] |
// afull; then the TMEM address and the abort flag.
constexpr int kBarFull = 0, kBarEmpty = kMaxStages, kBarAccF = 2 * kMaxStages,
              kBarAccE = kBarAccF + 2, kBarAFull = kBarAccE + 2, kBarCount = kBarAFull + 1;
constexpr int kBarBytes = 256;
static_assert(kBarCount * 8 + 8 <= kBarBytes, "barrier region");
struct TcSmem {
    int part, a_off, b_off, stage_bytes, ones_off, bar_off, total;
    __host__ __device__ TcSmem(int W, int nst) {
        part = part_bytes(W);
        a_off = 0;
        b_off = kQT * part;
        stage_bytes = part;
        ones_off = b_off + nst * stage_bytes;
        if (ones_off - b_off < 66 * kRows * 4) ones_off = b_off + 66 * kRows * 4;  // epilogue handoff
        bar_off = ones_off + kOnesBytes;
        total = bar_off + kBarBytes;
    }
};
constexpr int kSmemLimit = 232448;  // opt-in shared memory per CTA on sm_100
constexpr int kSmemPair = 115712;   // per CTA when two CTAs share an SM (228 KiB, 1 KiB each reserved)
// The deepest ring that still lets two CTAs share an SM, else (wide features)
// the deepest ring for one CTA per SM.
inline int stages_for(int W) {
    for (int nst = kMaxStages; nst >= 2; --nst)
        if (TcSmem(W, nst).total <= kSmemPair) return nst;
    for (int nst = kMaxStages; nst > 2; --nst)
        if (TcSmem(W, nst).total <= kSmemLimit) return nst;
    return 2;
}

// ---- PTX wrappers (tcgen05, mbarrier, bulk copies, proxies) -----------------
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
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
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
// Instruction descriptor: kind::tf32, A = B = tf32 (format 2, K-major), D =
// f32, M = 128, N = kTN.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
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

// Three-input maximum (PTX max.f32 with three sources; the scores it is used
// on are never NaN).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Round to tf32 (nearest, ties away from zero): 11 significant bits, the
// low 13 bits of the result are zero.
__device__ __forceinline__ uint32_t tf32_bits(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Arrive on bar and add tx bytes that the following bulk copies will complete.
__device__ __forceinline__ void bulk_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
// Plain (non-multicast) bulk copy global -> own shared memory; completion is
// signalled as tx bytes on bar.  Addresses and size are multiples of 16.
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// ---- 1. pack and norms --------------------------------------------------------
// Thread per (padded row, 8-feature chunk): 2^lg consecutive lanes per row
// (the chunk count Kpad / 8 rounded up to a power of two), so that a row's
// lanes form one aligned group of a warp; the packed row is W = Kpad + 8
// columns wide.  Grid (rows of one cloud, B, 2): z = 0 packs the references
// (ntiles * 128 rows per cloud), z = 1 the queries (mtiles * 128 rows; not
// launched when `same`: the queries are the references), y = the cloud, so
// no thread divides by a run-time row count.  Rows past n and features past
// D pack zeros.  Each lane sums the squares of its 8 features in order; a
// butterfly over the row's lanes gives the norm (every lane the same sum,
// fp32 addition being commutative); each lane packs its two 16-byte
// core-matrix rows of features, and lane 0 also the norm block: tf32(-n / 2)
// (references; -2^100 for padding rows) or zeros (queries).  vec: rows are
// read as float4 (D % 4 == 0 and 16-byte aligned bases).  nq receives the
// query norms; nmax = largest finite reference norm per cloud (one atomic per
// warp), bad = a norm that is not finite or above kHuge.
__global__ void fknn_prep_kernel(const float* __restrict__ q, const float* __restrict__ r,
                                 int64_t M, int64_t N, int D, int W, int64_t mtiles,
                                 int64_t ntiles, int vec, int same, int lg,
                                 unsigned char* __restrict__ qpack,
                                 unsigned char* __restrict__ rpack, float* __restrict__ nq,
                                 unsigned* __restrict__ nmax, int* __restrict__ bad) {
    const int chunks = W / 8 - 1;  // feature chunks (the norm block follows)
    const bool is_ref = blockIdx.z == 0;
    const int64_t b = blockIdx.y;
    const int64_t tiles = is_ref ? ntiles : mtiles, n = is_ref ? N : M;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t i = e >> lg;  // row within the cloud
    const int c = (int)(e & ((1 << lg) - 1));
    const bool row_live = i < tiles * 128;
    const bool point = row_live && i < n;
    float x[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) x[t] = 0.f;
    if (point && c * 8 < D) {
        const float* src = (is_ref ? r : q) + (b * n + i) * D + c * 8;
        if (vec && c * 8 + 8 <= D) {
            const float4 u = reinterpret_cast<const float4*>(src)[0];
            const float4 v = reinterpret_cast<const float4*>(src)[1];
            x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
            x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) x[t] = (c * 8 + t < D) ? src[t] : 0.f;
        }
    }
    float s = __fmul_rn(x[0], x[0]);
#pragma unroll
    for (int t = 1; t < 8; ++t) s = __fadd_rn(s, __fmul_rn(x[t], x[t]));
    for (int off = (1 << lg) >> 1; off >= 1; off >>= 1)
        s = __fadd_rn(s, __shfl_xor_sync(FULL_MASK, s, off));
    if (row_live && c < chunks) {
        const int64_t tile = i / 128;
        const int rr = (int)(i % 128);
        unsigned char* blk =
            (is_ref ? rpack : qpack) + (size_t)(b * tiles + tile) * part_bytes(W);
        const int row_off = (rr >> 3) * (W / 4 * 128) + (rr & 7) * 16;
        const int off = row_off + (2 * c) * 128;
        *reinterpret_cast<uint4*>(blk + off) =
            make_uint4(tf32_bits(x[0]), tf32_bits(x[1]), tf32_bits(x[2]), tf32_bits(x[3]));
        *reinterpret_cast<uint4*>(blk + off + 128) =
            make_uint4(tf32_bits(x[4]), tf32_bits(x[5]), tf32_bits(x[6]), tf32_bits(x[7]));
        if (c == 0) {
            // Norm block: -n / 2 (exact halving, then tf32) for a reference,
            // -2^100 for a padding reference row, zeros for a query.
            const float aug = is_ref ? (point ? -0.5f * s : -kPadNorm) : 0.f;
            const int noff = row_off + (2 * chunks) * 128;
            *reinterpret_cast<uint4*>(blk + noff) = make_uint4(tf32_bits(aug), 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(blk + noff + 128) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    unsigned bits = 0u;
    if (point && c == 0) {
        const bool ok = isfinite(s) && s <= kHuge;
        if (!ok) bad[b] = 1;
        if (!is_ref || same) nq[b * M + i] = s;
        if (is_ref && ok) bits = __float_as_uint(s);
    }
    if (is_ref) {  // block-uniform: one cloud's references per block
        // One atomic per block (same-address atomics serialise at L2).
        __shared__ unsigned s_mx[8];
        const unsigned mx = __reduce_max_sync(FULL_MASK, bits);
        if ((threadIdx.x & 31) == 0) s_mx[threadIdx.x >> 5] = mx;
        __syncthreads();
        if (threadIdx.x < 32) {
            const unsigned v = threadIdx.x < (blockDim.x >> 5) ? s_mx[threadIdx.x] : 0u;
            const unsigned bm = __reduce_max_sync(FULL_MASK, v);
            if (threadIdx.x == 0 && bm) atomicMax(&nmax[b], bm);
        }
    }
}

// Error coefficient C_K of the approximate score (per unit of n(q) + n(r),
// K = Kpad): 2 (2^-10 + 2^-22) for the tf32 rounding of the features,
// 2^-11 for the tf32 rounding of -n(r) / 2 (times 2: the score is -2 t),
// (K + 8) 2^-21 for the fp32 accumulation of K + 8 terms inside the tensor
// core (2 ulps per term), (3 D + 16) 2^-24 for the fp32 norms and the
// reference's own rounding; the whole sum is doubled as a margin.
__device__ __forceinline__ float eps_coef(int D) {
    const int K = kpad_of(D);
    return 2.f * (9.765625e-4f /* 2^-10 */ + 4.8828125e-4f /* 2^-11 */ +
                  2.384185791015625e-7f /* 2^-22 */ +
                  (float)(K + 8) * 4.76837158203125e-7f /* 2^-21 */ +
                  (3.f * (float)D + 16.f) * 5.9604644775390625e-8f /* 2^-24 */);
}

// ---- 2. approximate scores on the tensor cores ------------------------------
// Barriers: full[s] (producer expect_tx + bulk-copy bytes), empty[s] (MMA
// commit: operands of stage s read), accf[a] (MMA commit: accumulator a
// written), acce[a] (4 epilogue warps: accumulator a read), afull (query
// tile).  Phase parity of round n = n & 1; "free" barriers are waited with
// the opposite parity first.
//
// The accumulator holds t_j = -s_j / 2 (exactly: s'_j := -2 t'_j), so
//   pass 1: bucket maxima of t (= -1/2 x bucket minima of s), written to the
//           handoff area as s = -2 t; each epilogue group sorts its 32
//           buckets in registers and group 0 takes the k-th smallest of the
//           two sorted runs by a k-step merge;
//   pass 2: a column joins when t_j >= -(U + 2 eps) / 2, i.e. s_j <= U + 2 eps
//           (halving and -2 t are exact); the candidate mask of a 32-column
//           chunk costs one packed subtraction per two columns and one funnel
//           shift per column.
template <int PASS>
__global__ void __launch_bounds__(kThreadsTC, 2)
fknn_tc_kernel(const unsigned char* __restrict__ qpack, const unsigned char* __restrict__ rpack,
               int64_t M, int64_t N, int64_t mtiles, int64_t ntiles, int D, int k,
               const float* __restrict__ nq, const unsigned* __restrict__ nmax,
               const int* __restrict__ bad, float* __restrict__ ubound,
               unsigned* __restrict__ counts, uint2* __restrict__ cand,
               int* __restrict__ status, int nst) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.y;
    const int64_t mt = blockIdx.x;
    if (bad[b]) return;  // uniform: the cloud goes to the exact path
    const int Kpad = kpad_of(D), W = width_of(D);
    const TcSmem L(W, nst);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar = sbase + L.bar_off;
    auto B_ = [&](int i) { return bar + 8u * (uint32_t)i; };
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L.bar_off + kBarCount * 8);
    int* s_abort = reinterpret_cast<int*>(smem + L.bar_off + kBarCount * 8 + 4);

    // The ones block: column 0 of every row = 1.0 (tf32), else 0.  Written
    // with generic stores, then made visible to the tensor core's (async
    // proxy) operand reads before the CTA barrier.
    {
        uint32_t* ones = reinterpret_cast<uint32_t*>(smem + L.ones_off);
        for (int w = tid; w < kOnesBytes / 4; w += kThreadsTC) {
            // word w: byte 4 w = (row/8)*256 + (t/4)*128 + (row%8)*16 + (t%4)*4
            const int t = ((w >> 5) & 1) * 4 + (w & 3);
            ones[w] = t == 0 ? 0x3f800000u : 0u;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_u32(s_tmem), 2 * kQT * kTN);
    if (tid == 0) {
        for (int i = 0; i < kMaxStages; ++i) {
            mbar_init(B_(kBarFull + i), 1);
            mbar_init(B_(kBarEmpty + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(B_(kBarAccF + i), 1);
            mbar_init(B_(kBarAccE + i), 4 * kQT);
        }
        mbar_init(B_(kBarAFull), 1);
        *s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    const uint32_t sbo = (uint32_t)(W / 4 * 128);
    const uint32_t a_bytes = (uint32_t)L.part;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            // kQT consecutive query tiles (the pack has mtiles rounded up).
            const unsigned char* asrc = qpack + (size_t)(b * mtiles + mt * kQT) * a_bytes;
            bulk_expect(B_(kBarAFull), kQT * a_bytes);
            bulk_copy(sbase + L.a_off, asrc, kQT * a_bytes, B_(kBarAFull));
            int64_t issued = 0;
            for (int64_t t = 0; t < ntiles; ++t) {
                const int st = (int)(t % nst);
                const uint32_t n = (uint32_t)(t / nst);
                if (!mbar_wait(B_(kBarEmpty + st), (n & 1) ^ 1) || *(volatile int*)s_abort) {
                    atomicExch(status, 1);
                    *(volatile int*)s_abort = 1;
                    break;
                }
                const uint32_t dst = sbase + L.b_off + (uint32_t)(st * L.stage_bytes);
                bulk_expect(B_(kBarFull + st), a_bytes);
                bulk_copy(dst, rpack + (size_t)(b * ntiles + t) * a_bytes, a_bytes,
                          B_(kBarFull + st));
                ++issued;
            }
            // Copies still in flight (only after an abort) land before exit.
            mbar_wait(B_(kBarAFull), 0);
            for (int64_t t = max64(issued - nst, 0); t < issued; ++t)
                mbar_wait(B_(kBarFull + (int)(t % nst)), (uint32_t)((t / nst) & 1));
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t ones = sbase + L.ones_off;
            const int fsteps = Kpad / 8;  // K = 8 tf32 per MMA: 2 core matrices (256 bytes)
            bool ok = mbar_wait(B_(kBarAFull), 0);
            for (int64_t t = 0; t < ntiles && ok; ++t) {
                const int st = (int)(t % nst), ac = (int)(t & 1);
                const uint32_t n = (uint32_t)(t / nst), na = (uint32_t)(t >> 1);
                ok = mbar_wait(B_(kBarFull + st), n & 1) &&
                     mbar_wait(B_(kBarAccE + ac), (na & 1) ^ 1) && !*(volatile int*)s_abort;
                if (!ok) break;
                tc_fence_after();
                const uint32_t b0 = sbase + L.b_off + (uint32_t)(st * L.stage_bytes);
                for (int qt = 0; qt < kQT; ++qt) {
                    // Accumulator ac of query tile qt: columns (ac * kQT + qt) * kTN.
                    const uint32_t d = tmem + (uint32_t)((ac * kQT + qt) * kTN);
                    const uint32_t a0 = sbase + L.a_off + (uint32_t)qt * a_bytes;
                    for (int s = 0; s < fsteps; ++s) {
                        const uint32_t ko = (uint32_t)s * 256u;
                        mma_tf32(d, smem_desc(a0 + ko, 128, sbo), smem_desc(b0 + ko, 128, sbo),
                                 s == 0 ? 0u : 1u);
                    }
                    // + ones . (-n(r) / 2): the references' norm block.
                    mma_tf32(d, smem_desc(ones, 128, 256),
                             smem_desc(b0 + (uint32_t)fsteps * 256u, 128, sbo), 1u);
                }
                mma_commit(B_(kBarEmpty + st));  // stage st may be refilled
                mma_commit(B_(kBarAccF + ac));   // accumulator ac is ready
            }
            if (!ok) {
                atomicExch(status, 1);
                *(volatile int*)s_abort = 1;
            }
        }
    } else {
        // ---------------- epilogue ----------------
        // Warps 2-17 in sets of 4 (one per TMEM lane quarter): set = 2 g + qt
        // takes query tile qt of the reference tiles t = g (mod 2), i.e.
        // accumulator g; one thread per query.
        const int set = (warp - 2) >> 2;
        const int group = set / kQT, qt = set % kQT;
        const int quarter = warp & 3;
        const int row = qt * kTM + quarter * 32 + lane;
        const int64_t gq = mt * kRows + row;
        const bool qvalid = gq < M;
        const float nqi = qvalid ? nq[(int64_t)b * M + gq] : 0.f;
        const float eps = eps_coef(D) * (nqi + __uint_as_float(nmax[b]));
        // Pass 2: t_j >= tthr makes j a candidate (+inf: no candidates).
        // Group 0 fills the query's list from slot 0 up, group 1 from slot
        // kCap - 1 down.
        uint2* const crow = cand + ((int64_t)b * M + (qvalid ? gq : 0)) * kCap;
        float tthr = INFINITY;
        if (PASS == 2 && qvalid) tthr = -0.5f * (ubound[(int64_t)b * M + gq] + 2.f * eps);
        // Pass 1: bucket h * 16 + u of group g holds the maximum of t over
        // columns 2u and 2u + 1 of the 32-column chunks c with c & 1 == h of
        // the group's tiles; with the other group's buckets, the k-th smallest
        // of the 64 bucket minima of s = -2 t bounds the k-th smallest s from
        // above (k buckets -> k distinct columns).
        float bmax[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) bmax[i] = -INFINITY;
        unsigned found = 0;
        bool ok = true;
        for (int64_t t = group; t < ntiles; t += 2) {
            const int ac = group;
            const uint32_t n = (uint32_t)(t >> 1);
            const bool got = mbar_wait(B_(kBarAccF + ac), n & 1);
            ok = __all_sync(FULL_MASK, got) && !*(volatile int*)s_abort;
            if (!ok) break;
            tc_fence_after();
            // Chunks in pairs: chunk c feeds buckets (c & 1) * 16 + u, and
            // the pair index h = c & 1 is a compile-time constant.
#pragma unroll 1
            for (int c2 = 0; c2 < kTN / 32; c2 += 2) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int c = c2 + h;
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) +
                              (uint32_t)((ac * kQT + qt) * kTN + c * 32),
                          v);
                if (PASS == 1) {
                    // Columns 2u and 2u + 1 of the chunk -> bucket h * 16 + u.
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        bmax[16 * h + 2 * i] = fmax3(bmax[16 * h + 2 * i], v[4 * i], v[4 * i + 1]);
                        bmax[16 * h + 2 * i + 1] =
                            fmax3(bmax[16 * h + 2 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    }
                } else {
                    // Candidate mask of the 32 columns: d = t - tthr for two
                    // columns per packed subtraction; t_j >= tthr exactly when
                    // d_j's sign bit is clear (an exact difference of finite
                    // floats is never -0, and the subtraction keeps
                    // subnormals).  One funnel shift per column moves d_j's
                    // sign bit into a running word (four independent words
                    // of 8 columns), so bit 31 - j of `miss` is set when
                    // column j is not a candidate.
                    const f32x2 T2 = pack2(tthr, tthr);
                    uint32_t acc[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float d0, d1;
                        unpack2(sub2(pack2(v[2 * i], v[2 * i + 1]), T2), d0, d1);
                        uint32_t& a = acc[i >> 2];
                        a = __funnelshift_l(__float_as_uint(d0), a, 1);
                        a = __funnelshift_l(__float_as_uint(d1), a, 1);
                    }
                    uint32_t hits = ~((acc[0] << 24) | (acc[1] << 16) | (acc[2] << 8) | acc[3]);
                    if (hits) {
                        // Bit 31 - j set: column j is a candidate (about one
                        // column in 170).
                        const uint32_t col0 = (uint32_t)(t * kTN + c * 32);
                        do {
                            const int j = __clz(hits);
                            hits ^= 0x80000000u >> j;
                            if (found < (unsigned)kCap)
                                crow[group ? (int)(kCap - 1 - found) : (int)found] =
                                    make_uint2(col0 + (uint32_t)j, 0u);
                            ++found;
                        } while (hits);
                    }
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(B_(kBarAccE + ac));  // accumulator read
        }
        if (!ok) {
            if (lane == 0) atomicExch(status, 1);
            *(volatile int*)s_abort = 1;
        }
        // Hand group 1's state to group 0 through the (idle) B stages:
        // s_x[u * kRows + row] = bucket u of s (0-31 group 0, 32-63 group 1),
        // each group's run sorted ascending; then group 1's count and status.
        float* s_x = reinterpret_cast<float*>(smem + L.b_off);
        named_barrier_sync(1, 8 * kQT * 32);  // both epilogue groups finished their tiles
        if (PASS == 1) {
            // s = -2 t (exact); ascending s = descending t.  Bitonic network
            // over the 32 registers (compile-time indices).
#pragma unroll
            for (int i = 0; i < 32; ++i) bmax[i] = -2.f * bmax[i];
#pragma unroll
            for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int j = i ^ stride;
                        if (j > i) {
                            const float lo = fminf(bmax[i], bmax[j]), hi = fmaxf(bmax[i], bmax[j]);
                            const bool up = (i & size) == 0;
                            bmax[i] = up ? lo : hi;
                            bmax[j] = up ? hi : lo;
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) s_x[(32 * group + i) * kRows + row] = bmax[i];
        }
        if (group == 1) {
            s_x[64 * kRows + row] = __uint_as_float(found);
            s_x[65 * kRows + row] = ok ? 1.f : 0.f;
        }
        named_barrier_sync(1, 8 * kQT * 32);
        if (group == 0) {
            ok = ok && s_x[65 * kRows + row] != 0.f;
            if (PASS == 1) {
                // k-th smallest of the two sorted runs of 32 (k <= 32).
                int ia = 0, ib = 0;
                float kth = INFINITY;
                for (int i = 0; i < k; ++i) {
                    const float x0 = ia < 32 ? s_x[ia * kRows + row] : INFINITY;
                    const float x1 = ib < 32 ? s_x[(32 + ib) * kRows + row] : INFINITY;
                    const bool first = !(x1 < x0);
                    kth = first ? x0 : x1;
                    ia += first ? 1 : 0;
                    ib += first ? 0 : 1;
                }
                if (qvalid) ubound[(int64_t)b * M + gq] = ok ? kth : INFINITY;
            } else if (qvalid) {
                const unsigned f1 = __float_as_uint(s_x[64 * kRows + row]);
                // Packed (group 0 count, group 1 count); overflow -> exact path.
                counts[(int64_t)b * M + gq] =
                    (ok && found + f1 <= (unsigned)kCap) ? (found | (f1 << 16)) : 0xffffffffu;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * kQT * kTN);
    }
}

// ---- 3. exact re-rank --------------------------------------------------------
// Warp per query.  Normal case: the warp copies its candidates' reference rows
// (whole, or in two halves for 16-byte rows) into shared memory with
// coalesced cp.async (a lane per row would touch one cache line per lane and
// load), lane l computes the exact sequential-fp32 SD of candidates l and
// l + 32 from there (non-finite SD are dropped), and a warp bitonic sort of
// the (SD, index) keys gives the first k.  Overflowed lists and flagged
// clouds: the lanes scan every reference (j = lane mod 32) into per-lane
// sorted lists, merged by k rounds of warp minimum.

// Exact sequential SD of query row qs (shared memory) and reference row rp
// (global memory), reading the reference 32 features at a time (8 float4
// loads in flight per lane when rows are 16-byte aligned, vec != 0).
__device__ __forceinline__ float sqd_staged(const float* __restrict__ qs,
                                            const float* __restrict__ rp, int D, int vec) {
    if (!vec) return sqd_seq(qs, rp, D);
    const float4* r4 = reinterpret_cast<const float4*>(rp);
    float s = 0.f;
    for (int t0 = 0; t0 < D; t0 += 32) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            v[u] = (t0 + 4 * u < D) ? __ldg(r4 + t0 / 4 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int t = t0 + 4 * u;
            if (t < D) {
                float d = __fsub_rn(qs[t], v[u].x);
                s = (t == 0) ? __fmul_rn(d, d) : __fadd_rn(s, __fmul_rn(d, d));
                d = __fsub_rn(qs[t + 1], v[u].y);
                s = __fadd_rn(s, __fmul_rn(d, d));
                d = __fsub_rn(qs[t + 2], v[u].z);
                s = __fadd_rn(s, __fmul_rn(d, d));
                d = __fsub_rn(qs[t + 3], v[u].w);
                s = __fadd_rn(s, __fmul_rn(d, d));
            }
        }
    }
    return s;
}

// Row stride (floats) of the scalar re-rank's staged rows: an odd number of
// floats, so that 32 lanes reading the same column of 32 rows hit distinct
// banks.
__host__ __device__ constexpr int rerank_stride(int D) { return (D & 1) ? D : D + 1; }
constexpr int kRerankWarps = 8;
// Shared memory of one scalar re-rank CTA: per warp the query row and 32 staged rows.
inline size_t rerank_smem_bytes(int D) {
    return (size_t)kRerankWarps * 33 * rerank_stride(D) * sizeof(float);
}

// 16-byte rows (D % 4 == 0, both arrays 16-byte aligned): the candidates'
// rows are staged in two parts, features [0, Dh) and [Dh, D) with Dh the
// first half rounded to whole float4s; the sequential SD runs on across the
// parts.  A staged part's stride is an odd number of float4s (conflict-free
// lane-per-row float4 reads).
__host__ __device__ constexpr int half_split(int D) { return ((D / 4 + 1) / 2) * 4; }
__host__ __device__ constexpr int half_stride(int D) { return 4 * ((half_split(D) / 4) | 1); }
// Per warp: the query row (D floats) and 32 staged parts.
inline size_t rerank_half_smem_bytes(int D) {
    return (size_t)kRerankWarps * (D + 32 * half_stride(D)) * sizeof(float);
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// One compare-exchange stage of a warp bitonic sort over 64-bit keys: the
// element with position e (its lane, or 32 + lane for a second half) keeps
// the smaller key of its pair when its block of `size` sorts ascending and it
// is the lower element of the pair, or neither.
__device__ __forceinline__ uint64_t bitonic_step(uint64_t key, int e, int size, int stride) {
    const uint64_t other = __shfl_xor_sync(FULL_MASK, key, stride);
    const bool keep_min = ((e & size) == 0) == ((e & stride) == 0);
    const uint64_t lo = other < key ? other : key, hi = other < key ? key : other;
    return keep_min ? lo : hi;
}

// Rank the warp's (SD, index) pairs (lane holds candidates lane and 32 +
// lane; empty slots are (inf, kNoIndex)) and write the first k.
__device__ __forceinline__ void rerank_emit(const float (&sd)[2], const uint32_t (&jj)[2],
                                            unsigned cnt, int k, int lane,
                                            float* __restrict__ dist,
                                            int64_t* __restrict__ idx64,
                                            float* __restrict__ sqdist, int64_t o) {
    // Sort the (SD, index) pairs as 64-bit keys (finite SD >= 0: the bits
    // order like the values; an empty slot is (inf, kNoIndex), after all):
    // a warp bitonic sort of 32 keys, or of 64 keys (two per lane, element
    // 32 h + lane) when the list has more than 32 candidates.
    uint64_t a0 = ((uint64_t)__float_as_uint(sd[0]) << 32) | jj[0];
    if (cnt > 32u) {
        uint64_t a1 = ((uint64_t)__float_as_uint(sd[1]) << 32) | jj[1];
#pragma unroll
        for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                if (stride == 32) {
                    const uint64_t lo = a1 < a0 ? a1 : a0, hi = a1 < a0 ? a0 : a1;
                    a0 = lo;
                    a1 = hi;
                } else {
                    a0 = bitonic_step(a0, lane, size, stride);
                    a1 = bitonic_step(a1, 32 + lane, size, stride);
                }
            }
        }
    } else {
        // Up to 32 candidates: sort 32-bit keys (SD bits with the low five
        // bits replaced by the lane) and fetch each rank's entry from its
        // lane.  The order equals the (SD, index) order unless two finite SD
        // among the first k + 1 ranks agree above their low five bits; then
        // (rarely) the 64-bit keys are sorted instead.
        uint32_t k32 = (__float_as_uint(sd[0]) & ~31u) | (uint32_t)lane;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                const uint32_t other = __shfl_xor_sync(FULL_MASK, k32, stride);
                const bool keep_min = ((lane & size) == 0) == ((lane & stride) == 0);
                k32 = keep_min ? min(k32, other) : max(k32, other);
            }
        }
        const uint32_t prev = __shfl_up_sync(FULL_MASK, k32, 1);
        const bool close = lane >= 1 && lane <= k && (k32 >> 5) == (prev >> 5) &&
                           (k32 >> 5) < (0x7f800000u >> 5);
        if (__any_sync(FULL_MASK, close)) {
#pragma unroll
            for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
                for (int stride = size >> 1; stride > 0; stride >>= 1)
                    a0 = bitonic_step(a0, lane, size, stride);
            }
        } else {
            const int src = (int)(k32 & 31u);
            const uint32_t sj = __shfl_sync(FULL_MASK, jj[0], src);
            const float sdv = __shfl_sync(FULL_MASK, sd[0], src);
            a0 = ((uint64_t)__float_as_uint(sdv) << 32) | sj;
        }
    }
    if (lane < k) {
        const uint32_t j = (uint32_t)a0;
        const float d = __uint_as_float((uint32_t)(a0 >> 32));
        const bool filled = j != kNoIndex;
        dist[o + lane] = filled ? sqrtf(d) : INFINITY;
        if (sqdist) sqdist[o + lane] = filled ? d : INFINITY;
        idx64[o + lane] = filled ? (int64_t)j : -1;
    }
}

// Scalar rows (any alignment or width).  Grid (ceil(M / warps), B).  The
// warp copies its candidates' rows into shared memory with coalesced 4-byte
// cp.async (LPR lanes per row), lane l computes candidate l's exact SD from
// there, for candidates 0-31 and then 32-63.
__global__ void __launch_bounds__(kRerankWarps * 32)
fknn_rerank_kernel(const float* __restrict__ q, const float* __restrict__ r, int64_t M,
                   int64_t N, int D, int k, const int* __restrict__ bad,
                   const unsigned* __restrict__ counts, const uint2* __restrict__ cand,
                   float* __restrict__ dist, int64_t* __restrict__ idx64,
                   float* __restrict__ sqdist, unsigned* __restrict__ nover,
                   int64_t* __restrict__ over_rows) {
    static_assert(kCap == 64, "two candidates per lane");
    extern __shared__ __align__(16) float s_stage[];  // [warps][33][stride]
    const int lane = threadIdx.x & 31;
    const int64_t m = (int64_t)blockIdx.x * kRerankWarps + (threadIdx.x >> 5);
    if (m >= M) return;  // warp-uniform
    const int64_t b = blockIdx.y;
    const int64_t row = b * M + m;
    const float* rb = r + b * N * D;
    const int stride = rerank_stride(D);
    float* qp = s_stage + (threadIdx.x >> 5) * 33 * stride;
    float* rows = qp + stride;
    const unsigned packed = bad[b] ? 0xffffffffu : counts[row];
    const int64_t o = row * k;
    if (packed == 0xffffffffu) {  // exact scan by fknn_exact_rows_kernel
        if (lane == 0) over_rows[atomicAdd(nover, 1u)] = row;
        return;
    }
    // Candidates: slots [0, f0) from the even tiles, [kCap - f1, kCap) from
    // the odd tiles.
    const unsigned f0 = packed & 0xffffu, f1 = packed >> 16, cnt = f0 + f1;
    for (int t = lane; t < D; t += 32) qp[t] = q[row * D + t];
    // LPR lanes per row (the largest power of two <= min(D, 8)), so one copy
    // instruction covers R = 32 / LPR rows.
    const int LPR = D >= 8 ? 8 : (D >= 4 ? 4 : (D >= 2 ? 2 : 1));
    const int R = 32 / LPR;
    const int roff = lane / LPR;
    const int u0 = lane % LPR;
    float sd[2];
    uint32_t jj[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        sd[h] = INFINITY;
        jj[h] = kNoIndex;
        const unsigned c0 = 32u * (unsigned)h;
        if (c0 >= cnt) continue;  // warp-uniform
        const unsigned n = min(32u, cnt - c0);
        const unsigned c = c0 + (unsigned)lane;
        uint32_t j = kNoIndex;
        if (c < cnt) {
            const unsigned slot = c < f0 ? c : (unsigned)kCap - 1u - (c - f0);
            j = cand[row * kCap + slot].x;
        }
        for (unsigned base = 0; base < n; base += (unsigned)R) {
            const unsigned rl = base + (unsigned)roff;
            const uint32_t jr = __shfl_sync(FULL_MASK, j, (int)(rl & 31u));
            if (rl < n && jr < (uint32_t)N) {
                const float* src = rb + (int64_t)jr * D;
                float* dst = rows + rl * stride;
                for (int u = u0; u < D; u += LPR) cp_async4(dst + u, src + u);
            }
        }
        cp_async_wait_all();
        __syncwarp();
        if (c < cnt && j < (uint32_t)N) {
            const float v = sqd_seq(qp, rows + lane * stride, D);
            if (isfinite(v)) {
                sd[h] = v;
                jj[h] = j;
            }
        }
        __syncwarp();  // the rows are refilled for the second half
    }
    rerank_emit(sd, jj, cnt, k, lane, dist, idx64, sqdist, o);
}

// Exact sequential SD over features [t0, t1) (multiples of 4) of the query
// row qa and the staged part rb (rb holds features from t0 on), continuing
// the running sum s; t0 == 0 starts it.  Both rows 16-byte aligned.  The
// squares of two consecutive features do not depend on each other: each pair
// takes one packed subtraction and one packed square (each lane rounded on
// its own, the bits of __fsub_rn / __fmul_rn), and only the additions stay
// scalar and in feature order -- 4 instructions per two features instead of 6.
template <int T0, int T1>
__device__ __forceinline__ void sqd_part(const float* __restrict__ qa,
                                         const float* __restrict__ rb, int t0, int t1,
                                         float& s) {
    const int a = T1 ? T0 : t0, e = T1 ? T1 : t1;
#pragma unroll(T1 ? (T1 - T0) / 4 : 4)
    for (int t = a; t < e; t += 4) {
        const float4 x = *reinterpret_cast<const float4*>(qa + t);
        const float4 y = *reinterpret_cast<const float4*>(rb + (t - a));
        float p0, p1, p2, p3;
        unpack2(sq2(sub2(pack2(x.x, x.y), pack2(y.x, y.y))), p0, p1);
        unpack2(sq2(sub2(pack2(x.z, x.w), pack2(y.z, y.w))), p2, p3);
        s = (t == 0) ? p0 : __fadd_rn(s, p0);
        s = __fadd_rn(s, p1);
        s = __fadd_rn(s, p2);
        s = __fadd_rn(s, p3);
    }
}

// 16-byte rows.  Candidates' rows are staged in two half-row parts (so a
// warp needs 4.9 KB of shared memory at D = 64, 40 warps per SM), each copied
// with coalesced 16-byte cp.async: 8 lanes per row, four rows per copy
// instruction; the warp waits for its own copies with cp.async.wait_all.
// The sequential SD runs on across the parts.  Grid (ceil(M / warps), B).
template <int DC>
__global__ void __launch_bounds__(kRerankWarps * 32)
fknn_rerank_half_kernel(const float* __restrict__ q, const float* __restrict__ r, int64_t M,
                        int64_t N, int D_rt, int k, const int* __restrict__ bad,
                        const unsigned* __restrict__ counts, const uint2* __restrict__ cand,
                        float* __restrict__ dist, int64_t* __restrict__ idx64,
                        float* __restrict__ sqdist, unsigned* __restrict__ nover,
                        int64_t* __restrict__ over_rows) {
    static_assert(kCap == 64, "two candidates per lane");
    static_assert(DC % 4 == 0, "16-byte rows");
    extern __shared__ __align__(16) float s_stage[];  // [warps][D + 32 * stride]
    const int D = DC ? DC : D_rt;
    constexpr int DH = DC ? half_split(DC) : 0;
    const int Dh = DC ? DH : half_split(D);
    const int hs = half_stride(D);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t m = (int64_t)blockIdx.x * kRerankWarps + warp;
    if (m >= M) return;  // warp-uniform
    const int64_t b = blockIdx.y;
    const int64_t row = b * M + m;
    const float* rb = r + b * N * D;
    const float* qg = q + row * D;
    float* qp = s_stage + warp * (D + 32 * hs);
    float* rows = qp + D;
    float* part = rows + lane * hs;  // this lane's staged row part
    const unsigned packed = bad[b] ? 0xffffffffu : counts[row];
    const int64_t o = row * k;
    if (packed == 0xffffffffu) {  // exact scan by fknn_exact_rows_kernel
        if (lane == 0) over_rows[atomicAdd(nover, 1u)] = row;
        return;
    }
    const unsigned f0 = packed & 0xffffu, f1 = packed >> 16, cnt = f0 + f1;
    for (int t = 4 * lane; t < D; t += 128) cp_async16(qp + t, qg + t);
    const int roff = lane >> 3, u0 = lane & 7;  // 8 lanes per row, 4 rows per instruction
    float sd[2];
    uint32_t jj[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        sd[h] = INFINITY;
        jj[h] = kNoIndex;
        const unsigned c0 = 32u * (unsigned)h;
        if (c0 >= cnt) continue;  // warp-uniform
        const unsigned n = min(32u, cnt - c0);
        const unsigned c = c0 + (unsigned)lane;
        uint32_t j = kNoIndex;
        if (c < cnt) {
            const unsigned slot = c < f0 ? c : (unsigned)kCap - 1u - (c - f0);
            j = cand[row * kCap + slot].x;
        }
        const bool live = c < cnt && j < (uint32_t)N;
        float s = 0.f;
#pragma unroll
        for (int pt = 0; pt < 2; ++pt) {
            const int t0 = pt ? Dh : 0, t1 = pt ? D : Dh;
            const int U = (t1 - t0) / 4;  // float4 per part-row
            for (unsigned base = 0; base < n; base += 4u) {
                const unsigned rl = base + (unsigned)roff;
                const uint32_t jr = __shfl_sync(FULL_MASK, j, (int)(rl & 31u));
                if (rl < n && jr < (uint32_t)N) {
                    const float* src = rb + (int64_t)jr * D + t0;
                    float* dst = rows + rl * hs;
                    for (int u = u0; u < U; u += 8) cp_async16(dst + 4 * u, src + 4 * u);
                }
            }
            cp_async_wait_all();
            __syncwarp();
            if (DC) {
                if (pt == 0) sqd_part<0, DH>(qp, part, 0, 0, s);
                else sqd_part<DH, DC>(qp, part, 0, 0, s);
            } else {
                sqd_part<0, 0>(qp, part, t0, t1, s);
            }
            __syncwarp();  // the part is refilled next
        }
        if (live && isfinite(s)) {
            sd[h] = s;
            jj[h] = j;
        }
    }
    rerank_emit(sd, jj, cnt, k, lane, dist, idx64, sqdist, o);
}

// Rows whose candidate list overflowed, or whose cloud was flagged (listed
// by fknn_rerank_kernel): warp per row, lanes scan references j = lane mod 32
// into per-lane sorted lists, merged by k rounds of warp minimum.
template <int KCAP>
__global__ void __launch_bounds__(256)
fknn_exact_rows_kernel(const float* __restrict__ q, const float* __restrict__ r, int64_t B,
                       int64_t M, int64_t N, int D, int vec, int k,
                       const unsigned* __restrict__ nover,
                       const int64_t* __restrict__ over_rows, float* __restrict__ dist,
                       int64_t* __restrict__ idx64, float* __restrict__ sqdist) {
    extern __shared__ float s_q[];  // [8 warps][D]
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const unsigned nrows = *nover;
    for (int64_t li = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; li < nrows;
         li += warps) {
    const int64_t row = over_rows[li];
    const int64_t b = row / M;
    const float* rb = r + b * N * D;
    float* qp = s_q + (threadIdx.x >> 5) * D;
    for (int t = lane; t < D; t += 32) qp[t] = q[row * D + t];
    __syncwarp();
    const int64_t o = row * k;
    TopK<KCAP, kDropNonFinite> top;
    top.init(k);
    for (int64_t j = lane; j < N; j += 32)
        top.offer(sqd_staged(qp, rb + j * D, D, vec), (uint32_t)j);
    int used = 0;  // entries of this lane's list already emitted
    for (int t = 0; t < k; ++t) {
        float hd = INFINITY;
        uint32_t hj = kNoIndex;
#pragma unroll
        for (int s2 = 0; s2 < KCAP; ++s2) {
            if (s2 == top.base + used && used < top.cnt) {
                hd = top.d[s2];
                hj = top.i[s2];
            }
        }
        float bd = hd;
        uint32_t bj = hj;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float od = __shfl_xor_sync(FULL_MASK, bd, off);
            const uint32_t oj = __shfl_xor_sync(FULL_MASK, bj, off);
            if (oj != kNoIndex && (bj == kNoIndex || before<kDropNonFinite>(od, oj, bd, bj))) {
                bd = od;
                bj = oj;
            }
        }
        if (hj != kNoIndex && hj == bj) ++used;
        if (lane == 0) {
            const bool filled = bj != kNoIndex;
            dist[o + t] = filled ? sqrtf(bd) : INFINITY;
            if (sqdist) sqdist[o + t] = filled ? bd : INFINITY;
            idx64[o + t] = filled ? (int64_t)bj : -1;
        }
    }
    __syncwarp();
    }
}

struct Scratch {
    unsigned char* qpack;
    unsigned char* rpack;
    float* nq;
    float* ubound;
    unsigned* counts;
    uint2* cand;
    unsigned* nmax;
    int* bad;
    int* status;
    unsigned* nover;      // rows for the exact scan
    int64_t* over_rows;   // [B * M]
    size_t bytes;
};

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }
inline size_t flag_bytes(int64_t B) { return (sizeof(unsigned) + sizeof(int)) * B + 8; }

inline Scratch carve(void* base, int64_t B, int64_t M, int64_t N, int64_t D) {
    Scratch s{};
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t at = off;
        off += align256(n);
        return base ? static_cast<unsigned char*>(base) + at : nullptr;
    };
    // Query tiles rounded up to whole CTAs (kQT tiles each).
    const int64_t mt = ceil_div(M, kRows) * kQT, nt = ceil_div(N, kTN);
    const size_t tile = (size_t)part_bytes(width_of((int)D));
    s.qpack = take(tile * B * mt);
    s.rpack = take(tile * B * nt);
    s.nq = reinterpret_cast<float*>(take(sizeof(float) * B * M));
    s.ubound = reinterpret_cast<float*>(take(sizeof(float) * B * M));
    s.counts = reinterpret_cast<unsigned*>(take(sizeof(unsigned) * B * M));
    s.cand = reinterpret_cast<uint2*>(take(sizeof(uint2) * B * M * kCap));
    s.over_rows = reinterpret_cast<int64_t*>(take(sizeof(int64_t) * B * M));
    // nmax, bad, status and nover are contiguous so one memset clears them.
    unsigned char* flags = take(flag_bytes(B));
    s.nmax = reinterpret_cast<unsigned*>(flags);
    s.bad = flags ? reinterpret_cast<int*>(flags + sizeof(unsigned) * B) : nullptr;
    s.status = flags ? reinterpret_cast<int*>(flags + (sizeof(unsigned) + sizeof(int)) * B) : nullptr;
    s.nover = flags ? reinterpret_cast<unsigned*>(flags + (sizeof(unsigned) + sizeof(int)) * B + 4)
                    : nullptr;
    s.bytes = off;
    return s;
}

template <int KCAP>
int run_tc(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int D, int k,
           float* dist, int64_t* idx, float* sqdist, const Scratch& w, cudaStream_t s) {
    if (cudaMemsetAsync(w.nmax, 0, flag_bytes(B), s) != cudaSuccess)
        return fail(kCudaError, "knn: scratch reset failed");
    const int W = width_of(D);
    const int64_t mt = ceil_div(M, kRows) * kQT, nt = ceil_div(N, kTN);
    // kNN of a cloud against itself (knn(f, f, k)): one pack serves both operands.
    const int same = (query == ref && M == N) ? 1 : 0;
    int lg = 0;
    while ((1 << lg) < W / 8 - 1) ++lg;
    const int64_t rows = max64(nt, same ? 0 : mt) * 128;  // per cloud, the longer operand
    // 16-byte row loads only when every row starts on a 16-byte boundary.
    const int vec = (D % 4 == 0 && aligned_to(query, 16) && aligned_to(ref, 16)) ? 1 : 0;
    const dim3 pgrid((unsigned)ceil_div(rows << lg, 256), (unsigned)B, same ? 1u : 2u);
    fknn_prep_kernel<<<pgrid, 256, 0, s>>>(query, ref, M, N, D, W, mt, nt, vec, same, lg,
                                           w.qpack, w.rpack, w.nq, w.nmax, w.bad);
    int st = check_launch("fknn_prep_kernel");
    if (st) return st;
    const unsigned char* qpack = same ? w.rpack : w.qpack;
    const int nst = stages_for(W);
    const TcSmem L(W, nst);
    auto k1 = fknn_tc_kernel<1>;
    auto k2 = fknn_tc_kernel<2>;
    if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total) !=
            cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    dim3 grid((unsigned)(mt / kQT), (unsigned)B);
    k1<<<grid, kThreadsTC, L.total, s>>>(qpack, w.rpack, M, N, mt, nt, D, k, w.nq, w.nmax, w.bad,
                                         w.ubound, w.counts, w.cand, w.status, nst);
    st = check_launch("fknn_tc_kernel<1>");
    if (st) return st;
    k2<<<grid, kThreadsTC, L.total, s>>>(qpack, w.rpack, M, N, mt, nt, D, k, w.nq, w.nmax, w.bad,
                                         w.ubound, w.counts, w.cand, w.status, nst);
    st = check_launch("fknn_tc_kernel<2>");
    if (st) return st;
    // 16-byte rows: half-row parts by 16-byte cp.async (D = 64 compiled with
    // the width fixed); otherwise 4-byte cp.async of whole rows.
    auto rk = !vec ? fknn_rerank_kernel
                   : (D == 64 ? fknn_rerank_half_kernel<64> : fknn_rerank_half_kernel<0>);
    const size_t stage = vec ? rerank_half_smem_bytes(D) : rerank_smem_bytes(D);
    if (cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stage) !=
        cudaSuccess)
        return fail(kCudaError, "knn: cannot raise the shared-memory limit");
    const dim3 rgrid((unsigned)ceil_div(M, kRerankWarps), (unsigned)B);
    rk<<<rgrid, kRerankWarps * 32, stage, s>>>(query, ref, M, N, D, k, w.bad, w.counts, w.cand,
                                               dist, idx, sqdist, w.nover, w.over_rows);
    st = check_launch("fknn_rerank_kernel");
    if (st) return st;
    const size_t rsmem = (size_t)8 * D * sizeof(float);
    fknn_exact_rows_kernel<KCAP><<<(unsigned)(2 * sm_count()), 256, rsmem, s>>>(
        query, ref, B, M, N, D, vec, k, w.nover, w.over_rows, dist, idx, sqdist);
    return check_launch("fknn_exact_rows_kernel");
}

}  // namespace

// The tensor path serves D != 3 with 16 <= D <= 96, k <= 32 and reference
// clouds of at least 2048 points (smaller problems are cheap exactly).
bool fknn_tc_eligible(int64_t M, int64_t N, int64_t D, int64_t k) {
    return D != 3 && D >= 16 && D <= kMaxD && k >= 1 && k <= kMaxK && N >= 2048 && M >= 1 &&
           N <= 0x7fffffffLL;
}

size_t fknn_tc_workspace_bytes(int64_t B, int64_t M, int64_t N, int64_t D) {
    return carve(nullptr, B, M, N, D).bytes;
}

int fknn_tc_run(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int64_t D,
                int64_t k, float* dist, int64_t* idx, float* sqdist, void* workspace,
                size_t workspace_bytes, cudaStream_t s) {
    const Scratch w = carve(workspace, B, M, N, D);
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
