// Exact (SD, index) candidate selection shared by the kNN kernels: the
// candidate policies of the reference's kNN contracts and a register-resident
// sorted top-k list.
#pragma once

#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr uint32_t kNoIndex = 0xffffffffu;

// Candidate policies.
enum Policy : int {
    kDropNaN = 0,        // kNN, D == 3: NaN never enters, +inf is ranked
    kDropNonFinite = 1,  // kNN, D != 3: every non-finite SD is dropped
    kNaNLast = 2,        // three_nn: NaN ranks after every number
};

template <int POLICY>
__device__ __forceinline__ bool admissible(float d) {
    if (POLICY == kDropNaN) return !isnan(d);
    if (POLICY == kDropNonFinite) return isfinite(d);
    return true;
}

// Strict (SD, index) order; with kNaNLast a NaN sorts after every number and
// NaNs sort by index.
template <int POLICY>
__device__ __forceinline__ bool before(float d, uint32_t i, float e, uint32_t j) {
    if (POLICY == kNaNLast) {
        const bool dn = isnan(d), en = isnan(e);
        if (dn != en) return en;
        if (dn) return i < j;
    }
    return d < e || (d == e && i < j);
}

// Register-resident sorted list of capacity K.  The logical list of runtime
// length k (<= K) is right-aligned: physical slot s holds logical entry
// s - (K - k); the K - k leading slots hold (-inf, 0) sentinels that precede
// every candidate and never move.  The k-th entry is therefore always in the
// static slot K - 1 and no register array is ever indexed dynamically.
template <int K, int POLICY>
struct TopK {
    float d[K];
    uint32_t i[K];
    int cnt;   // filled logical entries
    int base;  // K - k

    __device__ __forceinline__ void init(int k) {
        base = K - k;
#pragma unroll
        for (int s = 0; s < K; ++s) {
            d[s] = s < base ? -INFINITY : INFINITY;
            i[s] = s < base ? 0u : kNoIndex;
        }
        cnt = 0;
    }

    // Offer (dd, jj): the candidate bubbles down the sorted list, swapping
    // with every entry it precedes (empty slots always yield).
    __device__ __forceinline__ void offer(float dd, uint32_t jj) {
        if (!admissible<POLICY>(dd)) return;
        if (cnt >= K - base && !before<POLICY>(dd, jj, d[K - 1], i[K - 1])) return;
        const int empty_from = base + cnt;
#pragma unroll
        for (int s = 0; s < K; ++s) {
            const bool take = (s >= empty_from) || before<POLICY>(dd, jj, d[s], i[s]);
            const float od = d[s];
            const uint32_t oi = i[s];
            d[s] = take ? dd : od;
            i[s] = take ? jj : oi;
            dd = take ? od : dd;
            jj = take ? oi : jj;
        }
        cnt = min(cnt + 1, K - base);
    }

    // Threshold for the hot-loop filter: a candidate with d > kth can never
    // enter (NaN and ties are decided in offer()).  Empty slots hold +inf.
    __device__ __forceinline__ float kth() const { return d[K - 1]; }
    __device__ __forceinline__ bool full() const { return cnt >= K - base; }
};

}  // namespace
}  // namespace mpo
