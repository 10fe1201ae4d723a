// Batch layouts shared by the search kernels: dense batches of equal-size
// clouds and the flat (ragged) batches of the torch_cluster API, whose
// sorted segments are given by offset arrays (gamzerA/mps-pointops
// mps_pointops/flat.py:67-97: ptr[b] = first row of segment b, ptr[B] = the
// row count).
//
// A search kernel processes a tile of `qpc` consecutive query rows per CTA,
// all of one segment, against that segment's reference rows.
//   * Dense: grid (ceil(M / qpc), B); CTA (t, b) takes rows t*qpc .. of cloud
//     b, and reports local reference indices.
//   * Flat: a 1-D grid of "virtual tiles".  Segment b owns the tiles
//     [start(b), start(b + 1)) with start(b) = floor(ptr_q[b] / qpc) + b.
//     start() is strictly increasing and
//         start(b + 1) - start(b) = floor(ptr_q[b+1]/qpc) - floor(ptr_q[b]/qpc) + 1
//                                 >= ceil((ptr_q[b+1] - ptr_q[b]) / qpc),
//     so every segment has enough tiles and the grid needs at most
//     floor(M / qpc) + B + 1 CTAs: no host-side scan of the offsets and no
//     extra launch.  A CTA finds its segment by binary search over ptr_q and
//     exits when its tile lies past the segment's last query.  Reference
//     indices are reported globally (ptr_r[b] + local index).
#pragma once

#include "mpo_common.cuh"

namespace mpo {
namespace {

// The rows one CTA works on.
struct Span {
    int64_t q0, q1;  // query rows [q0, q1), global
    int64_t r0, n;   // reference rows [r0, r0 + n), global
    int64_t obase;   // added to a local reference index on output
};

// Layout of one search launch (passed by value).
struct Layout {
    int64_t M, N;            // dense: rows per cloud; flat: total query / reference rows
    const int64_t* ptr_q;    // flat: (segs + 1) query offsets, else null
    const int64_t* ptr_r;    // flat: (segs + 1) reference offsets, else null
    int64_t segs;            // flat: segment count
    const int32_t* invalid;  // flat: nonzero once the offset check failed (nullable)
};

inline Layout dense_layout(int64_t M, int64_t N) { return Layout{M, N, nullptr, nullptr, 0, nullptr}; }

inline int64_t flat_tiles(int64_t M, int64_t segs, int qpc) { return M / qpc + segs + 1; }

template <bool FLAT>
__device__ __forceinline__ bool locate(const Layout& L, int qpc, Span& sp) {
    if (!FLAT) {
        const int64_t b = blockIdx.y;
        sp.q0 = b * L.M + (int64_t)blockIdx.x * qpc;
        sp.q1 = min64(b * L.M + L.M, sp.q0 + qpc);
        sp.r0 = b * L.N;
        sp.n = L.N;
        sp.obase = 0;
        return true;
    }
    if (L.segs <= 0 || (L.invalid != nullptr && *L.invalid != 0)) return false;
    const int64_t t = blockIdx.x;
    // Last segment b with start(b) <= t (start(0) = 0 <= t).
    int64_t lo = 0, hi = L.segs - 1;
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (L.ptr_q[mid] / qpc + mid <= t) lo = mid;
        else hi = mid - 1;
    }
    const int64_t qa = L.ptr_q[lo], qb = L.ptr_q[lo + 1];
    const int64_t ra = L.ptr_r[lo], rb = L.ptr_r[lo + 1];
    // The offsets were checked by flat_offsets_check_kernel earlier on the
    // stream; these bounds keep every access inside the arrays regardless.
    if (!(0 <= qa && qa <= qb && qb <= L.M && 0 <= ra && ra <= rb && rb <= L.N)) return false;
    sp.q0 = qa + (t - (qa / qpc + lo)) * (int64_t)qpc;
    if (sp.q0 >= qb) return false;
    sp.q1 = min64(qb, sp.q0 + qpc);
    sp.r0 = ra;
    sp.n = rb - ra;
    sp.obase = ra;
    return true;
}

}  // namespace
}  // namespace mpo
