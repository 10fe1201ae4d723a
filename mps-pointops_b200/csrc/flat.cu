// Offset checks of the flat (ragged) batch layout, run on the device ahead of
// the flat searches.  The reference validates its ptr arrays on the host
// (gamzerA/mps-pointops mps_pointops/_flat_search_mps.py:41-63, raising
// "ptr_x must start at 0 and end at ..." or "... must be nondecreasing ...");
// here the check runs on the stream, the searches that follow skip their work
// when it failed (segments.cuh), and the caller reads the flag.
#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

__global__ void flat_offsets_check_kernel(const int64_t* __restrict__ ptr_q,
                                          const int64_t* __restrict__ ptr_r, int64_t segs,
                                          int64_t M, int64_t N, int32_t* __restrict__ flag) {
    bool bad = false;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= segs;
         b += (int64_t)gridDim.x * blockDim.x) {
        const int64_t q = ptr_q[b], r = ptr_r[b];
        if (b == 0) bad |= q != 0 || r != 0;
        if (b == segs) bad |= q != M || r != N;
        if (b < segs) bad |= ptr_q[b + 1] < q || ptr_r[b + 1] < r;
    }
    if (bad) atomicExch(flag, 1);
}

}  // namespace

int flat_offsets_check(const int64_t* ptr_q, const int64_t* ptr_r, int64_t segs, int64_t M,
                       int64_t N, int32_t* flag, cudaStream_t s) {
    const int threads = 256;
    const int64_t blocks = min64(ceil_div(segs + 1, threads), (int64_t)sm_count() * 4);
    flat_offsets_check_kernel<<<(unsigned)blocks, threads, 0, s>>>(ptr_q, ptr_r, segs, M, N, flag);
    return check_launch("flat_offsets_check_kernel");
}

}  // namespace mpo
