// Cross-GPU all-reduce of one float per rank over peer memory (CUDA IPC
// mappings, NVLink stores), for the loss of a batch of Chamfer clouds split
// across the GPUs of one node: every rank's loss partial must reach every
// rank, and the sum must carry the same bits on all of them.
//
// Each rank owns one exchange array in its own HBM: 2 banks x kMaxRanks
// 64-bit words, shared with the node's other ranks through CUDA IPC.  At
// reduction number `seq` (a host counter that every rank advances in step,
// never 0) rank r stores the word (seq << 32 | bits(value_r)) into word
// [seq & 1][r] of EVERY rank's array (its own included) -- lane p of one warp
// writes rank p's copy -- and then lane p polls the rank's own array until
// word [seq & 1][p] carries seq.  Lane 0 sums the W values in rank order, so
// every rank obtains the same bits whatever order the words arrived in.  A
// word holds its sequence number and its value in one aligned 64-bit store,
// so it is never seen half written and needs no fence or separate flag.
//
// Two banks make the reuse safe: rank r reaches reduction seq + 2 (the same
// bank as seq) only after its reduction seq + 1 completed, which needed every
// rank's seq + 1 word, which each rank stores only after its own reduction
// seq has read bank seq & 1.
//
// The poll is bounded in real time (%globaltimer, timeout_ns): on expiry the
// kernel writes NaN as the result and 1 + (the lowest rank it did not hear
// from) into *status, and returns.  No trap, no unbounded wait.
#include <cstring>
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {
namespace {

constexpr int kMaxRanks = MPO_P2P_MAX_RANKS;
constexpr size_t kSlotsBytes = 2 * kMaxRanks * sizeof(unsigned long long);
static_assert(kMaxRanks == 32, "one lane per rank");
static_assert(sizeof(cudaIpcMemHandle_t) == MPO_P2P_IPC_HANDLE_BYTES, "IPC handle size");

struct PeerArrays {
    unsigned long long* p[kMaxRanks];
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32) allreduce_scalar_kernel(
    const float* __restrict__ value, float scale, float* __restrict__ out, PeerArrays peers,
    int world, int rank, unsigned seq, unsigned long long timeout_ns, int32_t* __restrict__ status) {
    const int lane = threadIdx.x;
    const int bank = (int)(seq & 1u) * kMaxRanks;
    const float v = __fmul_rn(value[0], scale);
    const unsigned long long word = ((unsigned long long)seq << 32) | __float_as_uint(v);
    if (lane < world) st_relaxed_sys_u64(peers.p[lane] + bank + rank, word);

    float got = 0.f;
    int missing = 0;
    if (lane < world) {
        const unsigned long long* mine = peers.p[rank] + bank + lane;
        unsigned long long w = ld_relaxed_sys_u64(mine);
        if ((unsigned)(w >> 32) != seq) {
            const unsigned long long t0 = globaltimer_ns();
            while ((unsigned)(w >> 32) != seq) {
                if (globaltimer_ns() - t0 > timeout_ns) {
                    missing = 1;
                    break;
                }
                w = ld_relaxed_sys_u64(mine);
            }
        }
        got = __uint_as_float((unsigned)w);
    }
    const unsigned miss = __ballot_sync(FULL_MASK, missing);
    float s = __shfl_sync(FULL_MASK, got, 0);
    for (int r = 1; r < world; ++r) s = __fadd_rn(s, __shfl_sync(FULL_MASK, got, r));
    if (lane == 0) {
        if (miss) {
            out[0] = __int_as_float(0x7fc00000);
            atomicExch(status, 1 + (__ffs((int)miss) - 1));
        } else {
            out[0] = s;
        }
    }
}

int cuda_fail(const char* who, cudaError_t e) {
    return fail(kCudaError, std::string(who) + ": " + cudaGetErrorString(e));
}

}  // namespace
}  // namespace mpo

extern "C" {

size_t mpo_p2p_slots_bytes(void) { return mpo::kSlotsBytes; }

int mpo_p2p_slots_create(void** slots, void* ipc_handle) {
    MPO_REQUIRE(slots != nullptr, "slots is NULL");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, mpo::kSlotsBytes);
    if (e != cudaSuccess) return mpo::cuda_fail("mpo_p2p_slots_create: cudaMalloc", e);
    e = cudaMemset(p, 0, mpo::kSlotsBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess && ipc_handle != nullptr) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, p);
        if (e == cudaSuccess) std::memcpy(ipc_handle, &h, sizeof(h));
    }
    if (e != cudaSuccess) {
        cudaFree(p);
        return mpo::cuda_fail("mpo_p2p_slots_create", e);
    }
    *slots = p;
    return mpo::kOk;
}

int mpo_p2p_slots_open(const void* ipc_handle, void** peer_slots) {
    MPO_REQUIRE(ipc_handle != nullptr && peer_slots != nullptr,
                "ipc_handle and peer_slots must not be NULL");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return mpo::cuda_fail("mpo_p2p_slots_open: cudaIpcOpenMemHandle", e);
    *peer_slots = p;
    return mpo::kOk;
}

int mpo_p2p_slots_close(void* peer_slots) {
    MPO_REQUIRE(peer_slots != nullptr, "peer_slots is NULL");
    const cudaError_t e = cudaIpcCloseMemHandle(peer_slots);
    if (e != cudaSuccess) return mpo::cuda_fail("mpo_p2p_slots_close: cudaIpcCloseMemHandle", e);
    return mpo::kOk;
}

int mpo_p2p_slots_destroy(void* slots) {
    MPO_REQUIRE(slots != nullptr, "slots is NULL");
    const cudaError_t e = cudaFree(slots);
    if (e != cudaSuccess) return mpo::cuda_fail("mpo_p2p_slots_destroy: cudaFree", e);
    return mpo::kOk;
}

int mpo_allreduce_sum_f32_p2p(const float* value, float scale, float* out, void* const* slots,
                              int64_t world, int64_t rank, uint32_t seq, int64_t timeout_ns,
                              int32_t* status, void* stream) {
    MPO_REQUIRE(value != nullptr && out != nullptr && slots != nullptr && status != nullptr,
                "value, out, slots and status must not be NULL");
    MPO_REQUIRE(world >= 1 && world <= mpo::kMaxRanks,
                "world must be in [1, " + std::to_string(mpo::kMaxRanks) + "]");
    MPO_REQUIRE(rank >= 0 && rank < world, "rank must be in [0, world)");
    MPO_REQUIRE(seq != 0u, "seq must not be 0 (fresh arrays hold zeros)");
    MPO_REQUIRE(timeout_ns > 0, "timeout_ns must be positive");
    mpo::PeerArrays peers{};
    for (int64_t r = 0; r < world; ++r) {
        MPO_REQUIRE(slots[r] != nullptr && mpo::aligned_to(slots[r], 8),
                    "slots[" + std::to_string((long long)r) +
                        "] must be a non-NULL 8-byte aligned device pointer");
        peers.p[r] = static_cast<unsigned long long*>(slots[r]);
    }
    mpo::allreduce_scalar_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        value, scale, out, peers, (int)world, (int)rank, seq, (unsigned long long)timeout_ns,
        status);
    return mpo::check_launch("allreduce_scalar_kernel");
}

}  // extern "C"
