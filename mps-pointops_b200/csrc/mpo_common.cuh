// Shared device helpers and host error plumbing for libmpo_b200.
//
// Arithmetic contract: every squared distance is formed with explicitly
// rounded single-precision intrinsics (__fsub_rn / __fmul_rn / __fadd_rn),
// which nvcc never contracts into an FMA, in the reference's order:
//   D == 3 : ((d0*d0 + d1*d1) + d2*d2),   d = a - b
//   D != 3 : s = d0*d0; s = s + dt*dt for t = 1 .. D-1
// (gamzerA/mps-pointops mps_pointops/reference.py:21-24, chamfer.py:199-201).
// The library is also compiled with -fmad=false so no other float expression
// is contracted either.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace mpo {

constexpr unsigned FULL_MASK = 0xffffffffu;

// ------------------------------------------------------------------ errors
// Status codes returned by every C-ABI entry point (see include/mpo_b200.h).
enum Status : int {
    kOk = 0,
    kInvalidArgument = 1,
    kCudaError = 2,
    kUnsupported = 3,
    kWorkspaceTooSmall = 4,
};

void set_last_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);  // also counts one kernel launch
void count_launches(uint64_t n);
int sm_count(int device = -1);

// Tensor-core feature kNN (feature_knn_tc.cu).
bool fknn_tc_eligible(int64_t M, int64_t N, int64_t D, int64_t k);
size_t fknn_tc_workspace_bytes(int64_t B, int64_t M, int64_t N, int64_t D);
int fknn_tc_run(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int64_t D,
                int64_t k, float* dist, int64_t* idx, float* sqdist, void* workspace,
                size_t workspace_bytes, cudaStream_t s);
int current_device();

// Flat (ragged) batches (flat.cu): one launch checks that ptr_q[0..segs] runs
// from 0 to M and ptr_r[0..segs] from 0 to N without decreasing, and sets
// *flag = 1 otherwise (the caller zeroes the flag first, on the same stream).
int flat_offsets_check(const int64_t* ptr_q, const int64_t* ptr_r, int64_t segs, int64_t M,
                       int64_t N, int32_t* flag, cudaStream_t s);

#define MPO_REQUIRE(cond, msg)                                   \
    do {                                                         \
        if (!(cond)) return ::mpo::fail(::mpo::kInvalidArgument, \
                                        std::string(__func__) + ": " + (msg)); \
    } while (0)

// Address alignment of a caller's buffer.  Kernels read a float array with
// 16-byte vector loads only when its base is 16-byte aligned (a contiguous
// tensor view can start at any 4-byte offset); workspaces must be 256-byte
// aligned, as cudaMalloc and the torch allocator return them, because the
// kernels place 64-bit atomics and bulk-copy sources at fixed offsets in them.
inline bool aligned_to(const void* p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}
#define MPO_REQUIRE_WORKSPACE(ws) \
    MPO_REQUIRE((ws) == nullptr || ::mpo::aligned_to((ws), 256), "workspace must be 256-byte aligned")

// ------------------------------------------------------------------ math
__device__ __forceinline__ float sqd3(float ax, float ay, float az, float bx, float by,
                                      float bz) {
    const float dx = __fsub_rn(ax, bx);
    const float dy = __fsub_rn(ay, by);
    const float dz = __fsub_rn(az, bz);
    return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

// Sequential D-dimensional squared distance, a and b in registers or memory.
__device__ __forceinline__ float sqd_seq(const float* a, const float* b, int D) {
    float d = __fsub_rn(a[0], b[0]);
    float s = __fmul_rn(d, d);
    for (int t = 1; t < D; ++t) {
        d = __fsub_rn(a[t], b[t]);
        s = __fadd_rn(s, __fmul_rn(d, d));
    }
    return s;
}

// Packed pairs of floats (PTX .f32x2, sm_100): two lanes of IEEE binary32
// arithmetic per instruction, each rounded to nearest on its own -- the same
// bits as two scalar __fsub_rn / __fmul_rn / __fadd_rn.  On B200 one packed
// instruction holds the FP32 pipe for two cycles: it halves the issue slots,
// not the pipe time, of the scalar form.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// a*b + c for both lanes, one rounding each (fmaf on two lanes).
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// Rounded square of both lanes, d*d.  ptxas contracts mul.rn.f32x2 followed
// by add.rn.f32x2 into a fused f32x2 FMA even under -fmad=false, which would
// change the low bit of about one squared distance in five.  The square is
// therefore written as fma.rn(d, d, +0.0): for a square (never -0) this is
// exactly the rounded product, and because fma(a, b, +0) differs from a*b
// when a*b is -0, the optimizer cannot rewrite it into a multiply and then
// contract it with the following add.
__device__ __forceinline__ f32x2 sq2(f32x2 d) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %1, %2;" : "=l"(r) : "l"(d), "l"(0ull));
    return r;
}
// ((dx*dx + dy*dy) + dz*dz) for two (a, b) pairs at once; bit-identical to
// two scalar sqd3() calls.
__device__ __forceinline__ f32x2 sqd3x2(f32x2 ax, f32x2 ay, f32x2 az, f32x2 bx, f32x2 by,
                                        f32x2 bz) {
    const f32x2 dx = sub2(ax, bx);
    const f32x2 dy = sub2(ay, by);
    const f32x2 dz = sub2(az, bz);
    return add2(add2(sq2(dx), sq2(dy)), sq2(dz));
}

// 16-byte shared-memory load of two packed pairs from a 32-bit shared-window
// address plus a compile-time byte offset (one base register per loop
// instead of 64-bit generic pointer arithmetic per load).
template <int OFF>
__device__ __forceinline__ void lds_pairs(uint32_t addr, f32x2& lo, f32x2& hi) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2+%3];" : "=l"(lo), "=l"(hi) : "r"(addr), "n"(OFF));
}

// NaN-propagating minimum (torch.minimum semantics): PTX min.NaN.f32.
__device__ __forceinline__ float fmin_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Monotone map of a float onto uint32 (larger float -> larger key) for
// argmax reductions.  -inf maps near 0, +inf to 0xff800000; NaN is mapped by
// callers that need it.
__device__ __forceinline__ uint32_t ordered_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float ordered_key_inv(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// Acquire / relaxed global loads used by the bounded spin waits.
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Nanosecond wall clock of the GPU, for bounding spin waits in real time.
__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) {
    return (a + b - 1) / b;
}
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

}  // namespace mpo
