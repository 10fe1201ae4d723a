// Library-wide C-ABI entry points: version, last error, device queries.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/mpo_b200.h"
#include "mpo_common.cuh"

namespace mpo {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void set_last_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(kCudaError, std::string(what) + ": " + cudaGetErrorString(e));
    }
    return kOk;
}

int current_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev;
}

int sm_count(int device) {
    static std::mutex mu;
    static int cache[64] = {0};
    if (device < 0) device = current_device();
    if (device >= 64) device = 63;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[device] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
            n <= 0) {
            n = 148;
        }
        cache[device] = n;
    }
    return cache[device];
}

}  // namespace mpo

extern "C" {

int32_t mpo_abi_version(void) { return MPO_ABI_VERSION; }

const char* mpo_last_error(void) { return mpo::g_last_error.c_str(); }

uint64_t mpo_launch_count(void) { return mpo::g_launches.load(std::memory_order_relaxed); }

int mpo_device_supported(int device) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        return mpo::fail(mpo::kCudaError, "mpo_device_supported: cannot query device");
    }
    if (prop.major != 10 || prop.minor != 0) {
        char buf[160];
        snprintf(buf, sizeof(buf),
                 "mpo_device_supported: device %d is sm_%d%d; this library is built for sm_100a "
                 "(B200) only",
                 device, prop.major, prop.minor);
        return mpo::fail(mpo::kUnsupported, buf);
    }
    return mpo::kOk;
}

}  // extern "C"
