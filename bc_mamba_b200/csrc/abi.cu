// abi.cu — status/error plumbing of the C ABI and cached device queries.
#include <stdarg.h>
#include <mutex>

#include "common.cuh"

namespace bcm {

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int sm_count() {
    // Cached per device; the query is cheap but sits on every launch path.
    // It only sizes grids.  When the device cannot be queried the failure is
    // recorded in the thread's error message and a B200's 148 SMs size the
    // grid; the launch that follows then fails and its check returns the
    // CUDA error as the call's status (a failed query leaves no sticky error).
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess || dev < 0 || dev >= 64) {
        set_error("SM count query: cudaGetDevice failed (%s, device %d)", cudaGetErrorString(err), dev);
        return 148;
    }
    {
        std::lock_guard<std::mutex> lk(mu);
        if (cache[dev]) return cache[dev];
    }
    int n = 0;
    err = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess || n <= 0) {
        set_error("SM count query on device %d failed: %s", dev, cudaGetErrorString(err));
        return 148;   // not cached: the next call queries again
    }
    std::lock_guard<std::mutex> lk(mu);
    cache[dev] = n;
    return n;
}

}  // namespace bcm

extern "C" const char* bcm_last_error(void) { return bcm::g_err; }
extern "C" int bcm_abi_version(void) { return BCM_ABI_VERSION; }
