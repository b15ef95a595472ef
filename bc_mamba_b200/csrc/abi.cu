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
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (cache[dev]) return cache[dev];
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    std::lock_guard<std::mutex> lk(mu);
    cache[dev] = n;
    return n;
}

}  // namespace bcm

extern "C" const char* bcm_last_error(void) { return bcm::g_err; }
extern "C" int bcm_abi_version(void) { return BCM_ABI_VERSION; }
