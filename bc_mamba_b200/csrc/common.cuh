// common.cuh — helpers shared by every kernel of libbcm_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "bcm_b200.h"

namespace bcm {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ---- thread-local error text (read back through bcm_last_error) ----------
void set_error(const char* fmt, ...);
void clear_error();

#define BCM_REQUIRE(cond, ...)                                   \
    do {                                                         \
        if (!(cond)) {                                           \
            ::bcm::set_error(__VA_ARGS__);                       \
            return BCM_ERR_INVALID_ARGUMENT;                     \
        }                                                        \
    } while (0)

#define BCM_CUDA_TRY(expr)                                                   \
    do {                                                                     \
        cudaError_t err__ = (expr);                                          \
        if (err__ != cudaSuccess) {                                          \
            ::bcm::set_error("%s failed: %s (%s:%d)", #expr,                 \
                             cudaGetErrorString(err__), __FILE__, __LINE__); \
            return BCM_ERR_CUDA;                                             \
        }                                                                    \
    } while (0)

#define BCM_LAUNCH_CHECK() BCM_CUDA_TRY(cudaGetLastError())

// ---- element conversion ---------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<double>(double v) { return (float)v; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ double from_f32<double>(float v) { return (double)v; }

inline size_t dtype_size(bcm_dtype t) { return t == BCM_F64 ? 8 : (t == BCM_F32 ? 4 : 2); }
inline bool dtype_ok(bcm_dtype t) { return t == BCM_F32 || t == BCM_F16 || t == BCM_BF16; }
inline bool dtype_ok64(bcm_dtype t) { return dtype_ok(t) || t == BCM_F64; }

// Dispatch a functor templated on the element type.
template <typename F>
bcm_status dispatch_dtype(bcm_dtype t, F&& f) {
    switch (t) {
        case BCM_F32: return f(float{});
        case BCM_F16: return f(__half{});
        case BCM_BF16: return f(__nv_bfloat16{});
    }
    set_error("unsupported dtype %d", (int)t);
    return BCM_ERR_INVALID_ARGUMENT;
}

// Same, with double added (extraction input and gather only).
template <typename F>
bcm_status dispatch_dtype64(bcm_dtype t, F&& f) {
    if (t == BCM_F64) return f(double{});
    return dispatch_dtype(t, f);
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- device info (cached per device, thread-safe after first call) -------
int sm_count();

// ---- warp helpers -----------------------------------------------------------
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

template <typename T>
__device__ __forceinline__ T warp_inclusive_sum(T v) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        T o = __shfl_up_sync(kFull, v, off);
        if (lane_id() >= off) v += o;
    }
    return v;
}

__device__ __forceinline__ int warp_inclusive_max(int v) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int o = __shfl_up_sync(kFull, v, off);
        if (lane_id() >= off) v = max(v, o);
    }
    return v;
}

// Exact-semantics decay factor of one event for one state:
// exp2(clamp(delta*A*log2e, -126, 126)); A2 = A*log2e is pre-multiplied.
__device__ __forceinline__ float decay(float delta, float A2) {
    float e = fmaxf(fminf(delta * A2, 126.0f), -126.0f);
    return exp2f(e);
}

}  // namespace bcm
