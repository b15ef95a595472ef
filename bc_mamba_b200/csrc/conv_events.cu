// conv_events.cu — the causal depthwise convolution + SiLU that feeds the
// event gather, evaluated only where events are.
//
// The reference computes x_conv = silu(conv1d(x))[..., :L] densely over
// (B, D, L) (spike_mamba/e_model.py:306-313, 442-451; causal_conv1d or
// nn.Conv1d with padding K-1, groups = D) and then gathers it at the events
// (GatherEventsFn, e_model.py:167-193); nothing else reads x_conv.  Here:
//   forward   u[e] = silu(bias[d] + sum_j w[d,j] * x[b,d,t_e-K+1+j])
//             (zero padding before position 0), one thread per event;
//   backward  dpre[e] = g[e] * silu'(pre[e]);
//             dx[b,d,tau] = sum_j w[d,j] * dpre(event at tau+K-1-j)  (dense,
//             zero where no event reaches), dw[d,j] = sum_e dpre*x[..],
//             dbias[d] = sum_e dpre.
// Backward layout: one warp per channel row walks the row in chunks of kCH
// positions; the chunk's x window and the dpre of the events that reach it
// are staged in shared memory, the dense dx chunk is written with coalesced
// stores, and weight/bias gradients are per-channel partials reduced over the
// batch rows of each feature in a fixed order (deterministic).
#include "common.cuh"

namespace bcm {
namespace {

constexpr int kMaxK = 8;     // longest supported kernel (the model uses 4)
constexpr int kCH = 256;     // positions per chunk (backward)
constexpr int kCW = 4;       // warps per CTA (backward)

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

template <typename T>
__global__ void conv_events_fwd_kernel(const T* __restrict__ x, int64_t n_ch, int D, int L,
                                       const float* __restrict__ w, const float* __restrict__ bias, int K,
                                       const int32_t* __restrict__ ch, const int32_t* __restrict__ ts,
                                       int64_t n_events, T* __restrict__ out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_events; e += stride) {
        const int c = ch[e], t = ts[e];
        float y = 0.f;
        if (c >= 0 && c < n_ch && t >= 0 && t < L) {
            const int d = c % D;
            const T* xr = x + (int64_t)c * L;
            float acc = bias ? bias[d] : 0.f;
            for (int j = 0; j < K; ++j) {
                const int tt = t - (K - 1) + j;
                if (tt >= 0) acc = fmaf(w[d * K + j], to_f32<T>(xr[tt]), acc);
            }
            y = acc * sigmoidf_(acc);
        }
        out[e] = from_f32<T>(y);
    }
}

template <typename T>
__global__ void __launch_bounds__(kCW * 32)
conv_events_bwd_kernel(const T* __restrict__ x, int64_t n_ch, int D, int L, const float* __restrict__ w,
                       const float* __restrict__ bias, int K, const int32_t* __restrict__ ts,
                       const int32_t* __restrict__ cu, const T* __restrict__ g, T* __restrict__ dx,
                       float* __restrict__ part) {
    __shared__ float s_x[kCW][kCH + 2 * kMaxK];     // x[c0-K+1 .. c0+kCH+K-2]
    __shared__ float s_dp[kCW][kCH + kMaxK];        // dpre by position t - c0
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t c = (int64_t)blockIdx.x * kCW + warp;
    if (c >= n_ch) return;
    const int d = (int)(c % D);
    float wj[kMaxK];
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) wj[j] = (j < K) ? w[d * K + j] : 0.f;
    const float bv = bias ? bias[d] : 0.f;
    const T* xr = x + c * L;
    T* dxr = dx + c * L;
    const int beg = cu[c], end = cu[c + 1];
    float* sx = s_x[warp];
    float* sdp = s_dp[warp];
    float dw[kMaxK];
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) dw[j] = 0.f;
    float db = 0.f;
    int ep = beg;                                   // first event at or after c0
    for (int c0 = 0; c0 < L; c0 += kCH) {
        const int hi = c0 + kCH + K - 1;            // events before hi reach this chunk
        for (int i = lane; i < kCH + 2 * K - 2; i += 32) {
            const int tt = c0 - K + 1 + i;
            sx[i] = (tt >= 0 && tt < L) ? to_f32<T>(xr[tt]) : 0.f;
        }
        for (int i = lane; i < kCH + K - 1; i += 32) sdp[i] = 0.f;
        __syncwarp();
        int owned = 0;                              // events with t < c0 + kCH (this chunk's)
        for (int e0 = ep; e0 < end; e0 += 32) {
            const int e = e0 + lane;
            const int t = (e < end) ? ts[e] : INT_MAX;
            const bool in = t >= c0 && t < hi && t < L;
            if (in) {
                const int r = t - c0;               // x window index of x[t-K+1] is r
                float pre = bv;
                for (int j = 0; j < K; ++j) pre = fmaf(wj[j], sx[r + j], pre);
                const float s = sigmoidf_(pre);
                const float dp = to_f32<T>(g[e]) * s * (1.0f + pre * (1.0f - s));
                sdp[r] = dp;
                if (t < c0 + kCH) {                 // owned: weight / bias gradients once
#pragma unroll
                    for (int j = 0; j < kMaxK; ++j)
                        if (j < K) dw[j] = fmaf(dp, sx[r + j], dw[j]);
                    db += dp;
                }
            }
            owned += __popc(__ballot_sync(kFull, e < end && t < c0 + kCH));
            if (__any_sync(kFull, e >= end || t >= hi)) break;
        }
        ep += owned;
        __syncwarp();
        for (int i = lane; i < kCH; i += 32) {
            const int tau = c0 + i;
            if (tau < L) {
                float v = 0.f;
                for (int j = 0; j < K; ++j) v = fmaf(wj[j], sdp[i + K - 1 - j], v);
                dxr[tau] = from_f32<T>(v);
            }
        }
        __syncwarp();
    }
    // per-channel partials (lanes hold different events)
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
        float v = dw[j];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
        if (lane == 0 && j < K) part[c * (K + 1) + j] = v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) db += __shfl_xor_sync(kFull, db, off);
    if (lane == 0) part[c * (K + 1) + K] = db;
}

// dweight[d, j] / dbias[d] = sum over batch rows b (in order) of the partials
// of channel b*D + d.
__global__ void conv_events_reduce_kernel(const float* __restrict__ part, int64_t B, int D, int K,
                                          float* __restrict__ dw, float* __restrict__ db) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // (d, j) with j == K the bias
    if (i >= D * (K + 1)) return;
    const int d = i / (K + 1), j = i % (K + 1);
    float s = 0.f;
    for (int64_t b = 0; b < B; ++b) s += part[(b * D + d) * (K + 1) + j];
    if (j < K) dw[d * K + j] = s;
    else if (db) db[d] = s;
}

}  // namespace
}  // namespace bcm

using namespace bcm;

extern "C" bcm_status bcm_conv_events_fwd(const void* x, bcm_dtype dtype, int64_t batch, int64_t dim,
                                          int64_t seqlen, const float* weight, const float* bias,
                                          int64_t kernel_size, const int32_t* channel_ids,
                                          const int32_t* time_steps, int64_t n_events, void* out,
                                          cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "conv_events_fwd: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(batch >= 0 && dim >= 1 && seqlen >= 0 && n_events >= 0, "conv_events_fwd: bad sizes");
    BCM_REQUIRE(kernel_size >= 1 && kernel_size <= kMaxK, "conv_events_fwd: kernel_size must be in [1, %d]",
                kMaxK);
    BCM_REQUIRE(seqlen < (1ll << 31), "conv_events_fwd: seqlen too large");
    if (n_events == 0) return BCM_OK;
    BCM_REQUIRE(x && weight && channel_ids && time_steps && out, "conv_events_fwd: null pointer");
    const int threads = 256;
    const int64_t want = (n_events + threads - 1) / threads;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * 16));
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        conv_events_fwd_kernel<T><<<grid, threads, 0, stream>>>(
            static_cast<const T*>(x), batch * dim, (int)dim, (int)seqlen, weight, bias, (int)kernel_size,
            channel_ids, time_steps, n_events, static_cast<T*>(out));
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}

extern "C" size_t bcm_conv_events_bwd_workspace_bytes(int64_t n_channels, int64_t kernel_size) {
    if (n_channels < 0 || kernel_size < 1) return 0;
    return align_up((size_t)n_channels * (size_t)(kernel_size + 1) * sizeof(float), 256);
}

extern "C" bcm_status bcm_conv_events_bwd(const void* x, bcm_dtype dtype, int64_t batch, int64_t dim,
                                          int64_t seqlen, const float* weight, const float* bias,
                                          int64_t kernel_size, const int32_t* time_steps,
                                          const int32_t* cu_seqlens, int64_t n_events, const void* grad,
                                          void* dx, float* dweight, float* dbias, void* workspace,
                                          size_t workspace_bytes, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "conv_events_bwd: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(batch >= 0 && dim >= 1 && seqlen >= 0 && n_events >= 0, "conv_events_bwd: bad sizes");
    BCM_REQUIRE(kernel_size >= 1 && kernel_size <= kMaxK, "conv_events_bwd: kernel_size must be in [1, %d]",
                kMaxK);
    BCM_REQUIRE(seqlen < (1ll << 31), "conv_events_bwd: seqlen too large");
    const int64_t NC = batch * dim;
    BCM_REQUIRE(dweight && (NC * seqlen == 0 || dx), "conv_events_bwd: null output");
    if (NC == 0 || seqlen == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(dweight, 0, sizeof(float) * dim * kernel_size, stream));
        if (dbias) BCM_CUDA_TRY(cudaMemsetAsync(dbias, 0, sizeof(float) * dim, stream));
        return BCM_OK;
    }
    BCM_REQUIRE(x && weight && cu_seqlens && (n_events == 0 || (time_steps && grad)),
                "conv_events_bwd: null pointer");
    const size_t need = bcm_conv_events_bwd_workspace_bytes(NC, kernel_size);
    if (!workspace || workspace_bytes < need) {
        set_error("conv_events_bwd: workspace of %zu bytes < required %zu", workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    float* part = static_cast<float*>(workspace);
    const int64_t blocks = (NC + kCW - 1) / kCW;
    BCM_REQUIRE(blocks < (1ll << 31), "conv_events_bwd: too many channels");
    bcm_status st = dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        conv_events_bwd_kernel<T><<<(unsigned)blocks, kCW * 32, 0, stream>>>(
            static_cast<const T*>(x), NC, (int)dim, (int)seqlen, weight, bias, (int)kernel_size, time_steps,
            cu_seqlens, static_cast<const T*>(grad), static_cast<T*>(dx), part);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
    if (st != BCM_OK) return st;
    const int n = (int)(dim * (kernel_size + 1));
    conv_events_reduce_kernel<<<(n + 255) / 256, 256, 0, stream>>>(part, batch, (int)dim, (int)kernel_size,
                                                                   dweight, dbias);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}
