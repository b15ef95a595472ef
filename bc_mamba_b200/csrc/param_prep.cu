// param_prep.cu — the event block's parameter transforms in one launch per
// direction: A = -exp(A_log), W_B / W_C = the two halves of W_BC, dt_idle /
// dt_active = softplus(a0 / a1) + eps (reference spike_mamba/e_model.py:
// 210-230 TwoLevelDelta, :321-334, :463, :475-476), and their backward.  In
// PyTorch these are eight small kernels and as many autograd nodes per block
// and direction; fused, the host enqueues one launch each way, which matters
// when a step is short enough for host time to set its pace (a batch sharded
// over many GPUs).  softplus follows torch.nn.functional.softplus (beta 1,
// identity above 20); its derivative is exp(x) / (exp(x) + 1) below.
#include <algorithm>

#include "common.cuh"

namespace bcm {
namespace {

__device__ __forceinline__ float softplus_t(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) {
    const float z = expf(x);
    return x > 20.f ? 1.f : z / (z + 1.f);
}

__global__ void params_fwd_kernel(const float* __restrict__ A_log, const float* __restrict__ W_BC,
                                  const float* __restrict__ a0, const float* __restrict__ a1, int dim, int N,
                                  float eps, float* __restrict__ A, float* __restrict__ W_B,
                                  float* __restrict__ W_C, float* __restrict__ dt_idle, float* __restrict__ dt_active) {
    const int64_t total = (int64_t)dim * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = i / N, s = i % N;
        A[i] = -expf(A_log[i]);
        W_B[i] = W_BC[d * 2 * N + s];
        W_C[i] = W_BC[d * 2 * N + N + s];
        if (s == 0) {
            dt_idle[d] = softplus_t(a0[d]) + eps;
            dt_active[d] = softplus_t(a1[d]) + eps;
        }
    }
}

__global__ void params_bwd_kernel(const float* __restrict__ A, const float* __restrict__ a0,
                                  const float* __restrict__ a1, const float* __restrict__ dA,
                                  const float* __restrict__ dW_B, const float* __restrict__ dW_C,
                                  const float* __restrict__ ddt_idle, const float* __restrict__ ddt_active, int dim,
                                  int N, float* __restrict__ dA_log, float* __restrict__ dW_BC,
                                  float* __restrict__ da0, float* __restrict__ da1) {
    const int64_t total = (int64_t)dim * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = i / N, s = i % N;
        // d(-exp(x))/dx = -exp(x) = A
        dA_log[i] = dA ? dA[i] * A[i] : 0.f;
        dW_BC[d * 2 * N + s] = dW_B ? dW_B[i] : 0.f;
        dW_BC[d * 2 * N + N + s] = dW_C ? dW_C[i] : 0.f;
        if (s == 0) {
            da0[d] = ddt_idle ? ddt_idle[d] * softplus_grad(a0[d]) : 0.f;
            da1[d] = ddt_active ? ddt_active[d] * softplus_grad(a1[d]) : 0.f;
        }
    }
}

int prep_grid(int64_t total) {
    const int64_t blocks = (total + 255) / 256;
    return (int)std::min<int64_t>(std::max<int64_t>(blocks, 1), 1024);
}

}  // namespace
}  // namespace bcm

using namespace bcm;

extern "C" bcm_status bcm_event_params_fwd(const float* A_log, const float* W_BC, const float* a0, const float* a1,
                                           int64_t dim, int64_t dstate, float eps, float* A, float* W_B,
                                           float* W_C, float* dt_idle, float* dt_active, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dim >= 1 && dstate >= 1 && dim * dstate < (1ll << 31), "event_params_fwd: bad sizes");
    BCM_REQUIRE(A_log && W_BC && a0 && a1 && A && W_B && W_C && dt_idle && dt_active,
                "event_params_fwd: null pointer");
    params_fwd_kernel<<<prep_grid(dim * dstate), 256, 0, stream>>>(A_log, W_BC, a0, a1, (int)dim, (int)dstate, eps,
                                                                   A, W_B, W_C, dt_idle, dt_active);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

extern "C" bcm_status bcm_event_params_bwd(const float* A, const float* a0, const float* a1, const float* dA,
                                           const float* dW_B, const float* dW_C, const float* ddt_idle,
                                           const float* ddt_active, int64_t dim, int64_t dstate, float* dA_log,
                                           float* dW_BC, float* da0, float* da1, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dim >= 1 && dstate >= 1 && dim * dstate < (1ll << 31), "event_params_bwd: bad sizes");
    BCM_REQUIRE(A && a0 && a1 && dA_log && dW_BC && da0 && da1, "event_params_bwd: null pointer");
    params_bwd_kernel<<<prep_grid(dim * dstate), 256, 0, stream>>>(A, a0, a1, dA, dW_B, dW_C, ddt_idle, ddt_active,
                                                                   (int)dim, (int)dstate, dA_log, dW_BC, da0, da1);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}
