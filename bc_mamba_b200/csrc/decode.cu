// decode.cu — the event path one token at a time (the model's decode step).
//
// The reference's step (spike_mamba/e_model.py:508-568) cannot run as written
// (it reads self.pw_B / self.pw_C, which Mamba does not define) and, as
// written, would update every channel at every token with a per-token dt.
// The decode here is defined instead as the training path evaluated one
// token at a time, so that a model decodes exactly what its forward computes:
// for channel c = b*D + d at token t,
//   spike  = spikes[b, d / expand] > threshold   (extraction's compare,
//            extract_events_cuda.cu:117-179)
//   k      = tokens since the channel's previous event (t + 1 for the first)
//   at a spike:  delta = dt_idle*(k-1) + dt_active, a_s = exp2(clamp(delta*A_s*log2e, +-126)),
//                eta_s = a_s*eta_s + delta*u^2,  y = D*u + u*sum_s W_B*W_C*eta_s
//                (the normalised depthwise scan of the flat-channel forward)
//   output: y of the channel's latest event among its first 4095 (the
//           restore's hold and search cap), 0 before its first event.
// The decay, the update and the output sum are formed exactly as the staged
// forward kernel forms them (same correctly rounded exp2, same FMA order,
// same four partial sums), so the decoded outputs equal the forward's
// restored outputs bit for bit.  With a conv state the token's x also passes
// the causal depthwise conv + SiLU first (e_model.py:512-518): the state
// holds the last K inputs of each channel and is rolled in place.
//
// One thread per channel: a token is ~B*D*N multiply-adds, latency bound.
#include "scan_common.cuh"

namespace bcm {
namespace {

constexpr int kDecodeThreads = 128;
constexpr int kDecodeMaxK = 8;
constexpr int kRestoreCap = 4095;   // addressable events of a channel in the batch restore

struct DecodeArgs {
    const void* x;           // [B, D] this token's input (conv input if conv_state, else u)
    const void* spikes;      // [B, d_model]
    int64_t n_ch;            // B * D
    int D, d_model, expand, N, K;
    float threshold;
    const float* dt_idle; const float* dt_active;
    const float* A; int64_t A_sd, A_sn;
    const float* W_B; const float* W_C; const float* Dskip;
    void* conv_state; const float* conv_w; const float* conv_b;
    float* eta; int32_t* counters; float* held;
    void* y;
};

__device__ __forceinline__ float sigmoid_(float v) { return 1.0f / (1.0f + expf(-v)); }

template <typename T>
__global__ void __launch_bounds__(kDecodeThreads) event_decode_kernel(DecodeArgs a) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= a.n_ch) return;
    const int64_t b = c / a.D;
    const int d = (int)(c % a.D);
    float u;
    if (a.conv_state != nullptr) {   // roll the conv state, then conv + SiLU
        T* cs = static_cast<T*>(a.conv_state) + c * a.K;
        for (int j = 0; j + 1 < a.K; ++j) cs[j] = cs[j + 1];
        cs[a.K - 1] = static_cast<const T*>(a.x)[c];
        float acc = a.conv_b ? a.conv_b[d] : 0.f;
        for (int j = 0; j < a.K; ++j) acc = fmaf(a.conv_w[d * a.K + j], to_f32<T>(cs[j]), acc);
        u = to_f32<T>(from_f32<T>(acc * sigmoid_(acc)));
    } else {
        u = to_f32<T>(static_cast<const T*>(a.x)[c]);
    }
    const float sv = to_f32<T>(static_cast<const T*>(a.spikes)[b * a.d_model + d / a.expand]);
    int32_t* cnt = a.counters + 2 * c;   // {tokens since the last event, events so far}
    const int k = cnt[0] + 1;
    float out = a.held[c];
    if (sv > a.threshold) {
        const float dl = event_delta(a.dt_idle[d], a.dt_active[d], k);
        const float w = dl * u * u;
        float* eta = a.eta + c * a.N;
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < a.N; ++s) {
            const float A2 = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
            const float e = fmaf(decay_exact(dl, A2), eta[s], w);
            eta[s] = e;
            s4[s & 3] = fmaf(a.W_B[d * a.N + s] * a.W_C[d * a.N + s], e, s4[s & 3]);
        }
        const float acc = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        const float yv = fmaf(a.Dskip ? a.Dskip[d] : 0.f, u, u * acc);
        cnt[0] = 0;
        const int n_ev = cnt[1] + 1;
        cnt[1] = n_ev;
        if (n_ev <= kRestoreCap) {
            out = to_f32<T>(from_f32<T>(yv));
            a.held[c] = out;
        }
    } else {
        cnt[0] = k;
    }
    static_cast<T*>(a.y)[c] = from_f32<T>(out);
}

}  // namespace
}  // namespace bcm

using namespace bcm;

extern "C" bcm_status bcm_event_decode_step(const void* x, const void* spikes, bcm_dtype dtype, int64_t batch,
                                            int64_t dim, int64_t d_model, int64_t dstate, float threshold,
                                            const float* dt_idle, const float* dt_active, const float* A,
                                            int64_t A_stride_d, int64_t A_stride_n, const float* W_B,
                                            const float* W_C, const float* D, void* conv_state,
                                            const float* conv_weight, const float* conv_bias,
                                            int64_t kernel_size, float* eta, int32_t* counters, float* held,
                                            void* y, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "event_decode_step: unsupported dtype");
    BCM_REQUIRE(batch >= 0 && dim >= 1 && d_model >= 1 && dim % d_model == 0,
                "event_decode_step: dim must be a multiple of d_model");
    BCM_REQUIRE(dstate >= 1 && dstate <= 256, "event_decode_step: dstate must be in [1, 256]");
    BCM_REQUIRE(batch * dim < (1ll << 31), "event_decode_step: too many channels");
    if (batch == 0) return BCM_OK;
    BCM_REQUIRE(x && spikes && dt_idle && dt_active && A && W_B && W_C && eta && counters && held && y,
                "event_decode_step: null pointer");
    BCM_REQUIRE(conv_state == nullptr || (conv_weight && kernel_size >= 1 && kernel_size <= kDecodeMaxK),
                "event_decode_step: a conv state needs conv_weight and 1 <= kernel_size <= 8");
    DecodeArgs a;
    a.x = x; a.spikes = spikes; a.n_ch = batch * dim;
    a.D = (int)dim; a.d_model = (int)d_model; a.expand = (int)(dim / d_model); a.N = (int)dstate;
    a.K = conv_state ? (int)kernel_size : 0; a.threshold = threshold;
    a.dt_idle = dt_idle; a.dt_active = dt_active; a.A = A; a.A_sd = A_stride_d; a.A_sn = A_stride_n;
    a.W_B = W_B; a.W_C = W_C; a.Dskip = D;
    a.conv_state = conv_state; a.conv_w = conv_weight; a.conv_b = conv_bias;
    a.eta = eta; a.counters = counters; a.held = held; a.y = y;
    const unsigned grid = (unsigned)((a.n_ch + kDecodeThreads - 1) / kDecodeThreads);
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        event_decode_kernel<T><<<grid, kDecodeThreads, 0, stream>>>(a);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}
