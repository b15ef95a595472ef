// scan_fwd.cu — forward of the flat-channel sparse selective scan.
//
// Semantics: csrc/selective_scan/selective_scan_fwd_kernel.cuh:403-728 (one
// channel's events, delta = dt_idle*(k-1)+dt_active, decay exp2(clamp(delta*A*
// log2e, +-126)), y = D*u + sum_s h*C, chunk-boundary (prod a, h) into x,
// optional silu(z) gate) and the depthwise B/C construction :568-611.
//
// Depthwise path (what the model runs): B_i,s = u_i*W_B[d,s] and C_i,s =
// u_i*W_C[d,s], so h_i,s = W_B[d,s]*eta_i,s with the normalised recurrence
//   eta_i,s = a_i,s*eta_{i-1},s + delta_i*u_i^2
// and y_i = D*u_i + u_i * sum_s (W_B*W_C)[d,s]*eta_i,s.  Per (event, state)
// that is one decay, one FMA for the state and one FMA for the output.
#include "scan_common.cuh"

namespace bcm {
namespace {

constexpr int kU = 8;  // events loaded per batch

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kScanThreads)
dw_fwd_kernel(ScanArgs a) {
    constexpr int CPB = kScanThreads / LPC;
    const bool HAS_Z = a.z != nullptr;
    const int tid = threadIdx.x;
    const int grp = tid / LPC, q = tid % LPC;
    const int ch = blockIdx.x * CPB + grp;
    const bool ch_ok = ch < a.n_channels;
    const int N = a.dstate;
    const int d = ch_ok ? ch % a.dim : 0;

    float A2[G], WB[G], cc[G], eta[G], P[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        const bool ok = ch_ok && s < N;
        const float Av = ok ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
        A2[g] = (float)((double)Av * 1.4426950408889634);
        WB[g] = ok ? a.B[d * N + s] : 0.f;
        cc[g] = ok ? WB[g] * a.C[d * N + s] : 0.f;
        eta[g] = 0.f;
        P[g] = 1.f;
    }
    const float dti = ch_ok ? a.dt_idle[d] : 0.f;
    const float dta = ch_ok ? a.dt_active[d] : 0.f;
    const float Dv = (ch_ok && a.D) ? a.D[d] : 0.f;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int n_warp = group_max_warp<LPC>(n);

    const T* u = static_cast<const T*>(a.u) + beg;
    const int32_t* kk = a.k + beg;
    T* out = static_cast<T*>(a.out) + beg;

    for (int j0 = 0; j0 < n_warp; j0 += kU) {
        float uv[kU];
        int kv[kU];
#pragma unroll
        for (int i = 0; i < kU; ++i) {
            const bool ok = j0 + i < n;
            uv[i] = ok ? to_f32<T>(u[j0 + i]) : 0.f;
            kv[i] = ok ? kk[j0 + i] : 1;
        }
#pragma unroll
        for (int i = 0; i < kU; ++i) {
            const int j = j0 + i;
            const bool ok = j < n;
            const float delta = event_delta(dti, dta, kv[i]);
            const float w = delta * uv[i] * uv[i];
            float acc = 0.f;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float dec = ok ? decay_exact(delta, A2[g]) : 1.f;
                eta[g] = fmaf(dec, eta[g], ok ? w : 0.f);
                P[g] *= dec;
                acc = fmaf(cc[g], eta[g], acc);
            }
            acc = group_sum<LPC>(acc);
            if (ok) {
                const float y = fmaf(Dv, uv[i], uv[i] * acc);
                if (q == 0) {
                    out[j] = from_f32<T>(y);
                    if (HAS_Z) {
                        const float zv = to_f32<T>(static_cast<const T*>(a.z)[beg + j]);
                        static_cast<T*>(a.out_z)[beg + j] = from_f32<T>(y * silu(zv));
                    }
                }
                if ((j + 1) % kChunkX == 0 || j == n - 1) {
                    const int c = j / kChunkX;
                    if (c < a.n_chunks) {
                        float* xo = a.x + ((int64_t)ch * a.n_chunks + c) * 2 * N;
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const int s = q * G + g;
                            if (s < N) {
                                xo[2 * s] = P[g];
                                xo[2 * s + 1] = WB[g] * eta[g];
                            }
                        }
                    }
                }
            }
        }
    }
}

// ---- generic path: B/C per event [N,E], per feature [N,dim] or tiled -------
struct BCAddr {
    int mode, var, N, dim, E, cs, nt;
    const float* p;
    const int32_t* toff;
    __device__ __forceinline__ float get(int ch, int d, int beg, int j, int s) const {
        if (mode == BCM_BC_TILED) {
            const int64_t tile = (int64_t)toff[ch] + j / cs;
            if (tile < 0 || tile >= nt) return 0.f;  // tile map inconsistent with B/C
            return p[(tile * N + s) * cs + j % cs];
        }
        if (var) return p[(int64_t)s * E + beg + j];
        return p[s * dim + d];
    }
};

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kScanThreads)
gen_fwd_kernel(ScanArgs a) {
    constexpr int CPB = kScanThreads / LPC;
    const bool HAS_Z = a.z != nullptr;
    const int tid = threadIdx.x;
    const int grp = tid / LPC, q = tid % LPC;
    const int ch = blockIdx.x * CPB + grp;
    const bool ch_ok = ch < a.n_channels;
    const int N = a.dstate;
    const int d = ch_ok ? ch % a.dim : 0;
    const BCAddr Bq{a.bc_mode, a.b_variable, N, a.dim, a.n_events, a.tile_cs, a.n_tiles, a.B, a.tile_off};
    const BCAddr Cq{a.bc_mode, a.c_variable, N, a.dim, a.n_events, a.tile_cs, a.n_tiles, a.C, a.tile_off};

    float A2[G], h[G], P[G];
    bool sok[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        sok[g] = ch_ok && s < N;
        const float Av = sok[g] ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
        A2[g] = (float)((double)Av * 1.4426950408889634);
        h[g] = 0.f;
        P[g] = 1.f;
    }
    const float dti = ch_ok ? a.dt_idle[d] : 0.f;
    const float dta = ch_ok ? a.dt_active[d] : 0.f;
    const float Dv = (ch_ok && a.D) ? a.D[d] : 0.f;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int n_warp = group_max_warp<LPC>(n);
    const T* u = static_cast<const T*>(a.u) + beg;
    T* out = static_cast<T*>(a.out) + beg;

    for (int j = 0; j < n_warp; ++j) {
        const bool ok = j < n;
        const float uv = ok ? to_f32<T>(u[j]) : 0.f;
        const float delta = event_delta(dti, dta, ok ? a.k[beg + j] : 1);
        const float du_ = delta * uv;
        float acc = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (ok && sok[g]) {
                const int s = q * G + g;
                const float dec = decay_fast(delta, A2[g]);
                const float Bv = Bq.get(ch, d, beg, j, s);
                const float Cv = Cq.get(ch, d, beg, j, s);
                h[g] = fmaf(dec, h[g], Bv * du_);
                P[g] *= dec;
                acc = fmaf(h[g], Cv, acc);
            }
        }
        acc = group_sum<LPC>(acc);
        if (ok) {
            const float y = fmaf(Dv, uv, acc);
            if (q == 0) {
                out[j] = from_f32<T>(y);
                if (HAS_Z) {
                    const float zv = to_f32<T>(static_cast<const T*>(a.z)[beg + j]);
                    static_cast<T*>(a.out_z)[beg + j] = from_f32<T>(y * silu(zv));
                }
            }
            if ((j + 1) % kChunkX == 0 || j == n - 1) {
                const int c = j / kChunkX;
                if (c < a.n_chunks) {
                    float* xo = a.x + ((int64_t)ch * a.n_chunks + c) * 2 * N;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const int s = q * G + g;
                        if (s < N) { xo[2 * s] = P[g]; xo[2 * s + 1] = h[g]; }
                    }
                }
            }
        }
    }
}

// W_eff[d,s] = sum_d' pw[d,d'] * W[d',s] (depthwise + pointwise mixing,
// selective_scan_fwd_kernel.cuh:492-510).
__global__ void pw_mix_kernel(const float* __restrict__ pw, const float* __restrict__ W,
                              int dim, int N, float* __restrict__ W_eff) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= dim * N) return;
    const int d = idx / N, s = idx % N;
    float acc = 0.f;
    for (int d2 = 0; d2 < dim; ++d2) acc = fmaf(pw[(int64_t)d * dim + d2], W[(int64_t)d2 * N + s], acc);
    W_eff[idx] = acc;
}

template <typename T, int G, int LPC>
bcm_status launch_fwd_tl(const ScanArgs& a, bool dw, bool has_z, cudaStream_t st) {
    constexpr int CPB = kScanThreads / LPC;
    const int grid = ceil_div(a.n_channels, CPB);
    if (dw) {
        dw_fwd_kernel<T, G, LPC><<<grid, kScanThreads, 0, st>>>(a);
    } else {
        gen_fwd_kernel<T, G, LPC><<<grid, kScanThreads, 0, st>>>(a);
    }
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T>
bcm_status launch_fwd(const ScanArgs& a, bool dw, bool has_z, cudaStream_t st) {
    int G, LPC;
    pick_layout(a.dstate, G, LPC);
    if (G == 8) return launch_fwd_tl<T, 8, 32>(a, dw, has_z, st);
    switch (LPC) {
        case 1: return launch_fwd_tl<T, 4, 1>(a, dw, has_z, st);
        case 2: return launch_fwd_tl<T, 4, 2>(a, dw, has_z, st);
        case 4: return launch_fwd_tl<T, 4, 4>(a, dw, has_z, st);
        case 8: return launch_fwd_tl<T, 4, 8>(a, dw, has_z, st);
        case 16: return launch_fwd_tl<T, 4, 16>(a, dw, has_z, st);
        default: return launch_fwd_tl<T, 4, 32>(a, dw, has_z, st);
    }
}

}  // namespace

// Validation shared by the forward and backward entry points.
bcm_status scan_validate(const bcm_flat_ch_args* p, bool bwd) {
    BCM_REQUIRE(p != nullptr, "flat_ch: null args");
    BCM_REQUIRE(dtype_ok(p->dtype), "flat_ch: u_flat must be fp16/bf16/fp32");
    BCM_REQUIRE(p->n_events >= 0 && p->n_events < (1ll << 31), "flat_ch: bad n_events");
    BCM_REQUIRE(p->n_channels >= 1 && p->n_channels < (1ll << 31), "flat_ch: bad n_channels");
    BCM_REQUIRE(p->dim >= 1, "flat_ch: bad dim");
    BCM_REQUIRE(p->dstate >= 1 && p->dstate <= 256, "flat_ch: dstate must be <= 256");
    BCM_REQUIRE(p->max_seqlen >= 0, "flat_ch: max_seqlen must be non-negative");
    BCM_REQUIRE(p->bc_mode == BCM_BC_DEPTHWISE || p->bc_mode == BCM_BC_FLAT ||
                    p->bc_mode == BCM_BC_TILED,
                "flat_ch: bad bc_mode %d", p->bc_mode);
    BCM_REQUIRE(p->cu_seqlens && p->dt_idle && p->dt_active && p->A && p->B && p->C,
                "flat_ch: null input pointer");
    BCM_REQUIRE(p->n_events == 0 || (p->u && p->k), "flat_ch: null u/k");
    BCM_REQUIRE(p->bc_mode != BCM_BC_TILED || p->tile_offsets, "flat_ch: tiled mode needs tile_offsets");
    BCM_REQUIRE((p->pw_B == nullptr) == (p->pw_C == nullptr), "flat_ch: pw_B and pw_C go together");
    BCM_REQUIRE(p->pw_B == nullptr || p->bc_mode == BCM_BC_DEPTHWISE,
                "flat_ch: pw_B/pw_C need the depthwise mode");
    if (!bwd) {
        BCM_REQUIRE(p->n_events == 0 || p->out, "flat_ch: null out");
        BCM_REQUIRE(p->x, "flat_ch: null x");
        BCM_REQUIRE(p->z == nullptr || p->out_z, "flat_ch: z given without out_z");
    }
    return BCM_OK;
}

void scan_fill_args(const bcm_flat_ch_args* p, ScanArgs& a) {
    a.n_channels = (int)p->n_channels;
    a.dim = (int)p->dim;
    a.dstate = (int)p->dstate;
    a.n_chunks = n_chunks_for(p->max_seqlen);
    a.n_events = (int)p->n_events;
    a.bc_mode = p->bc_mode;
    a.b_variable = p->bc_mode == BCM_BC_TILED ? 1 : p->b_variable;
    a.c_variable = p->bc_mode == BCM_BC_TILED ? 1 : p->c_variable;
    a.tile_cs = ref_chunk_size(p->max_seqlen);
    a.n_tiles = p->bc_mode == BCM_BC_TILED ? (int)p->n_tiles : 0;
    a.u = p->u; a.k = p->k; a.cu = p->cu_seqlens;
    a.dt_idle = p->dt_idle; a.dt_active = p->dt_active;
    a.A = p->A; a.A_sd = p->A_stride_d; a.A_sn = p->A_stride_n;
    a.B = p->B; a.C = p->C; a.D = p->D; a.z = p->z; a.tile_off = p->tile_offsets;
    a.out = p->out; a.x = p->x; a.out_z = p->out_z;
    a.dout = p->dout; a.out_fwd = p->out_fwd;
    a.du = p->du; a.dB_ev = nullptr; a.dC_ev = nullptr; a.dz = p->dz;
    a.ws_ckpt = nullptr; a.ws_part = nullptr; a.part_stride = 0;
    a.ckpt = nullptr;
    a.row_order = nullptr;
    a.dtab = nullptr;
    a.rank_major = 0;
    if (p->ckpt != nullptr && (seg_selected(a) || v3_ckpt_bytes(a) > 0)) a.ckpt = p->ckpt;   // else ignored
}

bcm_status scan_launch_pw_mix(const bcm_flat_ch_args* p, float* WB_eff, float* WC_eff,
                              cudaStream_t st) {
    const int n = (int)(p->dim * p->dstate);
    const int threads = 256;
    pw_mix_kernel<<<ceil_div(n, threads), threads, 0, st>>>(p->pw_B, p->B, (int)p->dim,
                                                           (int)p->dstate, WB_eff);
    BCM_LAUNCH_CHECK();
    pw_mix_kernel<<<ceil_div(n, threads), threads, 0, st>>>(p->pw_C, p->C, (int)p->dim,
                                                           (int)p->dstate, WC_eff);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

}  // namespace bcm

using namespace bcm;

// Forward workspace: [W_B/W_C mixed by pw (pw only)] then [decay tables
// (event-parallel kernels)] or [row order (staged kernels)]
static size_t fwd_pw_bytes(const bcm_flat_ch_args* p) {
    return p->pw_B == nullptr ? 0 : align_up((size_t)(2 * p->dim * p->dstate * sizeof(float)), 256);
}

static bool fwd_seg(const bcm_flat_ch_args* p, ScanArgs& a) {
    if (p->n_events <= 0 || p->n_channels <= 0 || p->dim <= 0 || p->dstate <= 0) return false;
    scan_fill_args(p, a);
    return seg_selected(a);
}

static bool fwd_staged(const bcm_flat_ch_args* p, const ScanArgs& a) {
    return p->n_events > 0 && p->bc_mode == BCM_BC_DEPTHWISE && dw_fast_supported(a.dstate) &&
           v3_supported(a, false);
}

extern "C" size_t bcm_flat_ch_fwd_workspace_bytes(const bcm_flat_ch_args* p) {
    if (!p) return 0;
    ScanArgs a;
    if (fwd_seg(p, a)) return fwd_pw_bytes(p) + seg_table_bytes(a);
    if (p->n_events > 0 && p->n_channels > 0 && p->dim > 0 && p->dstate > 0) {
        scan_fill_args(p, a);
        if (fwd_staged(p, a)) return fwd_pw_bytes(p) + staged_prep_bytes(a);
    }
    return fwd_pw_bytes(p);
}

extern "C" size_t bcm_flat_ch_ckpt_bytes(const bcm_flat_ch_args* p) {
    if (!p || p->n_events <= 0 || p->n_channels <= 0 || p->dim <= 0 || p->dstate <= 0) return 0;
    ScanArgs a;
    if (fwd_seg(p, a)) return seg_carry_bytes(a);
    return v3_ckpt_bytes(a);
}

extern "C" bcm_status bcm_flat_ch_fwd(const bcm_flat_ch_args* p, cudaStream_t stream) {
    clear_error();
    bcm_status st = scan_validate(p, false);
    if (st != BCM_OK) return st;
    ScanArgs a;
    scan_fill_args(p, a);
    const size_t need = bcm_flat_ch_fwd_workspace_bytes(p);
    if (need > 0 && (!p->workspace || p->workspace_bytes < need)) {
        set_error("flat_ch fwd: workspace of %zu bytes < required %zu", p->workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    if (p->pw_B) {
        float* WB_eff = static_cast<float*>(p->workspace);
        float* WC_eff = WB_eff + p->dim * p->dstate;
        st = scan_launch_pw_mix(p, WB_eff, WC_eff, stream);
        if (st != BCM_OK) return st;
        a.B = WB_eff;
        a.C = WC_eff;
    }
    const bool dw = p->bc_mode == BCM_BC_DEPTHWISE;
    const bool has_z = p->z != nullptr;
    if (p->n_events > 0 && seg_selected(a)) {
        // event-parallel kernels: write every slot of x themselves
        float* tab = reinterpret_cast<float*>(static_cast<char*>(p->workspace) + fwd_pw_bytes(p));
        return seg_fwd_launch(a, p->dtype, tab, a.ckpt, stream);
    }
    // x is written in full: the staged forward writes every slot itself,
    // every other path writes the chunks that exist onto zeros
    const bool staged = fwd_staged(p, a);
    if (staged) {
        // rows of similar event counts share a warp; decay tables once per call
        st = staged_prep_launch(a, static_cast<char*>(p->workspace) + fwd_pw_bytes(p), stream);
        if (st != BCM_OK) return st;
    }
    if (!staged)
        BCM_CUDA_TRY(cudaMemsetAsync(p->x, 0, (size_t)a.n_channels * a.n_chunks * 2 * a.dstate * sizeof(float),
                                     stream));
    if (p->n_events == 0) return BCM_OK;
    if (dw && dw_fast_supported(a.dstate)) return dw_fast_launch(a, p->dtype, false, stream);
    return dispatch_dtype(p->dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        return launch_fwd<T>(a, dw, has_z, stream);
    });
}
