// scan_bwd.cu — backward of the flat-channel sparse selective scan.
//
// Semantics: csrc/selective_scan/selective_scan_bwd_kernel.cuh:635-1169 — the
// gradient of the forward in scan_fwd.cu with respect to u, A, B/C (or the
// depthwise W_B/W_C, and pw_B/pw_C), dt_idle, dt_active, D and z.  The decay
// clamp is treated as identity in the derivative, like the reference.
//
// Per channel the reverse recurrence
//   g_i,s = dout_i*C_i,s + a_{i+1},s*g_{i+1},s
// needs the forward state h_{i-1},s at the same event.  We walk the channel in
// reverse, one 2048-event chunk (the x granularity) at a time:
//   pass 1  re-run the forward over the chunk from its saved start state and
//           store the state every kCkpt events (workspace, L2-resident);
//   pass 2  visit kCkpt-event tiles last to first: recompute the tile's states
//           into registers from its checkpoint, then run the reverse step over
//           the tile accumulating every gradient.
// Parameter gradients are summed per channel in registers, written as
// per-channel partials and reduced over the batch in a fixed order by a second
// kernel, so results are deterministic (the reference uses fp32 atomics).
//
// Depthwise mode uses the normalised variables of scan_fwd.cu:
//   h = W_B*eta, g = W_C*gamma, gamma_i = dout_i*u_i + a_{i+1}*gamma_{i+1},
// which turn every recurrence into a single FMA per (event, state):
//   dA_s  = W_B W_C sum_i gamma_i delta_i (eta_i - w_i)        (w = delta u^2)
//   dW_B_s = W_C sum_i gamma_i w_i,   dW_C_s = W_B sum_i dout_i u_i eta_i
//   du_i  = D dout_i + 2 u_i delta_i sum_s cc_s gamma_i + dout_i sum_s cc_s eta_i
//   ddelta_i = u_i^2 sum_s cc_s gamma_i + sum_s cc_s A_s gamma_i (eta_i - w_i)
// with cc = W_B*W_C.
#include "scan_common.cuh"

namespace bcm {

bcm_status scan_validate(const bcm_flat_ch_args* p, bool bwd);
void scan_fill_args(const bcm_flat_ch_args* p, ScanArgs& a);
bcm_status scan_launch_pw_mix(const bcm_flat_ch_args* p, float* WB_eff, float* WC_eff,
                              cudaStream_t st);

namespace {

// Gate backward (selective_scan_bwd_kernel.cuh:784-813): every lane of the
// channel scales dout by silu(z); lane `writer` also stores dz.
template <typename T>
__device__ __forceinline__ float gate_bwd(const ScanArgs& a, int e, float dout_gated, bool writer) {
    const float zv = to_f32<T>(static_cast<const T*>(a.z)[e]);
    const float sg = 1.0f / (1.0f + expf(-zv));
    if (writer) {
        const float ov = to_f32<T>(static_cast<const T*>(a.out_fwd)[e]);
        const float dz = dout_gated * ov * sg * (1.0f + zv * (1.0f - sg));
        static_cast<T*>(a.dz)[e] = from_f32<T>(dz);
    }
    return dout_gated * (zv * sg);
}

template <int G>
__device__ __forceinline__ void ckpt_store(float* p, const float (&v)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4)
            *reinterpret_cast<float4*>(p + g) = make_float4(v[g], v[g + 1], v[g + 2], v[g + 3]);
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) p[g] = v[g];
    }
}

template <int G>
__device__ __forceinline__ void ckpt_load(const float* p, float (&v)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4) {
            const float4 t = *reinterpret_cast<const float4*>(p + g);
            v[g] = t.x; v[g + 1] = t.y; v[g + 2] = t.z; v[g + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) v[g] = p[g];
    }
}

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kScanThreads, 3)
dw_bwd_kernel(ScanArgs a) {
    constexpr int CPB = kScanThreads / LPC;
    constexpr int NP = G * LPC;
    const bool HAS_Z = a.z != nullptr;
    const int tid = threadIdx.x;
    const int grp = tid / LPC, q = tid % LPC;
    const int ch = blockIdx.x * CPB + grp;
    const bool ch_ok = ch < a.n_channels;
    const int N = a.dstate;
    const int d = ch_ok ? ch % a.dim : 0;

    float A2[G], WB[G], WC[G], cc[G], ccA[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        const bool ok = ch_ok && s < N;
        const float Av = ok ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
        A2[g] = (float)((double)Av * 1.4426950408889634);
        WB[g] = ok ? a.B[d * N + s] : 0.f;
        WC[g] = ok ? a.C[d * N + s] : 0.f;
        cc[g] = WB[g] * WC[g];
        ccA[g] = cc[g] * Av;
    }
    const float dti = ch_ok ? a.dt_idle[d] : 0.f;
    const float dta = ch_ok ? a.dt_active[d] : 0.f;
    const float Dv = (ch_ok && a.D) ? a.D[d] : 0.f;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int nch = (n + kChunkX - 1) / kChunkX;
    const int nch_warp = group_max_warp<LPC>(nch);

    const T* u = static_cast<const T*>(a.u) + beg;
    const int32_t* kk = a.k + beg;
    const T* dout = static_cast<const T*>(a.dout) + beg;
    T* du = static_cast<T*>(a.du) + beg;
    float* ck = a.ws_ckpt + ((int64_t)(beg >> 3) + ch) * NP + q * G;

    float gam[G], anx[G], SA[G], SB[G], QE[G];
#pragma unroll
    for (int g = 0; g < G; ++g) { gam[g] = 0.f; anx[g] = 1.f; SA[g] = SB[g] = QE[g] = 0.f; }
    float s_ddi = 0.f, s_dda = 0.f, s_dD = 0.f;

    for (int c = nch_warp - 1; c >= 0; --c) {
        const bool c_ok = c < nch;
        const int cs = c * kChunkX;
        const int len = c_ok ? min(n - cs, kChunkX) : 0;
        const int len_warp = group_max_warp<LPC>(len);
        // ---- pass 1: checkpoints every kCkpt events of this chunk ----------
        float eta[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            eta[g] = 0.f;
            if (c_ok && c > 0 && c - 1 < a.n_chunks && q * G + g < N) {
                const float hv = a.x[((int64_t)ch * a.n_chunks + c - 1) * 2 * N + 2 * (q * G + g) + 1];
                eta[g] = (WB[g] != 0.f) ? hv / WB[g] : 0.f;
            }
        }
        for (int j0 = 0; j0 < len_warp; j0 += kCkpt) {
            if (j0 < len) ckpt_store<G>(ck + (int64_t)(j0 / kCkpt) * NP, eta);
            float uv[kCkpt];
            int kv[kCkpt];
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = j0 + i < len;
                uv[i] = ok ? to_f32<T>(u[cs + j0 + i]) : 0.f;
                kv[i] = ok ? kk[cs + j0 + i] : 1;
            }
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = j0 + i < len;
                const float delta = event_delta(dti, dta, kv[i]);
                const float w = ok ? delta * uv[i] * uv[i] : 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float dec = ok ? decay_exact(delta, A2[g]) : 1.f;
                    eta[g] = fmaf(dec, eta[g], w);
                }
            }
        }
        // ---- pass 2: tiles in reverse ---------------------------------------
        const int nt = (len + kCkpt - 1) / kCkpt;
        const int nt_warp = group_max_warp<LPC>(nt);
        for (int m = nt_warp - 1; m >= 0; --m) {
            const int jb = cs + m * kCkpt;
            const int cnt = (m < nt) ? min(kCkpt, cs + len - jb) : 0;
            float et[G];
            if (cnt > 0) ckpt_load<G>(ck + (int64_t)m * NP, et);
            else {
#pragma unroll
                for (int g = 0; g < G; ++g) et[g] = 0.f;
            }
            float uv[kCkpt], dv[kCkpt];
            int kv[kCkpt];
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = i < cnt;
                uv[i] = ok ? to_f32<T>(u[jb + i]) : 0.f;
                kv[i] = ok ? kk[jb + i] : 1;
                float dg = ok ? to_f32<T>(dout[jb + i]) : 0.f;
                if (HAS_Z && ok) dg = gate_bwd<T>(a, beg + jb + i, dg, q == 0);
                dv[i] = dg;
            }
            // tile-local partial sums, folded into the totals after the tile
            // (pairwise summation keeps long channels accurate in fp32)
            float tSA[G], tSB[G], tQE[G];
#pragma unroll
            for (int g = 0; g < G; ++g) tSA[g] = tSB[g] = tQE[g] = 0.f;
            // forward recompute of the tile
            float eti[kCkpt][G], deci[kCkpt][G], teta[kCkpt];
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = i < cnt;
                const float delta = event_delta(dti, dta, kv[i]);
                const float w = ok ? delta * uv[i] * uv[i] : 0.f;
                const float qv = dv[i] * uv[i];
                float te = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float dec = ok ? decay_exact(delta, A2[g]) : 1.f;
                    et[g] = fmaf(dec, et[g], w);
                    eti[i][g] = et[g];
                    deci[i][g] = dec;
                    te = fmaf(cc[g], et[g], te);
                    tQE[g] = fmaf(qv, et[g], tQE[g]);
                }
                teta[i] = te;
            }
            // reverse over the tile
            float tgam[kCkpt], tdA[kCkpt];
#pragma unroll
            for (int i = kCkpt - 1; i >= 0; --i) {
                const bool ok = i < cnt;
                const float delta = event_delta(dti, dta, kv[i]);
                const float w = delta * uv[i] * uv[i];
                const float qv = dv[i] * uv[i];
                float tg = 0.f, ta = 0.f;
                if (ok) {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        gam[g] = fmaf(anx[g], gam[g], qv);
                        const float e = eti[i][g] - w;
                        const float pr = gam[g] * e;
                        tSA[g] = fmaf(pr, delta, tSA[g]);
                        ta = fmaf(ccA[g], pr, ta);
                        tSB[g] = fmaf(gam[g], w, tSB[g]);
                        tg = fmaf(cc[g], gam[g], tg);
                        anx[g] = deci[i][g];
                    }
                }
                tgam[i] = tg;
                tdA[i] = ta;
            }
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                teta[i] = group_sum<LPC>(teta[i]);
                tgam[i] = group_sum<LPC>(tgam[i]);
                tdA[i] = group_sum<LPC>(tdA[i]);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) { SA[g] += tSA[g]; SB[g] += tSB[g]; QE[g] += tQE[g]; }
            if (q == 0) {
                float t_ddi = 0.f, t_dda = 0.f, t_dD = 0.f;
#pragma unroll
                for (int i = 0; i < kCkpt; ++i) {
                    if (i < cnt) {
                        const float delta = event_delta(dti, dta, kv[i]);
                        const float duv = fmaf(Dv, dv[i], fmaf(2.f * uv[i] * delta, tgam[i], dv[i] * teta[i]));
                        du[jb + i] = from_f32<T>(duv);
                        const float ddel = fmaf(uv[i] * uv[i], tgam[i], tdA[i]);
                        t_ddi = fmaf(ddel, (float)(kv[i] - 1), t_ddi);
                        t_dda += ddel;
                        t_dD = fmaf(dv[i], uv[i], t_dD);
                    }
                }
                s_ddi += t_ddi;
                s_dda += t_dda;
                s_dD += t_dD;
            }
        }
    }
    if (!ch_ok) return;
    float* part = a.ws_part + (int64_t)ch * a.part_stride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        if (s < N) {
            part[s] = cc[g] * SA[g];
            part[NP + s] = WC[g] * SB[g];
            part[2 * NP + s] = WB[g] * QE[g];
        }
    }
    if (q == 0) {
        part[3 * NP] = s_ddi;
        part[3 * NP + 1] = s_dda;
        part[3 * NP + 2] = s_dD;
    }
}

struct BCAddrB {
    int mode, var, N, dim, E, cs, nt;
    const float* p;
    const int32_t* toff;
    // element index, or -1 when the tile map points outside B/C
    __device__ __forceinline__ int64_t idx(int ch, int d, int beg, int j, int s) const {
        if (mode == BCM_BC_TILED) {
            const int64_t tile = (int64_t)toff[ch] + j / cs;
            if (tile < 0 || tile >= nt) return -1;
            return (tile * N + s) * cs + j % cs;
        }
        if (var) return (int64_t)s * E + beg + j;
        return (int64_t)s * dim + d;
    }
};

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kScanThreads, 3)
gen_bwd_kernel(ScanArgs a) {
    constexpr int CPB = kScanThreads / LPC;
    constexpr int NP = G * LPC;
    const bool HAS_Z = a.z != nullptr;
    const int tid = threadIdx.x;
    const int grp = tid / LPC, q = tid % LPC;
    const int ch = blockIdx.x * CPB + grp;
    const bool ch_ok = ch < a.n_channels;
    const int N = a.dstate;
    const int d = ch_ok ? ch % a.dim : 0;
    const BCAddrB Bq{a.bc_mode, a.b_variable, N, a.dim, a.n_events, a.tile_cs, a.n_tiles, a.B, a.tile_off};
    const BCAddrB Cq{a.bc_mode, a.c_variable, N, a.dim, a.n_events, a.tile_cs, a.n_tiles, a.C, a.tile_off};

    float A2[G], Ar[G];
    bool sok[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        sok[g] = ch_ok && s < N;
        Ar[g] = sok[g] ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
        A2[g] = (float)((double)Ar[g] * 1.4426950408889634);
    }
    const float dti = ch_ok ? a.dt_idle[d] : 0.f;
    const float dta = ch_ok ? a.dt_active[d] : 0.f;
    const float Dv = (ch_ok && a.D) ? a.D[d] : 0.f;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int nch = (n + kChunkX - 1) / kChunkX;
    const int nch_warp = group_max_warp<LPC>(nch);
    const T* u = static_cast<const T*>(a.u) + beg;
    const int32_t* kk = a.k + beg;
    const T* dout = static_cast<const T*>(a.dout) + beg;
    T* du = static_cast<T*>(a.du) + beg;
    float* ck = a.ws_ckpt + ((int64_t)(beg >> 3) + ch) * NP + q * G;

    float gg[G], anx[G], SA[G], SB[G], SC[G];
#pragma unroll
    for (int g = 0; g < G; ++g) { gg[g] = 0.f; anx[g] = 1.f; SA[g] = SB[g] = SC[g] = 0.f; }
    float s_ddi = 0.f, s_dda = 0.f, s_dD = 0.f;

    for (int c = nch_warp - 1; c >= 0; --c) {
        const bool c_ok = c < nch;
        const int cs = c * kChunkX;
        const int len = c_ok ? min(n - cs, kChunkX) : 0;
        const int len_warp = group_max_warp<LPC>(len);
        float h[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            h[g] = 0.f;
            if (c_ok && c > 0 && c - 1 < a.n_chunks && sok[g])
                h[g] = a.x[((int64_t)ch * a.n_chunks + c - 1) * 2 * N + 2 * (q * G + g) + 1];
        }
        for (int j0 = 0; j0 < len_warp; ++j0) {
            const bool ok = j0 < len;
            if (ok && j0 % kCkpt == 0) ckpt_store<G>(ck + (int64_t)(j0 / kCkpt) * NP, h);
            if (ok) {
                const int j = cs + j0;
                const float uv = to_f32<T>(u[j]);
                const float delta = event_delta(dti, dta, kk[j]);
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (sok[g]) {
                        const int64_t bi = Bq.idx(ch, d, beg, j, q * G + g);
                        const float Bv = bi >= 0 ? a.B[bi] : 0.f;
                        h[g] = fmaf(decay_fast(delta, A2[g]), h[g], Bv * (delta * uv));
                    }
            }
        }
        const int nt = (len + kCkpt - 1) / kCkpt;
        const int nt_warp = group_max_warp<LPC>(nt);
        for (int m = nt_warp - 1; m >= 0; --m) {
            const int jb = cs + m * kCkpt;
            const int cnt = (m < nt) ? min(kCkpt, cs + len - jb) : 0;
            float ht[G];
            if (cnt > 0) ckpt_load<G>(ck + (int64_t)m * NP, ht);
            else {
#pragma unroll
                for (int g = 0; g < G; ++g) ht[g] = 0.f;
            }
            float uv[kCkpt], dv[kCkpt];
            int kv[kCkpt];
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = i < cnt;
                uv[i] = ok ? to_f32<T>(u[jb + i]) : 0.f;
                kv[i] = ok ? kk[jb + i] : 1;
                float dg = ok ? to_f32<T>(dout[jb + i]) : 0.f;
                if (HAS_Z && ok) dg = gate_bwd<T>(a, beg + jb + i, dg, q == 0);
                dv[i] = dg;
            }
            float tSA[G], tSB[G], tSC[G];
#pragma unroll
            for (int g = 0; g < G; ++g) tSA[g] = tSB[g] = tSC[g] = 0.f;
            float hi[kCkpt][G], deci[kCkpt][G];
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                const bool ok = i < cnt;
                const float delta = event_delta(dti, dta, kv[i]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float dec = 1.f, bb = 0.f;
                    if (ok && sok[g]) {
                        dec = decay_fast(delta, A2[g]);
                        const int64_t bi = Bq.idx(ch, d, beg, jb + i, q * G + g);
                        bb = (bi >= 0 ? a.B[bi] : 0.f) * (delta * uv[i]);
                    }
                    ht[g] = fmaf(dec, ht[g], bb);
                    hi[i][g] = ht[g];
                    deci[i][g] = dec;
                }
            }
            float tdu[kCkpt], tdd[kCkpt];
#pragma unroll
            for (int i = kCkpt - 1; i >= 0; --i) {
                const bool ok = i < cnt;
                const float delta = event_delta(dti, dta, kv[i]);
                float t1 = 0.f, t2 = 0.f;
                if (ok) {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        if (!sok[g]) continue;
                        const int s = q * G + g;
                        const int64_t bi = Bq.idx(ch, d, beg, jb + i, s);
                        const int64_t ci = Cq.idx(ch, d, beg, jb + i, s);
                        const float Bv = bi >= 0 ? a.B[bi] : 0.f;
                        const float Cv = ci >= 0 ? a.C[ci] : 0.f;
                        gg[g] = fmaf(anx[g], gg[g], dv[i] * Cv);
                        const float bb = Bv * (delta * uv[i]);
                        const float e = hi[i][g] - bb;
                        const float gB = gg[g] * Bv;
                        t1 = fmaf(gB, delta, t1);                       // du via B*delta*u
                        t2 = fmaf(gB, uv[i], fmaf(gg[g] * Ar[g], e, t2)); // ddelta
                        tSA[g] = fmaf(gg[g] * delta, e, tSA[g]);
                        const float dBv = gg[g] * delta * uv[i];
                        const float dCv = dv[i] * hi[i][g];
                        if (a.b_variable) { if (bi >= 0) a.dB_ev[bi] = dBv; } else tSB[g] += dBv;
                        if (a.c_variable) { if (ci >= 0) a.dC_ev[ci] = dCv; } else tSC[g] += dCv;
                        anx[g] = deci[i][g];
                    }
                }
                tdu[i] = t1;
                tdd[i] = t2;
            }
#pragma unroll
            for (int i = 0; i < kCkpt; ++i) {
                tdu[i] = group_sum<LPC>(tdu[i]);
                tdd[i] = group_sum<LPC>(tdd[i]);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) { SA[g] += tSA[g]; SB[g] += tSB[g]; SC[g] += tSC[g]; }
            if (q == 0) {
                float t_ddi = 0.f, t_dda = 0.f, t_dD = 0.f;
#pragma unroll
                for (int i = 0; i < kCkpt; ++i) {
                    if (i < cnt) {
                        du[jb + i] = from_f32<T>(fmaf(Dv, dv[i], tdu[i]));
                        t_ddi = fmaf(tdd[i], (float)(kv[i] - 1), t_ddi);
                        t_dda += tdd[i];
                        t_dD = fmaf(dv[i], uv[i], t_dD);
                    }
                }
                s_ddi += t_ddi;
                s_dda += t_dda;
                s_dD += t_dD;
            }
        }
    }
    if (!ch_ok) return;
    float* part = a.ws_part + (int64_t)ch * a.part_stride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        if (s < N) {
            part[s] = SA[g];
            part[NP + s] = SB[g];
            part[2 * NP + s] = SC[g];
        }
    }
    if (q == 0) {
        part[3 * NP] = s_ddi;
        part[3 * NP + 1] = s_dda;
        part[3 * NP + 2] = s_dD;
    }
}

// Fixed-order batch reduction of the per-channel partials:
// out[d] = sum_b part[b*dim + d] for every field.
__global__ void reduce_parts_kernel(const float* __restrict__ part, int stride, int NP, int n_ch,
                                    int dim, int N, float* __restrict__ dA,
                                    float* __restrict__ dB, float* __restrict__ dC,
                                    int bc_dim_major,  // 1: dB/dC [dim,N], 0: [N,dim]
                                    int want_B, int want_C,
                                    float* __restrict__ ddi, float* __restrict__ dda,
                                    float* __restrict__ dD) {
    const int F = 3 * N + 3;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= dim * F) return;
    const int d = idx / F, f = idx % F;
    int off;
    if (f < 3 * N) off = (f / N) * NP + f % N;
    else off = 3 * NP + (f - 3 * N);
    float acc = 0.f;
#pragma unroll 8
    for (int ch = d; ch < n_ch; ch += dim) acc += part[(int64_t)ch * stride + off];
    if (f < N) dA[d * N + f] = acc;
    else if (f < 2 * N) {
        const int s = f - N;
        if (want_B) dB[bc_dim_major ? d * N + s : s * dim + d] = acc;
    } else if (f < 3 * N) {
        const int s = f - 2 * N;
        if (want_C) dC[bc_dim_major ? d * N + s : s * dim + d] = acc;
    } else if (f == 3 * N) ddi[d] = acc;
    else if (f == 3 * N + 1) dda[d] = acc;
    else if (dD) dD[d] = acc;
}

// Chain rule through W_eff = pw @ W:
//   dW[d',s] = sum_d pw[d,d'] dW_eff[d,s];  dpw[d,d'] = sum_s dW_eff[d,s] W[d',s]
__global__ void pw_grad_W_kernel(const float* __restrict__ pw, const float* __restrict__ dWe,
                                 int dim, int N, float* __restrict__ dW) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= dim * N) return;
    const int d2 = idx / N, s = idx % N;
    float acc = 0.f;
    for (int d = 0; d < dim; ++d) acc = fmaf(pw[(int64_t)d * dim + d2], dWe[(int64_t)d * N + s], acc);
    dW[idx] = acc;
}

__global__ void pw_grad_pw_kernel(const float* __restrict__ dWe, const float* __restrict__ W,
                                  int dim, int N, float* __restrict__ dpw) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)dim * dim) return;
    const int d = (int)(idx / dim), d2 = (int)(idx % dim);
    float acc = 0.f;
    for (int s = 0; s < N; ++s) acc = fmaf(dWe[(int64_t)d * N + s], W[(int64_t)d2 * N + s], acc);
    dpw[idx] = acc;
}

template <typename T, int G, int LPC>
bcm_status launch_bwd_tl(const ScanArgs& a, bool dw, bool has_z, cudaStream_t st) {
    constexpr int CPB = kScanThreads / LPC;
    const int grid = ceil_div(a.n_channels, CPB);
    if (dw) {
        dw_bwd_kernel<T, G, LPC><<<grid, kScanThreads, 0, st>>>(a);
    } else {
        gen_bwd_kernel<T, G, LPC><<<grid, kScanThreads, 0, st>>>(a);
    }
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T>
bcm_status launch_bwd(const ScanArgs& a, bool dw, bool has_z, cudaStream_t st) {
    int G, LPC;
    pick_layout(a.dstate, G, LPC);
    if (G == 8) return launch_bwd_tl<T, 8, 32>(a, dw, has_z, st);
    switch (LPC) {
        case 1: return launch_bwd_tl<T, 4, 1>(a, dw, has_z, st);
        case 2: return launch_bwd_tl<T, 4, 2>(a, dw, has_z, st);
        case 4: return launch_bwd_tl<T, 4, 4>(a, dw, has_z, st);
        case 8: return launch_bwd_tl<T, 4, 8>(a, dw, has_z, st);
        case 16: return launch_bwd_tl<T, 4, 16>(a, dw, has_z, st);
        default: return launch_bwd_tl<T, 4, 32>(a, dw, has_z, st);
    }
}

// Workspace of the backward: [checkpoints (staged kernels) | decay tables +
// tile carries (event-parallel kernels)] [per-row parameter partials]
// [W_B/W_C mixed by pw] [their gradients].
struct BwdLayout {
    size_t ckpt_off, ckpt_bytes, part_off, part_bytes, weff_off, weff_bytes, dweff_off, total;
    size_t tab_off, carry_off, order_off;
    int NP, part_stride, part_rows;
    bool seg, staged;
};

BwdLayout bwd_layout(const bcm_flat_ch_args* p) {
    BwdLayout L{};
    ScanArgs a;
    scan_fill_args(p, a);
    L.seg = p->n_events > 0 && seg_selected(a);
    L.staged = !L.seg && p->n_events > 0 && p->bc_mode == BCM_BC_DEPTHWISE &&
               dw_fast_supported((int)p->dstate) && v3_supported(a, true);
    int G, LPC;
    pick_layout((int)p->dstate, G, LPC);
    L.NP = G * LPC;
    if (p->bc_mode == BCM_BC_DEPTHWISE && dw_fast_supported((int)p->dstate))
        L.NP = dw_fast_np((int)p->dstate);
    L.part_rows = (int)p->n_channels;
    L.ckpt_off = 0;
    if (L.seg) {
        L.NP = (int)p->dstate;
        L.part_rows = seg_part_rows(a);
        L.tab_off = 0;
        L.carry_off = seg_table_bytes(a);
        L.ckpt_bytes = L.carry_off + seg_carry_bytes(a);
    } else {
        const size_t slots = (size_t)(p->n_events >> 3) + (size_t)p->n_channels + 1;
        L.ckpt_bytes = align_up(slots * L.NP * sizeof(float), 256);
    }
    L.part_stride = (3 * L.NP + 3 + 3) / 4 * 4;
    L.part_off = L.ckpt_off + L.ckpt_bytes;
    L.part_bytes = align_up((size_t)L.part_rows * L.part_stride * sizeof(float), 256);
    L.weff_off = L.part_off + L.part_bytes;
    L.weff_bytes = p->pw_B ? align_up((size_t)2 * p->dim * p->dstate * sizeof(float), 256) : 0;
    L.dweff_off = L.weff_off + L.weff_bytes;
    L.order_off = L.dweff_off + L.weff_bytes;
    L.total = L.order_off + (L.staged ? staged_prep_bytes(a) : 0);
    return L;
}

}  // namespace
}  // namespace bcm

using namespace bcm;

extern "C" size_t bcm_flat_ch_bwd_workspace_bytes(const bcm_flat_ch_args* p) {
    if (!p) return 0;
    return bwd_layout(p).total;
}

extern "C" bcm_status bcm_flat_ch_bwd(const bcm_flat_ch_args* p, cudaStream_t stream) {
    clear_error();
    bcm_status st = scan_validate(p, true);
    if (st != BCM_OK) return st;
    BCM_REQUIRE(p->x, "flat_ch bwd: null x");
    BCM_REQUIRE(p->n_events == 0 || (p->dout && p->du), "flat_ch bwd: null dout/du");
    BCM_REQUIRE(p->dA && p->ddt_idle && p->ddt_active && p->dB && p->dC, "flat_ch bwd: null gradient output");
    BCM_REQUIRE(p->z == nullptr || (p->out_fwd && p->dz), "flat_ch bwd: z needs out and dz");
    BCM_REQUIRE(p->pw_B == nullptr || (p->dpw_B && p->dpw_C), "flat_ch bwd: pw needs dpw outputs");
    const BwdLayout L = bwd_layout(p);
    if (!p->workspace || p->workspace_bytes < L.total) {
        set_error("flat_ch bwd: workspace of %zu bytes < required %zu", p->workspace_bytes, L.total);
        return BCM_ERR_WORKSPACE;
    }
    char* ws = static_cast<char*>(p->workspace);
    ScanArgs a;
    scan_fill_args(p, a);
    a.ws_ckpt = reinterpret_cast<float*>(ws + L.ckpt_off);
    a.ws_part = reinterpret_cast<float*>(ws + L.part_off);
    a.part_stride = L.part_stride;
    a.dB_ev = p->dB;
    a.dC_ev = p->dC;
    const bool dw = p->bc_mode == BCM_BC_DEPTHWISE;
    float* WB_eff = nullptr;
    float* WC_eff = nullptr;
    if (p->pw_B) {
        WB_eff = reinterpret_cast<float*>(ws + L.weff_off);
        WC_eff = WB_eff + p->dim * p->dstate;
        st = scan_launch_pw_mix(p, WB_eff, WC_eff, stream);
        if (st != BCM_OK) return st;
        a.B = WB_eff;
        a.C = WC_eff;
    }
    // every channel (warp group) writes its partial row, so no clearing is needed
    if (L.seg) {
        st = seg_bwd_launch(a, p->dtype, reinterpret_cast<float*>(ws + L.tab_off), a.ckpt,
                            reinterpret_cast<float*>(ws + L.carry_off), stream);
        if (st != BCM_OK) return st;
    } else if (p->n_events > 0 && dw && dw_fast_supported(a.dstate)) {
        if (L.staged) {
            st = staged_prep_launch(a, ws + L.order_off, stream);
            if (st != BCM_OK) return st;
        }
        st = dw_fast_launch(a, p->dtype, true, stream);
        if (st != BCM_OK) return st;
    } else if (p->n_events > 0) {
        st = dispatch_dtype(p->dtype, [&](auto tag) -> bcm_status {
            using T = decltype(tag);
            return launch_bwd<T>(a, dw, p->z != nullptr, stream);
        });
        if (st != BCM_OK) return st;
    } else {
        BCM_CUDA_TRY(cudaMemsetAsync(a.ws_part, 0, L.part_bytes, stream));
    }
    const int N = (int)p->dstate, dim = (int)p->dim;
    float* dWB_target = p->dB;
    float* dWC_target = p->dC;
    float* dWeB = nullptr;
    float* dWeC = nullptr;
    if (p->pw_B) {
        dWeB = reinterpret_cast<float*>(ws + L.dweff_off);
        dWeC = dWeB + p->dim * p->dstate;
        dWB_target = dWeB;
        dWC_target = dWeC;
    }
    const int want_B = dw ? 1 : (p->bc_mode == BCM_BC_FLAT && !p->b_variable);
    const int want_C = dw ? 1 : (p->bc_mode == BCM_BC_FLAT && !p->c_variable);
    {
        const int total = dim * (3 * N + 3);
        const int threads = 256;
        reduce_parts_kernel<<<ceil_div(total, threads), threads, 0, stream>>>(
            a.ws_part, L.part_stride, L.NP, L.part_rows, dim, N, p->dA, dWB_target,
            dWC_target, dw ? 1 : 0, want_B, want_C, p->ddt_idle, p->ddt_active, p->dD);
        BCM_LAUNCH_CHECK();
    }
    if (p->pw_B) {
        const int threads = 256;
        pw_grad_W_kernel<<<ceil_div(dim * N, threads), threads, 0, stream>>>(p->pw_B, dWeB, dim, N, p->dB);
        BCM_LAUNCH_CHECK();
        pw_grad_W_kernel<<<ceil_div(dim * N, threads), threads, 0, stream>>>(p->pw_C, dWeC, dim, N, p->dC);
        BCM_LAUNCH_CHECK();
        pw_grad_pw_kernel<<<ceil_div((int64_t)dim * dim, threads), threads, 0, stream>>>(dWeB, p->B, dim, N, p->dpw_B);
        BCM_LAUNCH_CHECK();
        pw_grad_pw_kernel<<<ceil_div((int64_t)dim * dim, threads), threads, 0, stream>>>(dWeC, p->C, dim, N, p->dpw_C);
        BCM_LAUNCH_CHECK();
    }
    return BCM_OK;
}
