// scan_dw.cu — depthwise fast path (dstate <= 64) of the flat-channel scan,
// forward and backward.  Same semantics as the kernels of scan_fwd.cu /
// scan_bwd.cu (reference selective_scan_fwd_kernel.cuh:403-728 and
// selective_scan_bwd_kernel.cuh:635-1169, depthwise B/C); this file only
// changes how the work is laid out on the SM:
//
//  * d-major channel order: the CPW = 32/LPC channels of a warp are
//    (d, b..b+CPW-1), so they share dt_idle/dt_active/A and therefore one
//    decay table.  Because delta depends on the event only through its integer
//    gap k, a_k,s = exp2(clamp((dt_idle*(k-1)+dt_active)*A_s*log2e, +-126)) is
//    tabulated per warp in shared memory for k = 1..KT (exp2f, bit-identical to
//    the direct evaluation used for longer gaps).  A state update then costs a
//    128-bit table load per 4 states and one FMA instead of a MUFU exp2 chain.
//  * the next batch of 8 events (u, k, dout, checkpoint) is loaded into
//    registers while the current one is processed;
//  * per-event sums over a channel's states are reduced across its LPC lanes
//    by a transpose-reduction (NE-1 shuffles for NE events instead of
//    NE*log2(LPC));
//  * the chunk product prod(a) is formed as exp2(A*log2e*sum(delta) +
//    clamp corrections) instead of one multiply per (event, state).
#include <stdlib.h>

#include "scan_common.cuh"

namespace bcm {

namespace {

constexpr int kWPB = 4;    // warps per CTA
constexpr int kB = 8;      // events per register batch; equals the checkpoint tile
static_assert(kB == kCkpt, "batch and checkpoint tile must match");

template <int G, int LPC>
struct DwL {
    static constexpr int NP = G * LPC;
    static constexpr int CPW = 32 / LPC;
    static constexpr int KT = NP <= 32 ? 64 : 32;
    static constexpr int TABLE = KT * NP;
    static constexpr int EPL = kB / LPC;   // events finalised per lane per batch
};

__device__ __forceinline__ int channel_of(int gid, int dim, int bn, int dmajor) {
    if (!dmajor) return gid;
    const int d = gid / bn;
    return (gid - d * bn) * dim + d;
}

template <int NP, int KT>
__device__ void build_table(float* tab, const ScanArgs& a, int d, int lane) {
    const float dti = a.dt_idle[d], dta = a.dt_active[d];
    for (int e = lane; e < KT * NP; e += 32) {
        const int kk = e / NP + 1, s = e % NP;
        float v = 1.f;
        if (s < a.dstate) {
            const float A2 = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
            v = decay_exact(event_delta(dti, dta, kk), A2);
        }
        tab[e] = v;
    }
    __syncwarp();
}

// This lane's G decays from a table row (vector shared-memory loads).
template <int G>
__device__ __forceinline__ void table_row(const float* p, float (&dec)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g4 = 0; g4 < G / 4; ++g4) {
            const float4 v = reinterpret_cast<const float4*>(p)[g4];
            dec[4 * g4] = v.x;
            dec[4 * g4 + 1] = v.y;
            dec[4 * g4 + 2] = v.z;
            dec[4 * g4 + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int g2 = 0; g2 < G / 2; ++g2) {
            const float2 v = reinterpret_cast<const float2*>(p)[g2];
            dec[2 * g2] = v.x;
            dec[2 * g2 + 1] = v.y;
        }
    }
}

template <int G, int NP, int KT>
__device__ __forceinline__ void lookup(const float* tab, bool tab_ok, int k, float delta,
                                       const float (&A2)[G], int q, float (&dec)[G]) {
    if (tab_ok && k >= 1 && k <= KT) {
        table_row<G>(tab + (k - 1) * NP + q * G, dec);
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) dec[g] = decay_fast(delta, A2[g]);
    }
}

// Per-lane constants of the depthwise scan.
template <int G>
struct DwParams {
    float A2[G], Ar[G], WB[G], WC[G], cc[G];
    float dti, dta, Dv;
    float dclamp;   // delta above this may hit the +-126 exponent clamp
    float dlim;     // the fast forward path takes events with delta <= dlim
};

template <int G>
__device__ __forceinline__ void load_params(DwParams<G>& P, const ScanArgs& a, bool ok, int d, int q) {
    float amax = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        const bool o = ok && s < a.dstate;
        P.Ar[g] = o ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
        P.A2[g] = (float)((double)P.Ar[g] * 1.4426950408889634);
        P.WB[g] = o ? a.B[d * a.dstate + s] : 0.f;
        P.WC[g] = o ? a.C[d * a.dstate + s] : 0.f;
        P.cc[g] = P.WB[g] * P.WC[g];
        amax = fmaxf(amax, fabsf(P.A2[g]));
    }
    P.dti = ok ? a.dt_idle[d] : 0.f;
    P.dta = ok ? a.dt_active[d] : 0.f;
    P.Dv = (ok && a.D) ? a.D[d] : 0.f;
    P.dclamp = amax > 0.f ? 126.0f / amax : INFINITY;
    // With dt_idle, dt_active >= 0 and every A <= 0 each exponent delta*A is
    // <= 0, so a clamp at -126 leaves the chunk product prod(a) at or below
    // 2^-126 whether or not the clamp is applied: the fast forward path skips
    // those corrections.  Otherwise it must leave every clamping event to the
    // general path, which applies them exactly.
    bool decaying = P.dti >= 0.f && P.dta >= 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) decaying = decaying && P.A2[g] <= 0.f;
    P.dlim = decaying ? INFINITY : P.dclamp;
}

template <typename T>
__device__ __forceinline__ void load_batch(const T* u, const int32_t* k, int j0, int n,
                                           float (&uv)[kB], int (&kv)[kB]) {
#pragma unroll
    for (int i = 0; i < kB; ++i) {
        const bool ok = j0 + i < n;
        uv[i] = ok ? to_f32<T>(u[j0 + i]) : 0.f;
        kv[i] = ok ? k[j0 + i] : 1;
    }
}

// ============================================================ forward ====
// A batch of kB events takes the fast path when, for every lane of the warp,
// all kB events are valid, every decay is a table hit, no exponent can clamp
// and no chunk state is due in the batch; the general path handles the rest.
template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kWPB * 32)
dw_fwd_v2(ScanArgs a, int bn, int dmajor) {
    using Ly = DwL<G, LPC>;
    constexpr int NP = Ly::NP, CPW = Ly::CPW, KT = Ly::KT, EPL = Ly::EPL;
    extern __shared__ float s_tab[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPC, q = lane % LPC;
    const int gid = (blockIdx.x * kWPB + warp) * CPW + grp;
    const bool ch_ok = gid < a.n_channels;
    const int ch = ch_ok ? channel_of(gid, a.dim, bn, dmajor) : 0;
    const int d = ch % a.dim;
    float* tab = s_tab + warp * Ly::TABLE;
    const int d_tab = __shfl_sync(kFull, d, 0);
    build_table<NP, KT>(tab, a, d_tab, lane);
    const bool tab_ok = d == d_tab;
    const float* tq = tab + q * G;

    DwParams<G> P;
    load_params<G>(P, a, ch_ok, d, q);
    const int N = a.dstate;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int n_warp = group_max_warp<LPC>(n);
    const T* u = static_cast<const T*>(a.u) + beg;
    const int32_t* kk = a.k + beg;
    T* out = static_cast<T*>(a.out) + beg;

    float eta[G], corr[G];
#pragma unroll
    for (int g = 0; g < G; ++g) eta[g] = corr[g] = 0.f;
    float sdel = 0.f;

    float uN[kB];
    int kN[kB];
    load_batch<T>(u, kk, 0, n, uN, kN);
    for (int j0 = 0; j0 < n_warp; j0 += kB) {
        float uv[kB], dl[kB];
        int kv[kB];
#pragma unroll
        for (int i = 0; i < kB; ++i) { uv[i] = uN[i]; kv[i] = kN[i]; }
        if (j0 + kB < n_warp) load_batch<T>(u, kk, j0 + kB, n, uN, kN);
        bool fast_lane = tab_ok && (j0 + kB < n) && ((j0 + kB) % kChunkX != 0);
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            dl[i] = event_delta(P.dti, P.dta, kv[i]);
            fast_lane = fast_lane && ((unsigned)(kv[i] - 1) < (unsigned)KT) && !(dl[i] > P.dlim);
        }
        float acc[kB];
        if (__all_sync(kFull, fast_lane)) {
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const float w = dl[i] * uv[i] * uv[i];
                float dec[G];
                table_row<G>(tq + (kv[i] - 1) * NP, dec);
                float s = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    eta[g] = fmaf(dec[g], eta[g], w);
                    s = fmaf(P.cc[g], eta[g], s);
                }
                acc[i] = s;
                sdel += dl[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                const int j = j0 + i;
                const bool ok = j < n;
                const float delta = dl[i];
                const float w = ok ? delta * uv[i] * uv[i] : 0.f;
                float dec[G];
                lookup<G, NP, KT>(tab, tab_ok, kv[i], delta, P.A2, q, dec);
                float s = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    eta[g] = fmaf(ok ? dec[g] : 1.f, eta[g], w);
                    s = fmaf(P.cc[g], eta[g], s);
                }
                acc[i] = s;
                if (ok) {
                    sdel += delta;
                    if (delta > P.dclamp) {
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float x = delta * P.A2[g];
                            corr[g] += fmaxf(fminf(x, 126.0f), -126.0f) - x;
                        }
                    }
                    if ((j + 1) % kChunkX == 0 || j == n - 1) {
                        const int c = j / kChunkX;
                        if (c < a.n_chunks) {
                            float* xo = a.x + ((int64_t)ch * a.n_chunks + c) * 2 * N;
#pragma unroll
                            for (int g = 0; g < G; ++g) {
                                const int st = q * G + g;
                                if (st < N) {
                                    xo[2 * st] = exp2f(fmaf(P.A2[g], sdel, corr[g]));
                                    xo[2 * st + 1] = P.WB[g] * eta[g];
                                }
                            }
                        }
                    }
                }
            }
        }
        group_transpose_sum<LPC, kB>(acc, q);
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            if (i / EPL == q) {
                const int j = j0 + i;
                if (j < n) {
                    const float y = fmaf(P.Dv, uv[i], uv[i] * acc[i % EPL]);
                    out[j] = from_f32<T>(y);
                    if (a.z != nullptr) {
                        const float zv = to_f32<T>(static_cast<const T*>(a.z)[beg + j]);
                        static_cast<T*>(a.out_z)[beg + j] = from_f32<T>(y * silu(zv));
                    }
                }
            }
        }
    }
}

// =========================================================== backward ====
template <typename T>
__device__ __forceinline__ void load_tile(const ScanArgs& a, const T* u, const int32_t* kk,
                                          const T* dout, int beg, int jb, int cnt, bool writer,
                                          float (&uv)[kB], int (&kv)[kB], float (&dv)[kB]) {
#pragma unroll
    for (int i = 0; i < kB; ++i) {
        const bool ok = i < cnt;
        uv[i] = ok ? to_f32<T>(u[jb + i]) : 0.f;
        kv[i] = ok ? kk[jb + i] : 1;
        dv[i] = ok ? to_f32<T>(dout[jb + i]) : 0.f;
    }
    if (a.z != nullptr) {
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            if (i < cnt) {
                const int e = beg + jb + i;
                const float zv = to_f32<T>(static_cast<const T*>(a.z)[e]);
                const float sg = 1.0f / (1.0f + expf(-zv));
                if (writer) {
                    const float ov = to_f32<T>(static_cast<const T*>(a.out_fwd)[e]);
                    static_cast<T*>(a.dz)[e] = from_f32<T>(dv[i] * ov * sg * (1.0f + zv * (1.0f - sg)));
                }
                dv[i] = dv[i] * (zv * sg);
            }
        }
    }
}

template <int G>
__device__ __forceinline__ void ckpt_put(float* p, const float (&v)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4)
            *reinterpret_cast<float4*>(p + g) = make_float4(v[g], v[g + 1], v[g + 2], v[g + 3]);
    } else {
#pragma unroll
        for (int g = 0; g < G; g += 2) *reinterpret_cast<float2*>(p + g) = make_float2(v[g], v[g + 1]);
    }
}

template <int G>
__device__ __forceinline__ void ckpt_get(const float* p, float (&v)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4) {
            const float4 t = *reinterpret_cast<const float4*>(p + g);
            v[g] = t.x; v[g + 1] = t.y; v[g + 2] = t.z; v[g + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int g = 0; g < G; g += 2) {
            const float2 t = *reinterpret_cast<const float2*>(p + g);
            v[g] = t.x; v[g + 1] = t.y;
        }
    }
}

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(kWPB * 32, 2)
dw_bwd_v2(ScanArgs a, int bn, int dmajor) {
    using Ly = DwL<G, LPC>;
    constexpr int NP = Ly::NP, CPW = Ly::CPW, KT = Ly::KT, EPL = Ly::EPL;
    extern __shared__ float s_tab[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPC, q = lane % LPC;
    const int gid = (blockIdx.x * kWPB + warp) * CPW + grp;
    const bool ch_ok = gid < a.n_channels;
    const int ch = ch_ok ? channel_of(gid, a.dim, bn, dmajor) : 0;
    const int d = ch % a.dim;
    float* tab = s_tab + warp * Ly::TABLE;
    const int d_tab = __shfl_sync(kFull, d, 0);
    build_table<NP, KT>(tab, a, d_tab, lane);
    const bool tab_ok = d == d_tab;
    const float* tq = tab + q * G;

    DwParams<G> P;
    load_params<G>(P, a, ch_ok, d, q);
    float ccA[G];
#pragma unroll
    for (int g = 0; g < G; ++g) ccA[g] = P.cc[g] * P.Ar[g];
    const int N = a.dstate;
    const int beg = ch_ok ? a.cu[ch] : 0;
    const int n = ch_ok ? a.cu[ch + 1] - beg : 0;
    const int nch = (n + kChunkX - 1) / kChunkX;
    const int nch_warp = group_max_warp<LPC>(nch);
    const T* u = static_cast<const T*>(a.u) + beg;
    const int32_t* kk = a.k + beg;
    const T* dout = static_cast<const T*>(a.dout) + beg;
    T* du = static_cast<T*>(a.du) + beg;
    float* ck = a.ws_ckpt + ((int64_t)(beg >> 3) + ch) * NP + q * G;

    // Parameter-gradient sums: per-tile partials are added into per-chunk
    // sums (at most 256 tiles), which are added into the totals at the end
    // of each chunk, so no fp32 sum runs over more than 256 terms.
    float gam[G], anx[G], SA[G], SB[G], QE[G], cA[G], cB[G], cQ[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        gam[g] = 0.f; anx[g] = 1.f;
        SA[g] = SB[g] = QE[g] = 0.f;
    }
    float s_ddi = 0.f, s_dda = 0.f, s_dD = 0.f;

    for (int c = nch_warp - 1; c >= 0; --c) {
        const bool c_ok = c < nch;
        const int cs = c * kChunkX;
        const int len = c_ok ? min(n - cs, kChunkX) : 0;
        const int len_warp = group_max_warp<LPC>(len);
#pragma unroll
        for (int g = 0; g < G; ++g) cA[g] = cB[g] = cQ[g] = 0.f;
        float c_ddi = 0.f, c_dda = 0.f, c_dD = 0.f;
        // ---- pass 1: state every kB events of the chunk -> workspace --------
        float eta[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            eta[g] = 0.f;
            if (c_ok && c > 0 && c - 1 < a.n_chunks && q * G + g < N) {
                const float hv = a.x[((int64_t)ch * a.n_chunks + c - 1) * 2 * N + 2 * (q * G + g) + 1];
                eta[g] = (P.WB[g] != 0.f) ? hv / P.WB[g] : 0.f;
            }
        }
        {
            float uN[kB];
            int kN[kB];
            load_batch<T>(u + cs, kk + cs, 0, len, uN, kN);
            for (int j0 = 0; j0 < len_warp; j0 += kB) {
                if (j0 < len) ckpt_put<G>(ck + (int64_t)(j0 / kB) * NP, eta);
                float uv[kB];
                int kv[kB];
#pragma unroll
                for (int i = 0; i < kB; ++i) { uv[i] = uN[i]; kv[i] = kN[i]; }
                if (j0 + kB < len_warp) load_batch<T>(u + cs, kk + cs, j0 + kB, len, uN, kN);
                bool fast_lane = tab_ok && (j0 + kB <= len);
#pragma unroll
                for (int i = 0; i < kB; ++i) fast_lane = fast_lane && ((unsigned)(kv[i] - 1) < (unsigned)KT);
                if (__all_sync(kFull, fast_lane)) {
#pragma unroll
                    for (int i = 0; i < kB; ++i) {
                        const float w = event_delta(P.dti, P.dta, kv[i]) * uv[i] * uv[i];
                        float dec[G];
                        table_row<G>(tq + (kv[i] - 1) * NP, dec);
#pragma unroll
                        for (int g = 0; g < G; ++g) eta[g] = fmaf(dec[g], eta[g], w);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < kB; ++i) {
                        const bool ok = j0 + i < len;
                        const float delta = event_delta(P.dti, P.dta, kv[i]);
                        const float w = ok ? delta * uv[i] * uv[i] : 0.f;
                        float dec[G];
                        lookup<G, NP, KT>(tab, tab_ok, kv[i], delta, P.A2, q, dec);
#pragma unroll
                        for (int g = 0; g < G; ++g) eta[g] = fmaf(ok ? dec[g] : 1.f, eta[g], w);
                    }
                }
            }
        }
        // ---- pass 2: tiles last to first --------------------------------------
        const int nt = (len + kB - 1) / kB;
        const int nt_warp = group_max_warp<LPC>(nt);
        float uN[kB], dN[kB], eN[G];
        int kN[kB];
        {
            const int m = nt_warp - 1;
            const int jb = cs + m * kB;
            const int cnt = (m >= 0 && m < nt) ? min(kB, cs + len - jb) : 0;
            load_tile<T>(a, u, kk, dout, beg, jb, cnt, q == 0, uN, kN, dN);
#pragma unroll
            for (int g = 0; g < G; ++g) eN[g] = 0.f;
            if (cnt > 0) ckpt_get<G>(ck + (int64_t)m * NP, eN);
        }
        for (int m = nt_warp - 1; m >= 0; --m) {
            const int jb = cs + m * kB;
            const int cnt = (m < nt) ? min(kB, cs + len - jb) : 0;
            float uv[kB], dv[kB], et[G], e0[G];
            int kv[kB];
#pragma unroll
            for (int i = 0; i < kB; ++i) { uv[i] = uN[i]; kv[i] = kN[i]; dv[i] = dN[i]; }
#pragma unroll
            for (int g = 0; g < G; ++g) et[g] = e0[g] = eN[g];
            if (m > 0) {  // prefetch the previous tile
                const int jp = jb - kB;
                const int cp = (m - 1 < nt) ? min(kB, cs + len - jp) : 0;
                load_tile<T>(a, u, kk, dout, beg, jp, cp, q == 0, uN, kN, dN);
                if (cp > 0) ckpt_get<G>(ck + (int64_t)(m - 1) * NP, eN);
                else {
#pragma unroll
                    for (int g = 0; g < G; ++g) eN[g] = 0.f;
                }
            }
            bool fast_lane = tab_ok && cnt == kB;
#pragma unroll
            for (int i = 0; i < kB; ++i) fast_lane = fast_lane && ((unsigned)(kv[i] - 1) < (unsigned)KT);
            const bool fast = __all_sync(kFull, fast_lane);
            float tSA[G], tSB[G], tQE[G];
#pragma unroll
            for (int g = 0; g < G; ++g) tSA[g] = tSB[g] = tQE[g] = 0.f;
            float eti[kB][G], teta[kB], tgam[kB], tdA[kB];
            if (fast) {
#pragma unroll
                for (int i = 0; i < kB; ++i) {
                    const float w = event_delta(P.dti, P.dta, kv[i]) * uv[i] * uv[i];
                    const float qv = dv[i] * uv[i];
                    float dec[G];
                    table_row<G>(tq + (kv[i] - 1) * NP, dec);
                    float te = 0.f;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        et[g] = fmaf(dec[g], et[g], w);
                        eti[i][g] = et[g];
                        te = fmaf(P.cc[g], et[g], te);
                        tQE[g] = fmaf(qv, et[g], tQE[g]);
                    }
                    teta[i] = te;
                }
#pragma unroll
                for (int i = kB - 1; i >= 0; --i) {
                    const float delta = event_delta(P.dti, P.dta, kv[i]);
                    const float w = delta * uv[i] * uv[i];
                    const float qv = dv[i] * uv[i];
                    float dec[G];
                    table_row<G>(tq + (kv[i] - 1) * NP, dec);
                    float tg = 0.f, ta = 0.f;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        gam[g] = fmaf(anx[g], gam[g], qv);
                        // gam * (eta_i - w_i) as gam * a_i * eta_{i-1} (no cancellation)
                        const float pr = gam[g] * (dec[g] * (i > 0 ? eti[i > 0 ? i - 1 : 0][g] : e0[g]));
                        tSA[g] = fmaf(pr, delta, tSA[g]);
                        ta = fmaf(ccA[g], pr, ta);
                        tSB[g] = fmaf(gam[g], w, tSB[g]);
                        tg = fmaf(P.cc[g], gam[g], tg);
                        anx[g] = dec[g];
                    }
                    tgam[i] = tg;
                    tdA[i] = ta;
                }
            } else {
#pragma unroll
                for (int i = 0; i < kB; ++i) {
                    const bool ok = i < cnt;
                    const float delta = event_delta(P.dti, P.dta, kv[i]);
                    const float w = ok ? delta * uv[i] * uv[i] : 0.f;
                    const float qv = dv[i] * uv[i];
                    float dec[G];
                    lookup<G, NP, KT>(tab, tab_ok, kv[i], delta, P.A2, q, dec);
                    float te = 0.f;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        et[g] = fmaf(ok ? dec[g] : 1.f, et[g], w);
                        eti[i][g] = et[g];
                        te = fmaf(P.cc[g], et[g], te);
                        tQE[g] = fmaf(qv, et[g], tQE[g]);
                    }
                    teta[i] = te;
                }
#pragma unroll
                for (int i = kB - 1; i >= 0; --i) {
                    const bool ok = i < cnt;
                    const float delta = event_delta(P.dti, P.dta, kv[i]);
                    const float w = delta * uv[i] * uv[i];
                    const float qv = dv[i] * uv[i];
                    float tg = 0.f, ta = 0.f;
                    if (ok) {
                        float dec[G];
                        lookup<G, NP, KT>(tab, tab_ok, kv[i], delta, P.A2, q, dec);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            gam[g] = fmaf(anx[g], gam[g], qv);
                            const float pr = gam[g] * (dec[g] * (i > 0 ? eti[i > 0 ? i - 1 : 0][g] : e0[g]));
                            tSA[g] = fmaf(pr, delta, tSA[g]);
                            ta = fmaf(ccA[g], pr, ta);
                            tSB[g] = fmaf(gam[g], w, tSB[g]);
                            tg = fmaf(P.cc[g], gam[g], tg);
                            anx[g] = dec[g];
                        }
                    }
                    tgam[i] = tg;
                    tdA[i] = ta;
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                cA[g] += tSA[g];
                cB[g] += tSB[g];
                cQ[g] += tQE[g];
            }
            group_transpose_sum<LPC, kB>(teta, q);
            group_transpose_sum<LPC, kB>(tgam, q);
            group_transpose_sum<LPC, kB>(tdA, q);
            float t_ddi = 0.f, t_dda = 0.f, t_dD = 0.f;
#pragma unroll
            for (int i = 0; i < kB; ++i) {
                if (i / EPL == q && i < cnt) {
                    const int e = i % EPL;
                    const float delta = event_delta(P.dti, P.dta, kv[i]);
                    const float duv = fmaf(P.Dv, dv[i], fmaf(2.f * uv[i] * delta, tgam[e], dv[i] * teta[e]));
                    du[jb + i] = from_f32<T>(duv);
                    const float ddel = fmaf(uv[i] * uv[i], tgam[e], tdA[e]);
                    t_ddi = fmaf(ddel, (float)(kv[i] - 1), t_ddi);
                    t_dda += ddel;
                    t_dD = fmaf(dv[i], uv[i], t_dD);
                }
            }
            c_ddi += t_ddi;
            c_dda += t_dda;
            c_dD += t_dD;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            SA[g] += cA[g];
            SB[g] += cB[g];
            QE[g] += cQ[g];
        }
        s_ddi += c_ddi;
        s_dda += c_dda;
        s_dD += c_dD;
    }
    // per-channel partials; the scalar sums are spread over the group's lanes
    const float r_ddi = group_sum<LPC>(s_ddi);
    const float r_dda = group_sum<LPC>(s_dda);
    const float r_dD = group_sum<LPC>(s_dD);
    if (!ch_ok) return;
    float* part = a.ws_part + (int64_t)ch * a.part_stride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        if (s < N) {
            part[s] = P.cc[g] * SA[g];
            part[NP + s] = P.WC[g] * SB[g];
            part[2 * NP + s] = P.WB[g] * QE[g];
        }
    }
    if (q == 0) {
        part[3 * NP] = r_ddi;
        part[3 * NP + 1] = r_dda;
        part[3 * NP + 2] = r_dD;
    }
}

template <int G, int LPC>
int dw_grid(const ScanArgs& a) {
    constexpr int CPB = kWPB * DwL<G, LPC>::CPW;
    return ceil_div(a.n_channels, CPB);
}

template <typename T, int G, int LPC>
bcm_status launch_dw_tl(const ScanArgs& a, bool bwd, cudaStream_t st) {
    const int bn = (a.n_channels % a.dim == 0) ? a.n_channels / a.dim : 0;
    const int dmajor = bn > 0 ? 1 : 0;
    const size_t smem = (size_t)kWPB * DwL<G, LPC>::TABLE * sizeof(float);
    if (bwd) dw_bwd_v2<T, G, LPC><<<dw_grid<G, LPC>(a), kWPB * 32, smem, st>>>(a, bn, dmajor);
    else dw_fwd_v2<T, G, LPC><<<dw_grid<G, LPC>(a), kWPB * 32, smem, st>>>(a, bn, dmajor);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T>
bcm_status launch_dw_t(const ScanArgs& a, bool bwd, cudaStream_t st) {
    const int N = a.dstate;
    // States per lane: more states give each lane more independent recurrences
    // (instruction-level parallelism), fewer give more warps.  BCM_SCAN_LPC
    // (lanes per channel) overrides the default for tuning.
    static const int lpc_env = [] {
        const char* e = getenv("BCM_SCAN_LPC");
        return e ? atoi(e) : 0;
    }();
    if (N <= 16) {
        const int lpc = lpc_env ? lpc_env : 4;
        if (N <= 8) {
            if (lpc >= 4) return launch_dw_tl<T, 2, 4>(a, bwd, st);
            if (lpc == 2) return launch_dw_tl<T, 4, 2>(a, bwd, st);
            return launch_dw_tl<T, 8, 1>(a, bwd, st);
        }
        if (lpc >= 8) return launch_dw_tl<T, 2, 8>(a, bwd, st);
        if (lpc == 4) return launch_dw_tl<T, 4, 4>(a, bwd, st);
        if (lpc == 2) return launch_dw_tl<T, 8, 2>(a, bwd, st);
        return bwd ? launch_dw_tl<T, 8, 2>(a, bwd, st) : launch_dw_tl<T, 16, 1>(a, bwd, st);
    }
    if (N <= 32) return launch_dw_tl<T, 4, 8>(a, bwd, st);
    return launch_dw_tl<T, 8, 8>(a, bwd, st);
}

}  // namespace

// Fast depthwise path for dstate <= 64.  The backward uses the same
// checkpoint / partial workspace layout as scan_bwd.cu with NP = G*LPC.
bool dw_fast_supported(int dstate) { return dstate <= 64; }

int dw_fast_np(int dstate) {
    if (dstate <= 8) return 8;
    if (dstate <= 16) return 16;
    if (dstate <= 32) return 32;
    return 64;
}

bcm_status dw_fast_launch(const ScanArgs& a, bcm_dtype dtype, bool bwd, cudaStream_t st) {
    if (v3_supported(a, bwd)) return v3_launch(a, dtype, bwd, st);
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        return launch_dw_t<T>(a, bwd, st);
    });
}

}  // namespace bcm
