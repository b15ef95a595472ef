// s6_dense.cu — the dense selective scan (Mamba's S6), real weights: the
// comparison denominator of the event path.  Semantics of the reference's
// selective_scan_cuda.fwd/bwd (csrc/selective_scan/selective_scan.cpp:
// 403-669; selective_scan_fwd_kernel.cuh:84-326 for the forward and its
// chunk states, selective_scan_bwd_kernel.cuh:31-500 for the gradients).
//
// Layout (ours).  A lane group of LPC lanes owns one channel (b, d); lane q
// holds states q*G .. q*G+G-1 of it, so a warp walks 32/LPC channels in
// lockstep over positions, each state a register recurrence.  Positions are
// staged 32 at a time: lane = position loads each channel's u, delta (and
// for variable B/C each state's row of B, C) with coalesced loads, and forms
// delta' = softplus(delta + bias) and delta'*u once per position; the state
// lanes read them back from shared memory.  The output's sum over states is
// a transposed reduction over the group's lanes once per 32 positions.
// The backward re-runs the recurrence from position 0, saving the state
// entering every 8-position tile in its workspace, then walks batches and
// tiles last to first, recomputing each tile's states into registers; sums
// over the channels of a group (variable dB, dC) and over the batch (dA,
// fixed dB / dC, dD, ddelta_bias) are fp32 atomics, as in the reference.
#include <map>
#include <mutex>

#include "scan_common.cuh"

namespace bcm {
namespace {

constexpr int kT6 = 32;      // positions per staged batch
constexpr int kTile6 = 8;    // positions per backward tile
constexpr int kP6 = kT6 + 1; // staging pitch

struct S6 {
    int batch, dim, L, N, groups, n_chunks, hpg;   // hpg = channels per group
    bool varB, varC, softplus;
    const void* u; int64_t u_sb, u_sd;
    const void* delta; int64_t dl_sb, dl_sd;
    const float* A; int64_t A_sd, A_sn;
    const void* B; int64_t B_sd, B_sn;
    const void* C; int64_t C_sd, C_sn;
    const float* D; const float* bias; const void* z;
    void* out; void* out_z; float* x;
    const void* dout; const void* out_fwd;
    void* du; void* ddelta; float* dA; float* dB; float* dC; float* dD; float* dbias; void* dz;
    float* ck;   // backward: state entering every tile, [channel][tile][NP]
};

__device__ __forceinline__ float softplus20(float v) { return v <= 20.f ? log1pf(expf(v)) : v; }
__device__ __forceinline__ float s6_decay(float dl, float A2) {
    return exp2f(fmaxf(fminf(dl * A2, 126.0f), -126.0f));
}

// Shared memory of one warp: per channel rows of delta', delta'*u, u, a
// fourth row (forward: output; backward: gated dout) and a fifth (backward:
// the softplus derivative), then the B and C tiles [CPW][N][kP6] when
// variable and (backward) tiles of the same shape for their gradients.
template <int CPW>
__host__ __device__ constexpr int s6_rows_floats() { return 5 * CPW * kP6; }
__host__ __device__ inline int s6_warp_floats(int cpw, int N, bool varB, bool varC, bool bwd = false) {
    const int tiles = (varB ? 1 : 0) + (varC ? 1 : 0);
    return (5 * cpw * kP6 + (bwd ? 2 : 1) * tiles * cpw * N * kP6 + 3) / 4 * 4;
}

// Stage positions t0 .. t0+31 of the warp's channels (lane = position).
template <typename T, int CPW, bool BWD>
__device__ __forceinline__ void s6_stage(const S6& p, const int64_t (&chb)[CPW], const int (&chd)[CPW],
                                         int t0, int lane, float* sw) {
    float* s_dl = sw;
    float* s_dlu = sw + CPW * kP6;
    float* s_u = sw + 2 * CPW * kP6;
    float* s_4 = sw + 3 * CPW * kP6;
    float* s_5 = sw + 4 * CPW * kP6;
    float* s_B = sw + 5 * CPW * kP6;
    float* s_C = s_B + (p.varB ? CPW * p.N * kP6 : 0);
    const int t = t0 + lane;
    const bool ok = t < p.L;
#pragma unroll
    for (int j = 0; j < CPW; ++j) {
        const int64_t b = chb[j];
        const int d = chd[j];
        const bool live = ok && d >= 0;
        float uv = 0.f, dl = 0.f, sg = 1.f;
        if (live) {
            uv = to_f32<T>(static_cast<const T*>(p.u)[b * p.u_sb + d * p.u_sd + t]);
            float raw = to_f32<T>(static_cast<const T*>(p.delta)[b * p.dl_sb + d * p.dl_sd + t]);
            if (p.bias) raw += p.bias[d];
            dl = p.softplus ? softplus20(raw) : raw;
            if (BWD && p.softplus) sg = raw <= 20.f ? 1.f / (1.f + expf(-raw)) : 1.f;
        }
        s_dl[j * kP6 + lane] = dl;
        s_dlu[j * kP6 + lane] = dl * uv;
        s_u[j * kP6 + lane] = uv;
        if (BWD) {
            const int64_t e = (b * p.dim + d) * (int64_t)p.L + t;
            float dy = 0.f;
            if (live) {
                dy = to_f32<T>(static_cast<const T*>(p.dout)[e]);
                if (p.z != nullptr) {
                    const float zv = to_f32<T>(static_cast<const T*>(p.z)[e]);
                    const float zs = 1.0f / (1.0f + expf(-zv));
                    const float ov = to_f32<T>(static_cast<const T*>(p.out_fwd)[e]);
                    static_cast<T*>(p.dz)[e] = from_f32<T>(dy * ov * zs * (1.0f + zv * (1.0f - zs)));
                    if (p.out_z != nullptr) static_cast<T*>(p.out_z)[e] = from_f32<T>(ov * zv * zs);
                    dy *= zv * zs;
                }
            }
            s_4[j * kP6 + lane] = dy;
            s_5[j * kP6 + lane] = sg;
        }
        if (p.varB || p.varC) {
            const int g = d >= 0 ? d / p.hpg : 0;
            const int64_t row0 = ((b * p.groups + g) * (int64_t)p.N) * p.L + t;
            for (int s = 0; s < p.N; ++s) {
                if (p.varB)
                    s_B[(j * p.N + s) * kP6 + lane] =
                        live ? to_f32<T>(static_cast<const T*>(p.B)[row0 + (int64_t)s * p.L]) : 0.f;
                if (p.varC)
                    s_C[(j * p.N + s) * kP6 + lane] =
                        live ? to_f32<T>(static_cast<const T*>(p.C)[row0 + (int64_t)s * p.L]) : 0.f;
            }
        }
    }
}

// Sum v[0..NE) over the LPC lanes of a group: afterwards lane q holds the
// total of entry (q % NE) * max(1, NE / LPC) + e in v[e], e < max(1, NE / LPC).
template <int LPC, int NE>
__device__ __forceinline__ void s6_group_reduce(float (&v)[NE], int q) {
    if constexpr (LPC > NE) {
#pragma unroll
        for (int off = LPC / 2; off >= NE; off >>= 1) {
#pragma unroll
            for (int e = 0; e < NE; ++e) v[e] += __shfl_xor_sync(kFull, v[e], off);
        }
        group_transpose_sum<NE, NE>(v, q % NE);
    } else {
        group_transpose_sum<LPC, NE>(v, q);
    }
}

// Channel of group slot j of warp w (d = -1 past the last channel).
template <int CPW>
__device__ __forceinline__ void s6_channels(const S6& p, int64_t warp_id, int64_t (&chb)[CPW], int (&chd)[CPW]) {
    const int64_t nch = (int64_t)p.batch * p.dim;
#pragma unroll
    for (int j = 0; j < CPW; ++j) {
        const int64_t c = warp_id * CPW + j;
        chb[j] = c < nch ? c / p.dim : 0;
        chd[j] = c < nch ? (int)(c % p.dim) : -1;
    }
}

template <typename T, int G, int LPC>
__global__ void __launch_bounds__(128)
s6_fwd_kernel(S6 p) {
    constexpr int CPW = 32 / LPC;
    constexpr int EPL = kT6 / LPC;   // positions a lane finalises per batch
    extern __shared__ __align__(16) float sm6[];
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp_id * CPW >= (int64_t)p.batch * p.dim) return;   // warp-uniform; no block barrier below
    float* sw = sm6 + (threadIdx.x >> 5) * s6_warp_floats(CPW, p.N, p.varB, p.varC);
    int64_t chb[CPW];
    int chd[CPW];
    s6_channels<CPW>(p, warp_id, chb, chd);
    const int j = lane / LPC, q = lane % LPC;
    const int d = chd[j];
    const int64_t ch = chb[j] * p.dim + (d >= 0 ? d : 0);
    float A2[G], Cf[G], h[G], P[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        const bool ok = d >= 0 && s < p.N;
        A2[g] = ok ? p.A[d * p.A_sd + s * p.A_sn] * kLog2e : 0.f;
        // fixed C (times fixed B): the whole output weight of the state
        float cw = 1.f;
        if (ok && !p.varC) cw = static_cast<const float*>(p.C)[d * p.C_sd + s * p.C_sn];
        if (ok && !p.varB) cw *= static_cast<const float*>(p.B)[d * p.B_sd + s * p.B_sn];
        Cf[g] = ok ? cw : 0.f;
        h[g] = 0.f;
        P[g] = 1.f;
    }
    const float Dv = (p.D && d >= 0) ? p.D[d] : 0.f;
    const float* s_dl = sw;
    const float* s_dlu = sw + CPW * kP6;
    const float* s_u = sw + 2 * CPW * kP6;
    float* s_y = sw + 3 * CPW * kP6;
    const float* s_B = sw + 5 * CPW * kP6;
    const float* s_C = s_B + (p.varB ? CPW * p.N * kP6 : 0);
    for (int t0 = 0; t0 < p.L; t0 += kT6) {
        __syncwarp();
        s6_stage<T, CPW, false>(p, chb, chd, t0, lane, sw);
        __syncwarp();
        float yv[kT6];
#pragma unroll
        for (int i = 0; i < kT6; ++i) {
            const float dl = s_dl[j * kP6 + i], dlu = s_dlu[j * kP6 + i];
            float y0 = 0.f, y1 = 0.f;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int s = q * G + g;
                const int sr = s < p.N ? s : 0;
                const float a = s6_decay(dl, A2[g]);
                const float bb = p.varB ? s_B[(j * p.N + sr) * kP6 + i] * dlu : dlu;
                h[g] = fmaf(a, h[g], bb);
                P[g] *= a;
                const float cw = p.varC ? s_C[(j * p.N + sr) * kP6 + i] * Cf[g] : Cf[g];
                if (g & 1) y1 = fmaf(cw, h[g], y1); else y0 = fmaf(cw, h[g], y0);
            }
            yv[i] = y0 + y1;
            // chunk state after every 2048 positions and after the last one
            const int t = t0 + i;
            if (t < p.L && ((t + 1) % kChunkX == 0 || t + 1 == p.L) && d >= 0) {
                float* xo = p.x + (ch * p.n_chunks + t / kChunkX) * 2 * p.N;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int s = q * G + g;
                    if (s < p.N) {
                        xo[2 * s] = P[g];
                        xo[2 * s + 1] = h[g];
                    }
                }
            }
        }
        s6_group_reduce<LPC, kT6>(yv, q);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const int i = q * EPL + e;
            s_y[j * kP6 + i] = fmaf(Dv, s_u[j * kP6 + i], yv[e]);
        }
        __syncwarp();
        {
            const int t = t0 + lane;
#pragma unroll
            for (int jj = 0; jj < CPW; ++jj) {
                if (t < p.L && chd[jj] >= 0) {
                    const int64_t e = (chb[jj] * p.dim + chd[jj]) * (int64_t)p.L + t;
                    const float y = s_y[jj * kP6 + lane];
                    static_cast<T*>(p.out)[e] = from_f32<T>(y);
                    if (p.z != nullptr) {
                        const float zv = to_f32<T>(static_cast<const T*>(p.z)[e]);
                        static_cast<T*>(p.out_z)[e] = from_f32<T>(y * silu(zv));
                    }
                }
            }
        }
    }
}

// Backward.  Pass 1 re-runs the recurrence and saves the state entering every
// tile of kTile6 positions (p.ck); pass 2 walks batches and tiles last to
// first: per tile the states are recomputed into registers from the saved
// one, then per position (last to first) and state
//   dh = a_{t+1}*dh + C'_t*dy_t,  pr = dh*h_{t-1}*a_t,
//   dA += pr*delta',  ddelta' += pr*A + dh*b'*u,  du += dh*b'*delta'
// (b' = B_t for variable B, else 1), with dB, dC from dh*delta'*u and
// dy*h; the per-position sums over states are reduced over the group's lanes
// once per tile.
template <typename T, int G, int LPC>
__global__ void __launch_bounds__(128)
s6_bwd_kernel(S6 p) {
    constexpr int CPW = 32 / LPC;
    constexpr int NP = G * LPC;
    constexpr int EPT = kTile6 >= LPC ? kTile6 / LPC : 1;   // positions a lane finalises per tile
    extern __shared__ __align__(16) float sm6[];
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp_id * CPW >= (int64_t)p.batch * p.dim) return;   // warp-uniform; no block barrier below
    float* sw = sm6 + (threadIdx.x >> 5) * s6_warp_floats(CPW, p.N, p.varB, p.varC, true);
    int64_t chb[CPW];
    int chd[CPW];
    s6_channels<CPW>(p, warp_id, chb, chd);
    const int j = lane / LPC, q = lane % LPC;
    const int d = chd[j];
    const bool live_ch = d >= 0;
    const int64_t b = chb[j];
    const int dd = live_ch ? d : 0;
    const int64_t ch = b * p.dim + dd;
    const int n_tiles = (p.L + kTile6 - 1) / kTile6;
    float* ckc = p.ck + ch * (int64_t)n_tiles * NP + q * G;
    // per-position gradients of variable B / C for the batch, [CPW][N][kP6]:
    // summed over the channels of one (batch row, group) and added to global
    // memory once per batch with position-coalesced atomics
    float* s_gB = sw + 5 * CPW * kP6 + ((p.varB ? 1 : 0) + (p.varC ? 1 : 0)) * CPW * p.N * kP6;
    float* s_gC = s_gB + (p.varB ? CPW * p.N * kP6 : 0);

    // Cx: fixed C (1 when variable), Bw: fixed B (1 when variable), Cf = Cx*Bw
    // (0 for padding states): the output weight without the variable C factor
    float A2[G], Cf[G], Cx[G], Bw[G], h[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        const bool ok = live_ch && s < p.N;
        A2[g] = ok ? p.A[dd * p.A_sd + s * p.A_sn] * kLog2e : 0.f;
        Cx[g] = (ok && !p.varC) ? static_cast<const float*>(p.C)[dd * p.C_sd + s * p.C_sn] : 1.f;
        Bw[g] = (ok && !p.varB) ? static_cast<const float*>(p.B)[dd * p.B_sd + s * p.B_sn] : 1.f;
        Cf[g] = ok ? Cx[g] * Bw[g] : 0.f;
        h[g] = 0.f;
    }
    const float Dv = (p.D && live_ch) ? p.D[dd] : 0.f;
    float* s_dl = sw;
    float* s_dlu = sw + CPW * kP6;
    const float* s_u = sw + 2 * CPW * kP6;
    const float* s_dy = sw + 3 * CPW * kP6;
    const float* s_sg = sw + 4 * CPW * kP6;
    const float* s_B = sw + 5 * CPW * kP6;
    const float* s_C = s_B + (p.varB ? CPW * p.N * kP6 : 0);
    auto sB = [&](int s, int i) { return p.varB ? s_B[(j * p.N + (s < p.N ? s : 0)) * kP6 + i] : 1.f; };
    auto sC = [&](int s, int i) { return p.varC ? s_C[(j * p.N + (s < p.N ? s : 0)) * kP6 + i] : 1.f; };

    // ---- pass 1: the state entering every tile
    for (int t0 = 0; t0 < p.L; t0 += kT6) {
        __syncwarp();
        s6_stage<T, CPW, false>(p, chb, chd, t0, lane, sw);
        __syncwarp();
#pragma unroll 1
        for (int i = 0; i < kT6; ++i) {
            const int t = t0 + i;
            if (t % kTile6 == 0 && t < p.L && live_ch) {
#pragma unroll
                for (int g = 0; g < G; ++g) ckc[(int64_t)(t / kTile6) * NP + g] = h[g];
            }
            const float dl = s_dl[j * kP6 + i], dlu = s_dlu[j * kP6 + i];
#pragma unroll
            for (int g = 0; g < G; ++g) h[g] = fmaf(s6_decay(dl, A2[g]), h[g], sB(q * G + g, i) * dlu);
        }
    }

    // ---- pass 2: batches and tiles last to first
    float dh[G], anx[G], aA[G], aB[G], aC[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dh[g] = anx[g] = aA[g] = aB[g] = aC[g] = 0.f;
    float aD = 0.f, aBias = 0.f;
    for (int t0 = ((p.L - 1) / kT6) * kT6; t0 >= 0; t0 -= kT6) {
        __syncwarp();
        s6_stage<T, CPW, true>(p, chb, chd, t0, lane, sw);
        __syncwarp();
        float res_du[kT6 / kTile6][EPT], res_dd[kT6 / kTile6][EPT];
#pragma unroll
        for (int tt = kT6 / kTile6 - 1; tt >= 0; --tt) {
            const int i0 = tt * kTile6;
            float tg[kTile6], tu[kTile6];
#pragma unroll
            for (int e = 0; e < kTile6; ++e) tg[e] = tu[e] = 0.f;
            if (t0 + i0 < p.L) {   // warp-uniform
                float hs[G], eti[kTile6][G];
#pragma unroll
                for (int g = 0; g < G; ++g) hs[g] = live_ch ? ckc[(int64_t)((t0 + i0) / kTile6) * NP + g] : 0.f;
#pragma unroll
                for (int ii = 0; ii < kTile6; ++ii) {
                    const int i = i0 + ii;
                    const float dl = s_dl[j * kP6 + i], dlu = s_dlu[j * kP6 + i];
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float prev = ii ? eti[ii - 1][g] : hs[g];
                        eti[ii][g] = fmaf(s6_decay(dl, A2[g]), prev, sB(q * G + g, i) * dlu);
                    }
                }
#pragma unroll
                for (int ii = kTile6 - 1; ii >= 0; --ii) {
                    const int i = i0 + ii;
                    const int t = t0 + i;
                    const float dl = s_dl[j * kP6 + i], dlu = s_dlu[j * kP6 + i];
                    const float uv = s_u[j * kP6 + i], dy = s_dy[j * kP6 + i];
                    float g0 = 0.f, u0 = 0.f;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const int s = q * G + g;
                        const float a = s6_decay(dl, A2[g]);
                        const float hp = ii ? eti[ii - 1][g] : hs[g];
                        const float ht = eti[ii][g];
                        const float cv = sC(s, i);
                        const float bv = sB(s, i);
                        dh[g] = fmaf(anx[g], dh[g], Cf[g] * cv * dy);
                        const float pr = dh[g] * hp * a;
                        aA[g] = fmaf(pr, dl, aA[g]);
                        g0 = fmaf(pr, A2[g], g0);                 // times ln 2 below
                        u0 = fmaf(dh[g], bv, u0);                 // times u (ddelta') and delta' (du)
                        if (p.varB) {
                            if (s < p.N) s_gB[(j * p.N + s) * kP6 + i] = dh[g] * dlu;
                        } else {
                            aB[g] = fmaf(dy * cv * Cx[g], ht, aB[g]);
                        }
                        if (p.varC) {
                            if (s < p.N) s_gC[(j * p.N + s) * kP6 + i] = dy * ht * Bw[g];
                        } else {
                            aC[g] = fmaf(dy * Bw[g], ht, aC[g]);
                        }
                        anx[g] = a;
                    }
                    tg[ii] = fmaf(u0, uv, g0 * 0.69314718055994531f);
                    tu[ii] = u0 * dl;
                }
            }
            s6_group_reduce<LPC, kTile6>(tg, q);
            s6_group_reduce<LPC, kTile6>(tu, q);
#pragma unroll
            for (int e = 0; e < EPT; ++e) {
                res_dd[tt][e] = tg[e];
                res_du[tt][e] = tu[e];
            }
        }
        // finalise the positions this lane owns: lanes q < min(LPC, kTile6)
        // own positions (q % kTile6) * EPT + e of every tile
        __syncwarp();
        if (q < (LPC < kTile6 ? LPC : kTile6)) {
#pragma unroll
            for (int tt = 0; tt < kT6 / kTile6; ++tt) {
#pragma unroll
                for (int e = 0; e < EPT; ++e) {
                    const int i = tt * kTile6 + q * EPT + e;
                    const int t = t0 + i;
                    const float dy = s_dy[j * kP6 + i];
                    const float uv = s_u[j * kP6 + i];
                    const float ddr = res_dd[tt][e] * s_sg[j * kP6 + i];
                    if (t < p.L && live_ch) {
                        aD = fmaf(dy, uv, aD);
                        aBias += ddr;
                    }
                    // outputs staged over the delta' / delta'*u rows (read no more)
                    s_dl[j * kP6 + i] = fmaf(Dv, dy, res_du[tt][e]);
                    s_dlu[j * kP6 + i] = ddr;
                }
            }
        }
        __syncwarp();
        {
            const int t = t0 + lane;
#pragma unroll
            for (int jj = 0; jj < CPW; ++jj) {
                if (t < p.L && chd[jj] >= 0) {
                    const int64_t e = (chb[jj] * p.dim + chd[jj]) * (int64_t)p.L + t;
                    static_cast<T*>(p.du)[e] = from_f32<T>(s_dl[jj * kP6 + lane]);
                    static_cast<T*>(p.ddelta)[e] = from_f32<T>(s_dlu[jj * kP6 + lane]);
                }
            }
            // variable dB / dC: lane = position; the warp's channels of one
            // (batch row, group) summed first, then one coalesced atomic row
            // per state.  Every slot read here was written this batch: the
            // positions of tiles past the sequence end are not read.
            if ((p.varB || p.varC) && t < p.L) {
                for (int s = 0; s < p.N; ++s) {
                    float accB = 0.f, accC = 0.f;
#pragma unroll
                    for (int jj = 0; jj < CPW; ++jj) {
                        if (chd[jj] < 0) break;
                        if (p.varB) accB += s_gB[(jj * p.N + s) * kP6 + lane];
                        if (p.varC) accC += s_gC[(jj * p.N + s) * kP6 + lane];
                        const bool last = jj + 1 == CPW || chd[jj + 1 < CPW ? jj + 1 : jj] < 0 ||
                                          chb[jj + 1 < CPW ? jj + 1 : jj] != chb[jj] ||
                                          chd[jj + 1 < CPW ? jj + 1 : jj] / p.hpg != chd[jj] / p.hpg;
                        if (last) {
                            const int64_t row =
                                ((chb[jj] * p.groups + chd[jj] / p.hpg) * (int64_t)p.N + s) * p.L + t;
                            if (p.varB) atomicAdd(p.dB + row, accB);
                            if (p.varC) atomicAdd(p.dC + row, accC);
                            accB = accC = 0.f;
                        }
                    }
                }
            }
        }
    }
    // ---- batch sums
    if (live_ch) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int s = q * G + g;
            if (s < p.N) {
                atomicAdd(p.dA + dd * p.N + s, aA[g]);
                if (!p.varB) atomicAdd(p.dB + dd * p.N + s, aB[g]);
                if (!p.varC) atomicAdd(p.dC + dd * p.N + s, aC[g]);
            }
        }
    }
    aD = group_sum<LPC>(aD);
    aBias = group_sum<LPC>(aBias);
    if (live_ch && q == 0) {
        if (p.dD) atomicAdd(p.dD + dd, aD);
        if (p.dbias) atomicAdd(p.dbias + dd, aBias);
    }
}

// (G, LPC) of a dstate: one state per lane up to 32 states (LPC the next
// power of two), then 32 lanes with 2, 4 or 8 states each.
inline void s6_layout(int N, int& G, int& LPC) {
    if (N <= 32) {
        G = 1;
        LPC = 1;
        while (LPC < N) LPC <<= 1;
    } else {
        LPC = 32;
        G = N <= 64 ? 2 : N <= 128 ? 4 : 8;
    }
}

template <typename K>
bcm_status s6_smem_optin(K kernel, size_t smem) {
    if (smem <= 48 * 1024) return BCM_OK;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> optin;
    int dev = 0;
    BCM_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
    auto it = optin.find(key);
    if (it == optin.end()) {
        int mx = 0;
        BCM_CUDA_TRY(cudaDeviceGetAttribute(&mx, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        BCM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mx));
        it = optin.emplace(key, mx).first;
    }
    if (smem > (size_t)it->second) {
        set_error("selective_scan: %zu bytes of shared memory exceed the device limit %d", smem, it->second);
        return BCM_ERR_UNSUPPORTED;
    }
    return BCM_OK;
}

template <typename T, int G, int LPC>
bcm_status s6_launch_t(const S6& p, bool bwd, cudaStream_t st) {
    constexpr int CPW = 32 / LPC;
    const int wpb = (p.varB || p.varC) && p.N > 64 ? 1 : 4;
    const int64_t warps = ((int64_t)p.batch * p.dim + CPW - 1) / CPW;
    const int64_t blocks = (warps + wpb - 1) / wpb;
    BCM_REQUIRE(blocks < (1ll << 31), "selective_scan: too many channels");
    const size_t smem = (size_t)wpb * s6_warp_floats(CPW, p.N, p.varB, p.varC, bwd) * sizeof(float);
    if (bwd) {
        bcm_status s = s6_smem_optin(s6_bwd_kernel<T, G, LPC>, smem);
        if (s != BCM_OK) return s;
        s6_bwd_kernel<T, G, LPC><<<(unsigned)blocks, wpb * 32, smem, st>>>(p);
    } else {
        bcm_status s = s6_smem_optin(s6_fwd_kernel<T, G, LPC>, smem);
        if (s != BCM_OK) return s;
        s6_fwd_kernel<T, G, LPC><<<(unsigned)blocks, wpb * 32, smem, st>>>(p);
    }
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T>
bcm_status s6_launch(const S6& p, bool bwd, cudaStream_t st) {
    int G = 1, LPC = 1;
    s6_layout(p.N, G, LPC);
    switch (G * 64 + LPC) {
        case 64 + 1: return s6_launch_t<T, 1, 1>(p, bwd, st);
        case 64 + 2: return s6_launch_t<T, 1, 2>(p, bwd, st);
        case 64 + 4: return s6_launch_t<T, 1, 4>(p, bwd, st);
        case 64 + 8: return s6_launch_t<T, 1, 8>(p, bwd, st);
        case 64 + 16: return s6_launch_t<T, 1, 16>(p, bwd, st);
        case 64 + 32: return s6_launch_t<T, 1, 32>(p, bwd, st);
        case 128 + 32: return s6_launch_t<T, 2, 32>(p, bwd, st);
        case 256 + 32: return s6_launch_t<T, 4, 32>(p, bwd, st);
        default: return s6_launch_t<T, 8, 32>(p, bwd, st);
    }
}

size_t s6_ckpt_bytes(const bcm_s6_args* a) {
    int G = 1, LPC = 1;
    s6_layout((int)a->dstate, G, LPC);
    const int64_t n_tiles = (a->seqlen + kTile6 - 1) / kTile6;
    return align_up((size_t)(a->batch * a->dim) * (size_t)n_tiles * (size_t)(G * LPC) * sizeof(float), 256);
}

bcm_status s6_fill(const bcm_s6_args* a, bool bwd, S6& p) {
    BCM_REQUIRE(a != nullptr, "selective_scan: null args");
    BCM_REQUIRE(a->dtype == BCM_F32 || a->dtype == BCM_F16 || a->dtype == BCM_BF16,
                "selective_scan: u must be float32, float16 or bfloat16");
    BCM_REQUIRE(a->batch >= 1 && a->dim >= 1 && a->seqlen >= 1, "selective_scan: bad sizes");
    BCM_REQUIRE(a->dstate >= 1 && a->dstate <= 256, "selective_scan only supports state dimension <= 256");
    BCM_REQUIRE(a->batch * a->dim < (1ll << 31) && a->seqlen < (1ll << 30), "selective_scan: sizes too large");
    const bool var = a->is_variable_B || a->is_variable_C;
    BCM_REQUIRE(!var || (a->n_groups >= 1 && a->dim % a->n_groups == 0),
                "selective_scan: dim must be a multiple of n_groups");
    BCM_REQUIRE(a->u && a->delta && a->A && a->B && a->C, "selective_scan: null input");
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.L = (int)a->seqlen; p.N = (int)a->dstate;
    p.groups = var ? (int)a->n_groups : 1;
    p.hpg = p.dim / p.groups;
    p.n_chunks = (int)((a->seqlen + kChunkX - 1) / kChunkX);
    p.varB = a->is_variable_B != 0; p.varC = a->is_variable_C != 0; p.softplus = a->delta_softplus != 0;
    p.u = a->u; p.u_sb = a->u_stride_b; p.u_sd = a->u_stride_d;
    p.delta = a->delta; p.dl_sb = a->delta_stride_b; p.dl_sd = a->delta_stride_d;
    p.A = a->A; p.A_sd = a->A_stride_d; p.A_sn = a->A_stride_n;
    p.B = a->B; p.B_sd = a->B_stride_d; p.B_sn = a->B_stride_n;
    p.C = a->C; p.C_sd = a->C_stride_d; p.C_sn = a->C_stride_n;
    p.D = a->D; p.bias = a->delta_bias; p.z = a->z;
    p.out = a->out; p.out_z = a->out_z; p.x = a->x;
    p.dout = a->dout; p.out_fwd = a->out_fwd;
    p.du = a->du; p.ddelta = a->ddelta; p.dA = a->dA; p.dB = a->dB; p.dC = a->dC;
    p.dD = a->dD; p.dbias = a->ddelta_bias; p.dz = a->dz;
    p.ck = nullptr;
    if (!bwd) {
        BCM_REQUIRE(a->out && a->x, "selective_scan fwd: null output");
        BCM_REQUIRE(!a->z || a->out_z, "selective_scan fwd: z given without out_z");
    } else {
        BCM_REQUIRE(a->dout && a->du && a->ddelta && a->dA && a->dB && a->dC, "selective_scan bwd: null output");
        BCM_REQUIRE(!a->z || (a->out_fwd && a->dz), "selective_scan bwd: z needs out and dz");
        BCM_REQUIRE(a->workspace && a->workspace_bytes >= s6_ckpt_bytes(a), "selective_scan bwd: workspace too small");
        p.ck = static_cast<float*>(a->workspace);
    }
    return BCM_OK;
}

}  // namespace
}  // namespace bcm

using namespace bcm;

extern "C" bcm_status bcm_s6_fwd(const bcm_s6_args* args, cudaStream_t stream) {
    clear_error();
    S6 p;
    bcm_status s = s6_fill(args, false, p);
    if (s != BCM_OK) return s;
    return dispatch_dtype(args->dtype, [&](auto tag) -> bcm_status { return s6_launch<decltype(tag)>(p, false, stream); });
}

extern "C" size_t bcm_s6_bwd_workspace_bytes(const bcm_s6_args* args) {
    if (!args || args->batch < 1 || args->dim < 1 || args->seqlen < 1 || args->dstate < 1 || args->dstate > 256)
        return 0;
    return s6_ckpt_bytes(args);
}

extern "C" bcm_status bcm_s6_bwd(const bcm_s6_args* args, cudaStream_t stream) {
    clear_error();
    S6 p;
    bcm_status s = s6_fill(args, true, p);
    if (s != BCM_OK) return s;
    return dispatch_dtype(args->dtype, [&](auto tag) -> bcm_status { return s6_launch<decltype(tag)>(p, true, stream); });
}
