// scan_seg.cu — event-parallel depthwise scan kernels (forward and backward).
//
// Semantics are those of the reference's flat-channel scan with depthwise B/C
// (selective_scan_fwd_kernel.cuh:403-728, selective_scan_bwd_kernel.cuh:
// 635-1169; B_i,s = u_i*W_B[d,s], C_i,s = u_i*W_C[d,s]), written with the
// normalised state eta (h = W_B*eta):
//   eta_i = a_i*eta_{i-1} + w_i,  w_i = delta_i*u_i^2,  y_i = D*u_i + u_i*sum_s cw_s*eta_i,s
// with cw_s = W_B[d,s]*W_C[d,s].  The work is partitioned by EVENTS, not by
// channels, so uneven per-channel counts cost nothing extra:
//
//  * a warp owns a group of `cpw` consecutive batch rows of one feature d and
//    walks the concatenation of their event streams (its "virtual stream") in
//    tiles of 32*R events; lane L owns events [L*R, L*R + R) of a tile;
//  * per state the recurrence is the (a, b) operator (a1,b1)o(a2,b2) =
//    (a2*a1, a2*b1 + b2) (the reference's SSMScanOp, selective_scan_common.h:
//    157-162): each lane folds its R events, a Kogge-Stone warp scan over the
//    32 lane aggregates gives every lane its incoming state, and a channel
//    start carries a = 0, which cuts the chain between channels (h_{-1} = 0);
//    the state leaving a tile is the next tile's carry;
//  * decays come from a per-feature table in shared memory (row k = gap k,
//    exp2 evaluated in double and rounded once; row 0 = 0 for channel starts,
//    the last row = 1 for padding slots); gaps past the table take the same
//    correctly rounded value computed on the spot;
//  * the forward stores the state entering every tile (N floats per 32*R
//    events) so the backward can start each tile without re-running the
//    recurrence before it; the backward walks tiles last to first with a
//    reverse scan for the adjoint gamma_i = a_{i+1}*gamma_{i+1} + g_i*u_i.
//
// Chunk states x[ch, c] = (prod a, h) after each 2048-event chunk, prod a
// over all events of the channel so far (the reference carries it across
// chunks), are written with prod a = exp2(A*log2(e)*sum delta), sum delta =
// dt_idle*(sum k - n) + dt_active*n from an integer segmented scan of the
// gaps; this equals the reference's running product of clamped decays except
// where an event's exponent exceeds +126 (a state growing by 2^126 in one
// step).
#include <stdlib.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "scan_common.cuh"

namespace bcm {

namespace {

constexpr int kSegTR = 258;          // table rows: 0 -> 0 (channel start), 1..256 -> gap k, 257 -> 1 (padding)
constexpr int kSegKMax = 256;        // largest tabulated gap
constexpr int kSegPadRow = 257;
constexpr int kSegMaxCPW = 16;       // batch rows per warp group
constexpr int kSegFwdWarps = 8;
constexpr int kSegBwdWarps = 4;

__device__ __forceinline__ int segpad(int q) { return q + (q >> 5); }

// Largest c in [0, nc) with vs[c] <= p (vs[0] = 0 <= p).  Skips empty channels.
__device__ __forceinline__ int seg_find(const int* vs, int nc, int p) {
    int lo = 0, hi = nc - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (vs[mid] <= p) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Per-feature decay tables tab[d][s][row] (rows as kSegTR).
__global__ void seg_table_kernel(ScanArgs a, float* __restrict__ tab) {
    const int64_t total = (int64_t)a.dim * a.dstate * kSegTR;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i % kSegTR);
        const int64_t ds = i / kSegTR;
        const int s = (int)(ds % a.dstate), d = (int)(ds / a.dstate);
        float v;
        if (row == 0) {
            v = 0.f;
        } else if (row == kSegPadRow) {
            v = 1.f;
        } else {
            const float A2 = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
            v = decay_exact(event_delta(a.dt_idle[d], a.dt_active[d], row), A2);
        }
        tab[i] = v;
    }
}

struct SegGeom {
    int cpw;            // batch rows per warp group
    int groups_per_d;   // warp groups per feature
    int ctas_per_d;     // CTAs per feature
    int warps;          // warps per CTA
};

// Warp-group bookkeeping in shared memory: vs[c] = start of channel c in the
// virtual stream (vs[nc] = total), base[c] = its first flat event, ch[c] its
// logical channel.
struct SegWarp {
    int vs[kSegMaxCPW + 1];
    int base[kSegMaxCPW];
    int ch[kSegMaxCPW];
};

__device__ __forceinline__ void seg_setup(const ScanArgs& a, int d, int b0, int nc, int lane, SegWarp* W) {
    int n = 0;
    if (lane < nc) {
        const int c = (b0 + lane) * a.dim + d;
        const int beg = a.cu[c];
        n = max(0, a.cu[c + 1] - beg);
        W->base[lane] = beg;
        W->ch[lane] = c;
    }
    const int incl = warp_inclusive_sum(n);
    if (lane < nc) W->vs[lane + 1] = incl;
    if (lane == 0) W->vs[0] = 0;
    __syncwarp();
}

// Kogge-Stone inclusive scan of the (a, b) operator over the warp's lanes
// (lane order = event order).
__device__ __forceinline__ void seg_scan_up(float& A, float& B, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float Ao = __shfl_up_sync(kFull, A, off);
        const float Bo = __shfl_up_sync(kFull, B, off);
        if (lane >= off) {
            B = fmaf(A, Bo, B);
            A *= Ao;
        }
    }
}

// Suffix (right-to-left) scan: lane L composes its map gamma_first(L) =
// M_L*gamma_first(L+1) + G_L with the lanes to its right.
__device__ __forceinline__ void seg_scan_down(float& M, float& G, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float Mo = __shfl_down_sync(kFull, M, off);
        const float Go = __shfl_down_sync(kFull, G, off);
        if (lane + off < 32) {
            G = fmaf(M, Go, G);
            M *= Mo;
        }
    }
}

template <int R>
struct SegTile {
    static constexpr int TILE = 32 * R;
    static constexpr int PADT = TILE + TILE / 32;
};

// Floats of one warp's shared-memory region (rounded to 16 bytes).
template <int R>
constexpr int seg_fwd_warp_floats(int N) {
    return (5 * SegTile<R>::PADT + 2 * N + (int)(sizeof(SegWarp) / 4) + 3) / 4 * 4;
}
template <int R>
constexpr int seg_bwd_warp_floats(int N) {
    return (4 * SegTile<R>::PADT + 3 * N + (int)(sizeof(SegWarp) / 4) + 64 * N + 3) / 4 * 4;
}

// =============================================================== forward ====
// CARRY_ONLY: only the state entering every tile (for a backward that was not
// given the forward's carries); no outputs.
template <typename T, int R, bool CARRY_ONLY>
__global__ void __launch_bounds__(32 * kSegFwdWarps)
seg_fwd_kernel(ScanArgs a, const float* __restrict__ gtab, SegGeom g, float* __restrict__ carries) {
    constexpr int TILE = SegTile<R>::TILE;
    constexpr int PADT = SegTile<R>::PADT;
    extern __shared__ __align__(16) float sm[];
    const int N = a.dstate;
    const int d = blockIdx.x / g.ctas_per_d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* tab = sm;
    float* s_cw = tab + N * kSegTR;
    float* s_wb = s_cw + N;
    float* s_A2 = s_wb + N;
    const int head = (N * kSegTR + 3 * N + 3) / 4 * 4;
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < (size_t)(head + g.warps * seg_fwd_warp_floats<R>(N)) * sizeof(float)) return;
    }
    float* wr = sm + head + warp * seg_fwd_warp_floats<R>(N);
    float* su = wr;
    int* sk = reinterpret_cast<int*>(su + PADT);
    int* se = sk + PADT;
    int* sxr = se + PADT;
    float* ssd = reinterpret_cast<float*>(sxr + PADT);
    float* carry = ssd + PADT;                        // [2][N]
    SegWarp* W = reinterpret_cast<SegWarp*>(carry + 2 * N);

    {
        const float* src = gtab + (int64_t)d * N * kSegTR;
        for (int i = threadIdx.x; i < N * kSegTR; i += blockDim.x) tab[i] = src[i];
        for (int s = threadIdx.x; s < N; s += blockDim.x) {
            const float wb = a.B[d * N + s];
            s_cw[s] = wb * a.C[d * N + s];
            s_wb[s] = wb;
            s_A2[s] = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
        }
    }
    __syncthreads();
    const int grp = (blockIdx.x % g.ctas_per_d) * g.warps + warp;
    if (grp >= g.groups_per_d) return;        // no barrier below
    const int Bn = a.n_channels / a.dim;
    const int b0 = grp * g.cpw;
    const int nc = min(g.cpw, Bn - b0);
    seg_setup(a, d, b0, nc, lane, W);
    const int* vs = W->vs;
    const int Ew = vs[nc];
    const float dti = a.dt_idle[d], dta = a.dt_active[d];
    const float Dv = a.D ? a.D[d] : 0.f;
    const T* u = static_cast<const T*>(a.u);
    const int nchk = a.n_chunks;

    if (!CARRY_ONLY) {
        // chunk states past each channel's last chunk are zero
        for (int c = 0; c < nc; ++c) {
            const int n = vs[c + 1] - vs[c];
            const int first = (n + kChunkX - 1) / kChunkX;
            const int cnt = (nchk - first) * 2 * N;
            float* xo = a.x + ((int64_t)W->ch[c] * nchk + first) * 2 * N;
            for (int i = lane; i < cnt; i += 32) xo[i] = 0.f;
        }
    }
    for (int s = lane; s < N; s += 32) carry[s] = 0.f;
    int kc = 0;    // gap sum of the chunk running into the next tile (warp-uniform)
    const int n_tiles = (Ew + TILE - 1) / TILE;
    __syncwarp();

    for (int t = 0; t < n_tiles; ++t) {
        const int p0 = t * TILE;
        float* cin = carry + (t & 1) * N;
        float* cout = carry + ((t + 1) & 1) * N;
        // ---- stage the tile: coalesced along each channel's events
#pragma unroll
        for (int m = 0; m < R; ++m) {
            const int q = m * 32 + lane, p = p0 + q;
            float uv = 0.f;
            int kv = 0, e = -1;
            if (p < Ew) {
                const int c = seg_find(vs, nc, p);
                e = W->base[c] + (p - vs[c]);
                if (e >= 0 && e < a.n_events) {     // a malformed cu_seqlens is skipped, not read past
                    uv = to_f32<T>(u[e]);
                    kv = a.k[e];
                } else {
                    e = -1;
                }
            }
            su[segpad(q)] = uv;
            sk[segpad(q)] = kv;
            se[segpad(q)] = e;
        }
        if (carries != nullptr && t > 0) {
            // the state entering this tile, at slot (first flat event)/TILE + channel
            const int c0 = seg_find(vs, nc, p0);
            const int e0 = W->base[c0] + (p0 - vs[c0]);
            if (e0 >= 0 && e0 < a.n_events) {
                const int64_t slot = (int64_t)e0 / TILE + W->ch[c0];
                for (int s = lane; s < N; s += 32) carries[slot * N + s] = cin[s];
            }
        }
        __syncwarp();

        // ---- this lane's events
        const int q0 = lane * R, pl = p0 + q0;
        float w[R];
        int ix[R], kk[R];
        unsigned exm = 0, cem = 0, hdm = 0;
        {
            int c = seg_find(vs, nc, min(pl, Ew - 1));
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int p = pl + r;
                const float uv = su[segpad(q0 + r)];
                const int kv = sk[segpad(q0 + r)];
                kk[r] = kv;
                if (p < Ew) {
                    while (p >= vs[c + 1]) ++c;
                    const int j = p - vs[c], n = vs[c + 1] - vs[c];
                    const float dl = event_delta(dti, dta, kv);
                    w[r] = dl * uv * uv;
                    const bool hit = (unsigned)(kv - 1) < (unsigned)kSegKMax;
                    ix[r] = (j == 0) ? 0 : (hit ? kv : kSegPadRow);
                    if (j != 0 && !hit) exm |= 1u << r;
                    if (j == 0) hdm |= 1u << r;
                    if (((j + 1) & (kChunkX - 1)) == 0 || j == n - 1) cem |= 1u << r;
                } else {
                    w[r] = 0.f;
                    ix[r] = kSegPadRow;
                    kk[r] = 0;
                }
            }
        }
        // ---- chunk bookkeeping for x: gap sums since the channel's first
        // event (prod a of x runs from the channel start, as the reference's
        // chunk prefix does), segmented at channel starts
        if (!CARRY_ONLY) {
            int v = 0, f = 0;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (hdm >> r & 1) { v = 0; f = 1; }
                v += kk[r];
            }
            int vi = v, fi = f;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int vo = __shfl_up_sync(kFull, vi, off);
                const int fo = __shfl_up_sync(kFull, fi, off);
                if (lane >= off) {
                    if (!fi) vi += vo;
                    fi |= fo;
                }
            }
            int ve = __shfl_up_sync(kFull, vi, 1), fe = __shfl_up_sync(kFull, fi, 1);
            if (lane == 0) { ve = 0; fe = 0; }
            const int kbase = fe ? ve : kc + ve;
            const int v31 = __shfl_sync(kFull, vi, 31), f31 = __shfl_sync(kFull, fi, 31);
            kc = f31 ? v31 : kc + v31;
            if (cem) {
                int K = kbase;
                int c = seg_find(vs, nc, min(pl, Ew - 1));
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (hdm >> r & 1) K = 0;
                    K += kk[r];
                    if (cem >> r & 1) {
                        const int p = pl + r;
                        while (p >= vs[c + 1]) ++c;
                        const int j = p - vs[c];
                        const int cnt = j + 1;
                        const int chunk = j / kChunkX;
                        sxr[segpad(q0 + r)] = chunk < nchk ? W->ch[c] * nchk + chunk : -1;
                        ssd[segpad(q0 + r)] = fmaf(dti, (float)(K - cnt), dta * (float)cnt);
                    }
                }
            }
        }

        // ---- states
        const bool wexact = __any_sync(kFull, exm != 0);
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        for (int s = 0; s < N; ++s) {
            const float* ts = tab + s * kSegTR;
            float av[R];
#pragma unroll
            for (int r = 0; r < R; ++r) av[r] = ts[ix[r]];
            if (wexact && exm) {
                const float A2 = s_A2[s];
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (exm >> r & 1) av[r] = decay_fast(event_delta(dti, dta, kk[r]), A2);
            }
            float A = av[0], Bv = w[0];
#pragma unroll
            for (int r = 1; r < R; ++r) {
                Bv = fmaf(av[r], Bv, w[r]);
                A *= av[r];
            }
            seg_scan_up(A, Bv, lane);
            const float c_in = cin[s];
            // the carries-only pass computes the states exactly as here, so a
            // backward from either pass sees bit-identical carries
            float Ae = __shfl_up_sync(kFull, A, 1), Be = __shfl_up_sync(kFull, Bv, 1);
            if (lane == 0) { Ae = 1.f; Be = 0.f; }
            float eta = fmaf(Ae, c_in, Be);
            const float cw = s_cw[s];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                eta = fmaf(av[r], eta, w[r]);
                acc[r] = fmaf(cw, eta, acc[r]);
                if (!CARRY_ONLY && (cem >> r & 1)) {
                    const int xr = sxr[segpad(q0 + r)];
                    if (xr >= 0) {
                        float* xo = a.x + (int64_t)xr * 2 * N;
                        xo[2 * s] = exp2f(s_A2[s] * ssd[segpad(q0 + r)]);
                        xo[2 * s + 1] = s_wb[s] * eta;
                    }
                }
            }
            const float cnew = __shfl_sync(kFull, eta, 31);
            if (lane == 0) cout[s] = cnew;
        }
        if (!CARRY_ONLY) {
            // ---- outputs y = D*u + u*acc, stored coalesced
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float uv = su[segpad(q0 + r)];
                su[segpad(q0 + r)] = fmaf(Dv, uv, uv * acc[r]);
            }
            __syncwarp();
            T* out = static_cast<T*>(a.out);
#pragma unroll
            for (int m = 0; m < R; ++m) {
                const int q = m * 32 + lane;
                const int e = se[segpad(q)];
                if (e >= 0) out[e] = from_f32<T>(su[segpad(q)]);
            }
        }
        __syncwarp();
    }
}

// ============================================================== backward ====
// Per tile (last to first) and state: forward scan for eta from the tile's
// incoming state, reverse scan for gamma (the adjoint of eta divided by cw)
// from the next tile's outgoing term, then
//   du_i  = D*g_i + g_i*sum_s cw_s*eta_i,s + 2*delta_i*u_i*sum_s cw_s*gamma_i,s
//   dd_i  = u_i^2*sum_s cw_s*gamma_i,s + sum_s cw_s*A_s*gamma_i,s*a_i,s*eta_{i-1},s
//   dA_s  = cw_s*sum_i gamma_i,s*a_i,s*eta_{i-1},s*delta_i
//   dW_B_s = W_C_s*sum_i gamma_i,s*w_i,  dW_C_s = W_B_s*sum_i gamma_i,s*w_i
//   ddt_idle = sum_i dd_i*(k_i - 1), ddt_active = sum_i dd_i, dD = sum_i g_i*u_i
// (sum_i gamma_i*w_i = sum_i g_i*u_i*eta_i: both W gradients use it).
// Parameter sums are per-warp partials, rows grp*dim + d of ws_part, reduced
// over the groups of a feature in a fixed order afterwards.
template <typename T, int R>
__global__ void __launch_bounds__(32 * kSegBwdWarps)
seg_bwd_kernel(ScanArgs a, const float* __restrict__ gtab, SegGeom g, const float* __restrict__ carries) {
    constexpr int TILE = SegTile<R>::TILE;
    constexpr int PADT = SegTile<R>::PADT;
    extern __shared__ __align__(16) float sm[];
    const int N = a.dstate;
    const int d = blockIdx.x / g.ctas_per_d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* tab = sm;
    float* s_cw = tab + N * kSegTR;
    float* s_cwA = s_cw + N;
    float* s_A2 = s_cwA + N;
    const int head = (N * kSegTR + 3 * N + 3) / 4 * 4;
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < (size_t)(head + g.warps * seg_bwd_warp_floats<R>(N)) * sizeof(float)) return;
    }
    float* wr = sm + head + warp * seg_bwd_warp_floats<R>(N);
    float* su = wr;
    int* sk = reinterpret_cast<int*>(su + PADT);
    float* sd = reinterpret_cast<float*>(sk + PADT);
    int* se = reinterpret_cast<int*>(sd + PADT);
    float* gcar = reinterpret_cast<float*>(se + PADT);   // [2][N] gamma terms entering from the next tile
    float* ecar = gcar + 2 * N;                          // [N] state entering the tile
    SegWarp* W = reinterpret_cast<SegWarp*>(ecar + N);
    float2* sacc = reinterpret_cast<float2*>(wr + (seg_bwd_warp_floats<R>(N) - 64 * N));   // [N][32]

    {
        const float* src = gtab + (int64_t)d * N * kSegTR;
        for (int i = threadIdx.x; i < N * kSegTR; i += blockDim.x) tab[i] = src[i];
        for (int s = threadIdx.x; s < N; s += blockDim.x) {
            const float Ar = a.A[d * a.A_sd + s * a.A_sn];
            const float cw = a.B[d * N + s] * a.C[d * N + s];
            s_cw[s] = cw;
            s_cwA[s] = cw * Ar;
            s_A2[s] = (float)((double)Ar * 1.4426950408889634);
        }
    }
    __syncthreads();
    const int grp = (blockIdx.x % g.ctas_per_d) * g.warps + warp;
    if (grp >= g.groups_per_d) return;
    const int Bn = a.n_channels / a.dim;
    const int b0 = grp * g.cpw;
    const int nc = min(g.cpw, Bn - b0);
    seg_setup(a, d, b0, nc, lane, W);
    const int* vs = W->vs;
    const int Ew = vs[nc];
    const float dti = a.dt_idle[d], dta = a.dt_active[d];
    const float Dv = a.D ? a.D[d] : 0.f;
    const T* u = static_cast<const T*>(a.u);
    const T* dout = static_cast<const T*>(a.dout);
    T* du = static_cast<T*>(a.du);

    for (int s = 0; s < N; ++s) sacc[s * 32 + lane] = make_float2(0.f, 0.f);
    const int n_tiles = (Ew + TILE - 1) / TILE;
    for (int s = lane; s < N; s += 32) gcar[(n_tiles & 1) * N + s] = 0.f;
    float l_ddi = 0.f, l_dda = 0.f, l_dD = 0.f;
    __syncwarp();

    for (int t = n_tiles - 1; t >= 0; --t) {
        const int p0 = t * TILE;
        const float* gin = gcar + ((t + 1) & 1) * N;
        float* gout = gcar + (t & 1) * N;
#pragma unroll
        for (int m = 0; m < R; ++m) {
            const int q = m * 32 + lane, p = p0 + q;
            float uv = 0.f, gv = 0.f;
            int kv = 0, e = -1;
            if (p < Ew) {
                const int c = seg_find(vs, nc, p);
                e = W->base[c] + (p - vs[c]);
                if (e >= 0 && e < a.n_events) {
                    uv = to_f32<T>(u[e]);
                    gv = to_f32<T>(dout[e]);
                    kv = a.k[e];
                } else {
                    e = -1;
                }
            }
            su[segpad(q)] = uv;
            sd[segpad(q)] = gv;
            sk[segpad(q)] = kv;
            se[segpad(q)] = e;
        }
        const int c0 = seg_find(vs, nc, p0);
        const int e0 = W->base[c0] + (p0 - vs[c0]);
        if (t > 0 && e0 >= 0 && e0 < a.n_events) {
            const int64_t slot = (int64_t)e0 / TILE + W->ch[c0];
            for (int s = lane; s < N; s += 32) ecar[s] = carries[slot * N + s];
        } else {
            for (int s = lane; s < N; s += 32) ecar[s] = 0.f;
        }
        __syncwarp();

        const int q0 = lane * R, pl = p0 + q0;
        float w[R], qv[R], dl[R];
        int ix[R];
        unsigned exm = 0, lsm = 0;
        {
            int c = seg_find(vs, nc, min(pl, Ew - 1));
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int p = pl + r;
                const float uv = su[segpad(q0 + r)];
                const float gv = sd[segpad(q0 + r)];
                const int kv = sk[segpad(q0 + r)];
                if (p < Ew) {
                    while (p >= vs[c + 1]) ++c;
                    const int j = p - vs[c], n = vs[c + 1] - vs[c];
                    dl[r] = event_delta(dti, dta, kv);
                    w[r] = dl[r] * uv * uv;
                    qv[r] = gv * uv;
                    const bool hit = (unsigned)(kv - 1) < (unsigned)kSegKMax;
                    ix[r] = (j == 0) ? 0 : (hit ? kv : kSegPadRow);
                    if (j != 0 && !hit) exm |= 1u << r;
                    if (j == n - 1) lsm |= 1u << r;
                } else {
                    dl[r] = 0.f;
                    w[r] = 0.f;
                    qv[r] = 0.f;
                    ix[r] = kSegPadRow;
                    lsm |= 1u << r;     // nothing after a padding slot
                }
            }
        }
        const bool wexact = __any_sync(kFull, exm != 0);
        float te[R], tg[R], ta[R];
#pragma unroll
        for (int r = 0; r < R; ++r) te[r] = tg[r] = ta[r] = 0.f;

        for (int s = 0; s < N; ++s) {
            const float* ts = tab + s * kSegTR;
            float av[R];
#pragma unroll
            for (int r = 0; r < R; ++r) av[r] = ts[ix[r]];
            if (wexact && exm) {
                const float A2 = s_A2[s];
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (exm >> r & 1) av[r] = decay_fast(event_delta(dti, dta, sk[segpad(q0 + r)]), A2);
            }
            // forward: incoming state of each lane
            float A = av[0], Bv = w[0];
#pragma unroll
            for (int r = 1; r < R; ++r) {
                Bv = fmaf(av[r], Bv, w[r]);
                A *= av[r];
            }
            seg_scan_up(A, Bv, lane);
            float Ae = __shfl_up_sync(kFull, A, 1), Be = __shfl_up_sync(kFull, Bv, 1);
            if (lane == 0) { Ae = 1.f; Be = 0.f; }
            const float eta_in = fmaf(Ae, ecar[s], Be);
            // reverse: multiplier of event r is the next event's decay (0 after
            // a channel's last event); lane 31's last event takes the term
            // entering from the next tile instead
            const float a_next = __shfl_down_sync(kFull, av[0], 1);
            const float g_in = gin[s];
            float mlast = (lane == 31) ? 1.f : a_next;
            if (lsm >> (R - 1) & 1) mlast = (lane == 31) ? 1.f : 0.f;
            float G = (lane == 31) ? g_in : 0.f;
            float M = (lane == 31) ? 0.f : 1.f;
            G = fmaf(mlast, G, qv[R - 1]);
            M *= mlast;
#pragma unroll
            for (int r = R - 2; r >= 0; --r) {
                const float m = (lsm >> r & 1) ? 0.f : av[r + 1];
                G = fmaf(m, G, qv[r]);
                M *= m;
            }
            seg_scan_down(M, G, lane);
            const float X = __shfl_down_sync(kFull, G, 1);
            // pass 2: states and adjoints of the lane's events
            const float cw = s_cw[s], cwA = s_cwA[s];
            float ap[R];
            float eta = eta_in;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                ap[r] = av[r] * eta;
                eta = ap[r] + w[r];
                te[r] = fmaf(cw, eta, te[r]);
            }
            float gam = (lane == 31) ? g_in : X;
            float SA = 0.f, SB = 0.f;
#pragma unroll
            for (int r = R - 1; r >= 0; --r) {
                const float m = (r == R - 1) ? mlast : ((lsm >> r & 1) ? 0.f : av[r + 1]);
                gam = fmaf(m, gam, qv[r]);
                tg[r] = fmaf(cw, gam, tg[r]);
                const float pr = gam * ap[r];
                ta[r] = fmaf(cwA, pr, ta[r]);
                SA = fmaf(pr, dl[r], SA);
                SB = fmaf(gam, w[r], SB);
            }
            // term entering the previous tile: this tile's first decay x gamma
            if (lane == 0) gout[s] = av[0] * gam;
            float2 acc2 = sacc[s * 32 + lane];
            acc2.x += SA;
            acc2.y += SB;
            sacc[s * 32 + lane] = acc2;
        }
        // ---- per-event outputs
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float uv = su[segpad(q0 + r)];
            const float gv = sd[segpad(q0 + r)];
            const float duv = fmaf(Dv, gv, fmaf(2.f * uv * dl[r], tg[r], gv * te[r]));
            const float ddel = fmaf(uv * uv, tg[r], ta[r]);
            if (pl + r < Ew) {
                l_ddi = fmaf(ddel, (float)(sk[segpad(q0 + r)] - 1), l_ddi);
                l_dda += ddel;
                l_dD = fmaf(gv, uv, l_dD);
            }
            su[segpad(q0 + r)] = duv;
        }
        __syncwarp();
#pragma unroll
        for (int m = 0; m < R; ++m) {
            const int q = m * 32 + lane;
            const int e = se[segpad(q)];
            if (e >= 0) du[e] = from_f32<T>(su[segpad(q)]);
        }
        __syncwarp();
    }
    // ---- per-warp parameter partials (row grp*dim + d)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        l_ddi += __shfl_xor_sync(kFull, l_ddi, off);
        l_dda += __shfl_xor_sync(kFull, l_dda, off);
        l_dD += __shfl_xor_sync(kFull, l_dD, off);
    }
    float* part = a.ws_part + ((int64_t)grp * a.dim + d) * a.part_stride;
    for (int s = lane; s < N; s += 32) {
        float SA = 0.f, SB = 0.f;
        for (int l = 0; l < 32; ++l) {
            const float2 v = sacc[s * 32 + l];
            SA += v.x;
            SB += v.y;
        }
        part[s] = s_cw[s] * SA;
        part[N + s] = a.C[d * N + s] * SB;
        part[2 * N + s] = a.B[d * N + s] * SB;
    }
    if (lane == 0) {
        part[3 * N] = l_ddi;
        part[3 * N + 1] = l_dda;
        part[3 * N + 2] = l_dD;
    }
}

// ================================================================ host ====
constexpr int kSegR = 8;

SegGeom seg_geom(const ScanArgs& a, int warps) {
    SegGeom g{};
    const int Bn = a.n_channels / a.dim;
    const int64_t avg = std::max<int64_t>(1, (int64_t)a.n_events / std::max(1, a.n_channels));
    // several tiles per warp group (fewer partly filled tiles), but enough
    // groups to give every SM's schedulers several warps
    int cpw = 1;
    while (cpw * 2 <= kSegMaxCPW && cpw * 2 <= Bn && cpw * 2 * avg <= 2048 &&
           (int64_t)a.n_channels / (cpw * 2) >= (int64_t)sm_count() * 16)
        cpw *= 2;
    // BCM_SEG_CPW pins the rows per group (read on every call; the tests use
    // it to cover groups of many short channels at small sizes)
    if (const char* e = getenv("BCM_SEG_CPW")) {
        const int v = atoi(e);
        if (v >= 1) cpw = std::min(std::min(v, kSegMaxCPW), Bn);
    }
    g.cpw = cpw;
    g.groups_per_d = (Bn + cpw - 1) / cpw;
    g.warps = warps;
    g.ctas_per_d = (g.groups_per_d + warps - 1) / warps;
    return g;
}

size_t seg_fwd_smem(int N) {
    const int head = (N * kSegTR + 3 * N + 3) / 4 * 4;
    return (size_t)(head + kSegFwdWarps * seg_fwd_warp_floats<kSegR>(N)) * sizeof(float);
}
size_t seg_bwd_smem(int N) {
    const int head = (N * kSegTR + 3 * N + 3) / 4 * 4;
    return (size_t)(head + kSegBwdWarps * seg_bwd_warp_floats<kSegR>(N)) * sizeof(float);
}

// Opt a kernel into the device's shared-memory maximum (once per kernel and
// device).  Keyed by the kernel's address: the instantiations share one
// function type, so a per-type cache would skip all but the first.
bcm_status seg_optin(const void* kernel, size_t smem, const char* what) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;
    int dev = 0;
    BCM_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    int& mx = done[{kernel, dev}];
    if (mx == 0) {
        int lim = 0;
        BCM_CUDA_TRY(cudaDeviceGetAttribute(&lim, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        BCM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
        mx = lim;
    }
    if (smem > (size_t)mx) {
        set_error("%s: %zu bytes of shared memory exceed the device limit %d", what, smem, mx);
        return BCM_ERR_UNSUPPORTED;
    }
    return BCM_OK;
}

bcm_status seg_build_table(const ScanArgs& a, float* tab, cudaStream_t st) {
    const int64_t total = (int64_t)a.dim * a.dstate * kSegTR;
    const int threads = 256;
    const int grid = (int)std::min<int64_t>((total + threads - 1) / threads, (int64_t)sm_count() * 8);
    seg_table_kernel<<<grid, threads, 0, st>>>(a, tab);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T, bool CARRY_ONLY>
bcm_status seg_fwd_t(const ScanArgs& a, const float* tab, float* carries, cudaStream_t st) {
    const SegGeom g = seg_geom(a, kSegFwdWarps);
    const size_t smem = seg_fwd_smem(a.dstate);
    auto kern = seg_fwd_kernel<T, kSegR, CARRY_ONLY>;
    if (smem > 48 * 1024) {
        const bcm_status s = seg_optin(reinterpret_cast<const void*>(kern), smem, "flat_ch fwd");
        if (s != BCM_OK) return s;
    }
    kern<<<a.dim * g.ctas_per_d, 32 * kSegFwdWarps, smem, st>>>(a, tab, g, carries);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <typename T>
bcm_status seg_bwd_t(const ScanArgs& a, const float* tab, const float* carries, cudaStream_t st) {
    const SegGeom g = seg_geom(a, kSegBwdWarps);
    const size_t smem = seg_bwd_smem(a.dstate);
    auto kern = seg_bwd_kernel<T, kSegR>;
    if (smem > 48 * 1024) {
        const bcm_status s = seg_optin(reinterpret_cast<const void*>(kern), smem, "flat_ch bwd");
        if (s != BCM_OK) return s;
    }
    kern<<<a.dim * g.ctas_per_d, 32 * kSegBwdWarps, smem, st>>>(a, tab, g, carries);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

}  // namespace

// The event-parallel kernels serve the depthwise mode without the silu gate
// for dstate <= 64 when every feature has the same number of batch rows.
bool seg_supported(const ScanArgs& a) {
    return a.bc_mode == BCM_BC_DEPTHWISE && a.z == nullptr && a.dstate <= 64 && a.dim > 0 &&
           a.n_channels % a.dim == 0 && a.n_events > 0;
}

bool seg_selected(const ScanArgs& a) {
    const char* e = getenv("BCM_SCAN_SEG");
    const int mode = e ? atoi(e) : 1;
    if (mode == 0 || !seg_supported(a)) return false;
    if (mode >= 2) return true;
    return !(v3_supported(a, false) && v3_supported(a, true));
}

size_t seg_table_bytes(const ScanArgs& a) {
    return align_up((size_t)a.dim * a.dstate * kSegTR * sizeof(float), 256);
}

size_t seg_carry_bytes(const ScanArgs& a) {
    const size_t slots = (size_t)a.n_events / SegTile<kSegR>::TILE + (size_t)a.n_channels + 1;
    return align_up(slots * a.dstate * sizeof(float), 256);
}

// Rows of partials the backward writes (groups per feature x dim).
int seg_part_rows(const ScanArgs& a) { return seg_geom(a, kSegBwdWarps).groups_per_d * a.dim; }

bcm_status seg_fwd_launch(const ScanArgs& a, bcm_dtype dtype, float* table_ws, float* carries,
                          cudaStream_t st) {
    bcm_status s = seg_build_table(a, table_ws, st);
    if (s != BCM_OK) return s;
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        return seg_fwd_t<T, false>(a, table_ws, carries, st);
    });
}

bcm_status seg_bwd_launch(const ScanArgs& a, bcm_dtype dtype, float* table_ws, const float* fwd_carries,
                          float* carry_ws, cudaStream_t st) {
    bcm_status s = seg_build_table(a, table_ws, st);
    if (s != BCM_OK) return s;
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        const float* car = fwd_carries;
        if (car == nullptr) {
            // no carries from the forward: one carries-only pass writes them
            const bcm_status s2 = seg_fwd_t<T, true>(a, table_ws, carry_ws, st);
            if (s2 != BCM_OK) return s2;
            car = carry_ws;
        }
        return seg_bwd_t<T>(a, table_ws, car, st);
    });
}

}  // namespace bcm
