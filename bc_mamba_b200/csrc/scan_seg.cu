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
#include <type_traits>
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

// States are processed in pairs (s, s+1) with the packed fp32x2 FMA of
// sm_100 (per component the same rounding as fmaf); an odd dstate gets one
// padding state with A = 0 and W = 0, which contributes nothing.
__host__ __device__ __forceinline__ int seg_pairs(int N) { return (N + 1) >> 1; }

__device__ __forceinline__ int segpad(int q) { return q + (q >> 5); }
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// Largest c in [0, nc) with vs[c] <= p (vs[0] = 0 <= p).  Skips empty channels.
__device__ __forceinline__ int seg_find(const int* vs, int nc, int p) {
    int lo = 0, hi = nc - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (vs[mid] <= p) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ float seg_A2(const ScanArgs& a, int d, int s) {
    return s < a.dstate ? (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634) : 0.f;
}

// Per-feature decay tables of state pairs, tab[d][pair][row] (rows as kSegTR).
__global__ void seg_table_kernel(ScanArgs a, float2* __restrict__ tab) {
    const int NP2 = seg_pairs(a.dstate);
    const int64_t total = (int64_t)a.dim * NP2 * kSegTR;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i % kSegTR);
        const int64_t dp = i / kSegTR;
        const int sp = (int)(dp % NP2), d = (int)(dp / NP2);
        float2 v;
        if (row == 0) {
            v = make_float2(0.f, 0.f);
        } else if (row == kSegPadRow) {
            v = make_float2(1.f, 1.f);
        } else {
            const float dl = event_delta(a.dt_idle[d], a.dt_active[d], row);
            v = make_float2(decay_exact(dl, seg_A2(a, d, 2 * sp)), decay_exact(dl, seg_A2(a, d, 2 * sp + 1)));
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

__device__ __forceinline__ float2 shfl_up2(float2 v, int off) {
    return make_float2(__shfl_up_sync(kFull, v.x, off), __shfl_up_sync(kFull, v.y, off));
}
__device__ __forceinline__ float2 shfl_down2(float2 v, int off) {
    return make_float2(__shfl_down_sync(kFull, v.x, off), __shfl_down_sync(kFull, v.y, off));
}

// Kogge-Stone inclusive scan of the (a, b) operator over the warp's lanes
// (lane order = event order), two states at once.
__device__ __forceinline__ void seg_scan_up(float2& A, float2& B, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float2 Ao = shfl_up2(A, off);
        const float2 Bo = shfl_up2(B, off);
        if (lane >= off) {
            B = __ffma2_rn(A, Bo, B);
            A = __fmul2_rn(A, Ao);
        }
    }
}

// Suffix (right-to-left) scan: lane L composes its map gamma_first(L) =
// M_L*gamma_first(L+1) + G_L with the lanes to its right.
__device__ __forceinline__ void seg_scan_down(float2& M, float2& G, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float2 Mo = shfl_down2(M, off);
        const float2 Go = shfl_down2(G, off);
        if (lane + off < 32) {
            G = __ffma2_rn(M, Go, G);
            M = __fmul2_rn(M, Mo);
        }
    }
}

template <int R>
struct SegTile {
    static constexpr int TILE = 32 * R;
    static constexpr int PADT = TILE + TILE / 32;
};

// Shared memory (floats): a CTA head with the table and per-pair constants,
// then one region per warp (all rounded to 16 bytes).
__host__ __device__ constexpr int seg_head_floats(int N) {
    return (2 * seg_pairs(N) * kSegTR + 6 * seg_pairs(N) + 3) / 4 * 4;
}
template <int R>
__host__ __device__ constexpr int seg_fwd_warp_floats(int N) {
    return (5 * SegTile<R>::PADT + 4 * seg_pairs(N) + (int)(sizeof(SegWarp) / 4) + 3) / 4 * 4;
}
template <int R>
__host__ __device__ constexpr int seg_bwd_warp_floats(int N) {
    return (4 * SegTile<R>::PADT + 6 * seg_pairs(N) + (int)(sizeof(SegWarp) / 4) + 128 * seg_pairs(N) + 3) / 4 * 4;
}

// Copy the feature's table and per-pair constants into the CTA head:
// c0 = (W_B*W_C) pairs, c1 = W_B pairs (forward) or W_B*W_C*A pairs
// (backward), c2 = A*log2(e) pairs.
__device__ __forceinline__ void seg_load_head(const ScanArgs& a, int d, const float2* gtab, float2* tab,
                                              float2* c0, float2* c1, float2* c2, bool bwd) {
    const int N = a.dstate, NP2 = seg_pairs(N);
    const float2* src = gtab + (int64_t)d * NP2 * kSegTR;
    for (int i = threadIdx.x; i < NP2 * kSegTR; i += blockDim.x) tab[i] = src[i];
    for (int sp = threadIdx.x; sp < NP2; sp += blockDim.x) {
        float cw[2], x1[2], A2[2];
        for (int h = 0; h < 2; ++h) {
            const int s = 2 * sp + h;
            const bool ok = s < N;
            const float wb = ok ? a.B[d * N + s] : 0.f;
            cw[h] = ok ? wb * a.C[d * N + s] : 0.f;
            x1[h] = bwd ? (ok ? cw[h] * a.A[d * a.A_sd + s * a.A_sn] : 0.f) : wb;
            A2[h] = seg_A2(a, d, s);
        }
        c0[sp] = make_float2(cw[0], cw[1]);
        c1[sp] = make_float2(x1[0], x1[1]);
        c2[sp] = make_float2(A2[0], A2[1]);
    }
}

// =============================================================== forward ====
// CARRY_ONLY: only the state entering every tile (for a backward that was not
// given the forward's carries); no outputs.
template <typename T, int R, bool CARRY_ONLY>
__global__ void __launch_bounds__(32 * kSegFwdWarps, 2)
seg_fwd_kernel(ScanArgs a, const float2* __restrict__ gtab, SegGeom g, float* __restrict__ carries) {
    constexpr int TILE = SegTile<R>::TILE;
    constexpr int PADT = SegTile<R>::PADT;
    extern __shared__ __align__(16) float sm[];
    const int N = a.dstate, NP2 = seg_pairs(N);
    const int d = blockIdx.x / g.ctas_per_d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = seg_head_floats(N);
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < (size_t)(head + g.warps * seg_fwd_warp_floats<R>(N)) * sizeof(float)) return;
    }
    float2* tab = reinterpret_cast<float2*>(sm);
    float2* s_cw = tab + NP2 * kSegTR;
    float2* s_wb = s_cw + NP2;
    float2* s_A2 = s_wb + NP2;
    float* wr = sm + head + warp * seg_fwd_warp_floats<R>(N);
    float* su = wr;
    int* sk = reinterpret_cast<int*>(su + PADT);
    int* se = sk + PADT;
    int* sxr = se + PADT;
    float* ssd = reinterpret_cast<float*>(sxr + PADT);
    float2* carry = reinterpret_cast<float2*>(ssd + PADT);      // [2][NP2]
    SegWarp* W = reinterpret_cast<SegWarp*>(carry + 2 * NP2);

    seg_load_head(a, d, gtab, tab, s_cw, s_wb, s_A2, false);
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
    for (int sp = lane; sp < NP2; sp += 32) carry[sp] = make_float2(0.f, 0.f);
    int kc = 0;    // gap sum since the start of the channel running into the next tile
    const int n_tiles = (Ew + TILE - 1) / TILE;
    __syncwarp();

    for (int t = 0; t < n_tiles; ++t) {
        const int p0 = t * TILE;
        const float2* cin = carry + (t & 1) * NP2;
        float2* cout = carry + ((t + 1) & 1) * NP2;
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
                float2* dst = reinterpret_cast<float2*>(carries) + ((int64_t)e0 / TILE + W->ch[c0]) * NP2;
                for (int sp = lane; sp < NP2; sp += 32) dst[sp] = cin[sp];
            }
        }
        __syncwarp();

        // ---- this lane's events
        const int q0 = lane * R, pl = p0 + q0;
        float w[R];
        int ix[R];
        unsigned exm = 0, cem = 0, hdm = 0;
        {
            int c = seg_find(vs, nc, min(pl, Ew - 1));
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int p = pl + r;
                const float uv = su[segpad(q0 + r)];
                const int kv = sk[segpad(q0 + r)];
                if (p < Ew) {
                    while (p >= vs[c + 1]) ++c;
                    const int j = p - vs[c], n = vs[c + 1] - vs[c];
                    w[r] = event_delta(dti, dta, kv) * uv * uv;
                    const bool hit = (unsigned)(kv - 1) < (unsigned)kSegKMax;
                    ix[r] = (j == 0) ? 0 : (hit ? kv : kSegPadRow);
                    if (j != 0 && !hit) exm |= 1u << r;
                    if (j == 0) hdm |= 1u << r;
                    if (((j + 1) & (kChunkX - 1)) == 0 || j == n - 1) cem |= 1u << r;
                } else {
                    w[r] = 0.f;
                    ix[r] = kSegPadRow;
                }
            }
        }
        const bool wexact = __any_sync(kFull, exm != 0);
        const bool wchunk = !CARRY_ONLY && __any_sync(kFull, cem != 0);
        // ---- chunk bookkeeping for x (tiles holding a chunk end): gap sums
        // since each channel's first event (prod a of x runs from the channel
        // start, as the reference's chunk prefix does), segmented at channel
        // starts; kc carries the running sum into the next tile
        if (!CARRY_ONLY) {
            int v = 0, f = 0;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (hdm >> r & 1) { v = 0; f = 1; }
                v += sk[segpad(q0 + r)];
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
            if (wchunk && cem) {
                int ve = __shfl_up_sync(kFull, vi, 1), fe = __shfl_up_sync(kFull, fi, 1);
                if (lane == 0) { ve = 0; fe = 0; }
                int K = fe ? ve : kc + ve;
                int c = seg_find(vs, nc, min(pl, Ew - 1));
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (hdm >> r & 1) K = 0;
                    K += sk[segpad(q0 + r)];
                    if (cem >> r & 1) {
                        const int p = pl + r;
                        while (p >= vs[c + 1]) ++c;
                        const int j = p - vs[c];
                        const int chunk = j / kChunkX;
                        sxr[segpad(q0 + r)] = chunk < nchk ? W->ch[c] * nchk + chunk : -1;
                        ssd[segpad(q0 + r)] = fmaf(dti, (float)(K - (j + 1)), dta * (float)(j + 1));
                    }
                }
            } else if (wchunk) {
                (void)__shfl_up_sync(kFull, vi, 1);
                (void)__shfl_up_sync(kFull, fi, 1);
            }
            const int v31 = __shfl_sync(kFull, vi, 31), f31 = __shfl_sync(kFull, fi, 31);
            kc = f31 ? v31 : kc + v31;
        }

        // ---- state pairs
        float2 acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = make_float2(0.f, 0.f);
        auto pair_pass = [&](auto chunk_c, int sp) {
            constexpr bool CHUNK = decltype(chunk_c)::value;
            const float2* ts = tab + sp * kSegTR;
            float2 av[R];
#pragma unroll
            for (int r = 0; r < R; ++r) av[r] = ts[ix[r]];
            if (wexact && exm) {
                const float2 A2 = s_A2[sp];
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (exm >> r & 1) {
                        const float dl = event_delta(dti, dta, sk[segpad(q0 + r)]);
                        av[r] = make_float2(decay_fast(dl, A2.x), decay_fast(dl, A2.y));
                    }
            }
            float2 A = av[0], Bv = f2(w[0]);
#pragma unroll
            for (int r = 1; r < R; ++r) {
                Bv = __ffma2_rn(av[r], Bv, f2(w[r]));
                A = __fmul2_rn(A, av[r]);
            }
            seg_scan_up(A, Bv, lane);
            // the carries-only pass computes the states exactly as here, so a
            // backward from either pass sees bit-identical carries
            float2 Ae = shfl_up2(A, 1), Be = shfl_up2(Bv, 1);
            if (lane == 0) {
                Ae = make_float2(1.f, 1.f);
                Be = make_float2(0.f, 0.f);
            }
            float2 eta = __ffma2_rn(Ae, cin[sp], Be);
            const float2 cw = s_cw[sp];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                eta = __ffma2_rn(av[r], eta, f2(w[r]));
                acc[r] = __ffma2_rn(cw, eta, acc[r]);
                if (CHUNK && (cem >> r & 1)) {
                    const int xr = sxr[segpad(q0 + r)];
                    if (xr >= 0) {
                        float* xo = a.x + (int64_t)xr * 2 * N;
                        const float sd = ssd[segpad(q0 + r)];
                        const float2 A2 = s_A2[sp], wb = s_wb[sp];
                        xo[4 * sp] = exp2f(A2.x * sd);
                        xo[4 * sp + 1] = wb.x * eta.x;
                        if (2 * sp + 1 < N) {
                            xo[4 * sp + 2] = exp2f(A2.y * sd);
                            xo[4 * sp + 3] = wb.y * eta.y;
                        }
                    }
                }
            }
            const float2 cnew = make_float2(__shfl_sync(kFull, eta.x, 31), __shfl_sync(kFull, eta.y, 31));
            if (lane == 0) cout[sp] = cnew;
        };
        if (wchunk) {
            for (int sp = 0; sp < NP2; ++sp) pair_pass(std::true_type{}, sp);
        } else {
#pragma unroll 2
            for (int sp = 0; sp < NP2; ++sp) pair_pass(std::false_type{}, sp);
        }
        if (!CARRY_ONLY) {
            // ---- outputs y = D*u + u*acc, stored coalesced
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float uv = su[segpad(q0 + r)];
                su[segpad(q0 + r)] = fmaf(Dv, uv, uv * (acc[r].x + acc[r].y));
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
// Per tile (last to first) and state pair: forward scan for eta from the
// tile's incoming state, reverse scan for gamma (the adjoint of eta divided by
// cw) from the next tile's outgoing term, then
//   du_i  = D*g_i + g_i*sum_s cw_s*eta_i,s + 2*delta_i*u_i*sum_s cw_s*gamma_i,s
//   dd_i  = u_i^2*sum_s cw_s*gamma_i,s + sum_s cw_s*A_s*gamma_i,s*a_i,s*eta_{i-1},s
//   dA_s  = cw_s*sum_i gamma_i,s*a_i,s*eta_{i-1},s*delta_i
//   dW_B_s = W_C_s*sum_i gamma_i,s*w_i,  dW_C_s = W_B_s*sum_i gamma_i,s*w_i
//   ddt_idle = sum_i dd_i*(k_i - 1), ddt_active = sum_i dd_i, dD = sum_i g_i*u_i
// (sum_i gamma_i*w_i = sum_i g_i*u_i*eta_i: both W gradients use it).
// Parameter sums are per-warp partials, rows grp*dim + d of ws_part, reduced
// over the groups of a feature in a fixed order afterwards.
template <typename T, int R>
__global__ void __launch_bounds__(32 * kSegBwdWarps, 3)
seg_bwd_kernel(ScanArgs a, const float2* __restrict__ gtab, SegGeom g, const float* __restrict__ carries) {
    constexpr int TILE = SegTile<R>::TILE;
    constexpr int PADT = SegTile<R>::PADT;
    extern __shared__ __align__(16) float sm[];
    const int N = a.dstate, NP2 = seg_pairs(N);
    const int d = blockIdx.x / g.ctas_per_d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = seg_head_floats(N);
    {
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < (size_t)(head + g.warps * seg_bwd_warp_floats<R>(N)) * sizeof(float)) return;
    }
    float2* tab = reinterpret_cast<float2*>(sm);
    float2* s_cw = tab + NP2 * kSegTR;
    float2* s_cwA = s_cw + NP2;
    float2* s_A2 = s_cwA + NP2;
    float* wr = sm + head + warp * seg_bwd_warp_floats<R>(N);
    float* su = wr;
    int* sk = reinterpret_cast<int*>(su + PADT);
    float* sd = reinterpret_cast<float*>(sk + PADT);
    int* se = reinterpret_cast<int*>(sd + PADT);
    float2* gcar = reinterpret_cast<float2*>(se + PADT);   // [2][NP2] terms entering from the next tile
    float2* ecar = gcar + 2 * NP2;                          // [NP2] state entering the tile
    SegWarp* W = reinterpret_cast<SegWarp*>(ecar + NP2);
    float4* sacc = reinterpret_cast<float4*>(wr + (seg_bwd_warp_floats<R>(N) - 128 * NP2));   // [NP2][32]

    seg_load_head(a, d, gtab, tab, s_cw, s_cwA, s_A2, true);
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

    for (int sp = 0; sp < NP2; ++sp) sacc[sp * 32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int n_tiles = (Ew + TILE - 1) / TILE;
    for (int sp = lane; sp < NP2; sp += 32) gcar[(n_tiles & 1) * NP2 + sp] = make_float2(0.f, 0.f);
    float l_ddi = 0.f, l_dda = 0.f, l_dD = 0.f;
    __syncwarp();

    for (int t = n_tiles - 1; t >= 0; --t) {
        const int p0 = t * TILE;
        const float2* gin = gcar + ((t + 1) & 1) * NP2;
        float2* gout = gcar + (t & 1) * NP2;
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
        {
            const int c0 = seg_find(vs, nc, p0);
            const int e0 = W->base[c0] + (p0 - vs[c0]);
            const float2* src = reinterpret_cast<const float2*>(carries) + ((int64_t)e0 / TILE + W->ch[c0]) * NP2;
            const bool from = t > 0 && e0 >= 0 && e0 < a.n_events;
            for (int sp = lane; sp < NP2; sp += 32) ecar[sp] = from ? src[sp] : make_float2(0.f, 0.f);
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

        for (int sp = 0; sp < NP2; ++sp) {
            const float2* ts = tab + sp * kSegTR;
            float2 av[R];
#pragma unroll
            for (int r = 0; r < R; ++r) av[r] = ts[ix[r]];
            if (wexact && exm) {
                const float2 A2 = s_A2[sp];
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (exm >> r & 1) {
                        const float dlr = event_delta(dti, dta, sk[segpad(q0 + r)]);
                        av[r] = make_float2(decay_fast(dlr, A2.x), decay_fast(dlr, A2.y));
                    }
            }
            // forward: incoming state of each lane
            float2 A = av[0], Bv = f2(w[0]);
#pragma unroll
            for (int r = 1; r < R; ++r) {
                Bv = __ffma2_rn(av[r], Bv, f2(w[r]));
                A = __fmul2_rn(A, av[r]);
            }
            seg_scan_up(A, Bv, lane);
            float2 Ae = shfl_up2(A, 1), Be = shfl_up2(Bv, 1);
            if (lane == 0) {
                Ae = make_float2(1.f, 1.f);
                Be = make_float2(0.f, 0.f);
            }
            const float2 eta_in = __ffma2_rn(Ae, ecar[sp], Be);
            // reverse: multiplier of event r is the next event's decay (0 after
            // a channel's last event); lane 31's last event takes the term
            // entering from the next tile instead
            const float2 a_next = shfl_down2(av[0], 1);
            const float2 g_in = gin[sp];
            const bool top = lane == 31;
            float2 mlast = top ? f2(1.f) : a_next;
            if (!top && (lsm >> (R - 1) & 1)) mlast = f2(0.f);
            float2 G = top ? g_in : f2(0.f);
            float2 M = top ? f2(0.f) : f2(1.f);
            G = __ffma2_rn(mlast, G, f2(qv[R - 1]));
            M = __fmul2_rn(M, mlast);
#pragma unroll
            for (int r = R - 2; r >= 0; --r) {
                const float2 m = (lsm >> r & 1) ? f2(0.f) : av[r + 1];
                G = __ffma2_rn(m, G, f2(qv[r]));
                M = __fmul2_rn(M, m);
            }
            seg_scan_down(M, G, lane);
            const float2 X = shfl_down2(G, 1);
            // pass 2: states and adjoints of the lane's events
            const float2 cw = s_cw[sp], cwA = s_cwA[sp];
            float2 ap[R];
            float2 eta = eta_in;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                ap[r] = __fmul2_rn(av[r], eta);
                eta = __fadd2_rn(ap[r], f2(w[r]));
                te[r] = fmaf(cw.x, eta.x, fmaf(cw.y, eta.y, te[r]));
            }
            float2 gam = top ? g_in : X;
            float2 SA = f2(0.f), SB = f2(0.f);
#pragma unroll
            for (int r = R - 1; r >= 0; --r) {
                const float2 m = (r == R - 1) ? mlast : ((lsm >> r & 1) ? f2(0.f) : av[r + 1]);
                gam = __ffma2_rn(m, gam, f2(qv[r]));
                tg[r] = fmaf(cw.x, gam.x, fmaf(cw.y, gam.y, tg[r]));
                const float2 pr = __fmul2_rn(gam, ap[r]);
                ta[r] = fmaf(cwA.x, pr.x, fmaf(cwA.y, pr.y, ta[r]));
                SA = __ffma2_rn(pr, f2(dl[r]), SA);
                SB = __ffma2_rn(gam, f2(w[r]), SB);
            }
            // term entering the previous tile: this tile's first decay x gamma
            if (lane == 0) gout[sp] = __fmul2_rn(av[0], gam);
            float4 acc4 = sacc[sp * 32 + lane];
            acc4.x += SA.x;
            acc4.y += SA.y;
            acc4.z += SB.x;
            acc4.w += SB.y;
            sacc[sp * 32 + lane] = acc4;
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
    for (int sp = lane; sp < NP2; sp += 32) {
        float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int l = 0; l < 32; ++l) {
            const float4 v = sacc[sp * 32 + l];
            t4.x += v.x;
            t4.y += v.y;
            t4.z += v.z;
            t4.w += v.w;
        }
        const float2 cw = s_cw[sp];
        const float sa[2] = {t4.x, t4.y}, sb[2] = {t4.z, t4.w}, c[2] = {cw.x, cw.y};
        for (int h = 0; h < 2; ++h) {
            const int s = 2 * sp + h;
            if (s < N) {
                part[s] = c[h] * sa[h];
                part[N + s] = a.C[d * N + s] * sb[h];
                part[2 * N + s] = a.B[d * N + s] * sb[h];
            }
        }
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
    return (size_t)(seg_head_floats(N) + kSegFwdWarps * seg_fwd_warp_floats<kSegR>(N)) * sizeof(float);
}
size_t seg_bwd_smem(int N) {
    return (size_t)(seg_head_floats(N) + kSegBwdWarps * seg_bwd_warp_floats<kSegR>(N)) * sizeof(float);
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
    const int64_t total = (int64_t)a.dim * seg_pairs(a.dstate) * kSegTR;
    const int threads = 256;
    const int grid = (int)std::min<int64_t>((total + threads - 1) / threads, (int64_t)sm_count() * 8);
    seg_table_kernel<<<grid, threads, 0, st>>>(a, reinterpret_cast<float2*>(tab));
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
    kern<<<a.dim * g.ctas_per_d, 32 * kSegFwdWarps, smem, st>>>(a, reinterpret_cast<const float2*>(tab), g,
                                                                 carries);
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
    kern<<<a.dim * g.ctas_per_d, 32 * kSegBwdWarps, smem, st>>>(a, reinterpret_cast<const float2*>(tab), g,
                                                                 carries);
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
    if (!(v3_supported(a, false) && v3_supported(a, true))) return true;
    // the staged kernels walk each channel's events in one warp lane group:
    // with few batch rows per feature (a batch sharded over many ranks) they
    // leave the SMs short of warps, and the event-parallel kernels, whose
    // warps hold whole tiles of events, are faster (B200, the 4-block stack
    // at 16 rows per feature: scan 0.88 ms per step against 1.10 ms; at 32
    // rows 1.39 against 1.31)
    return v3_bwd_warps(a) < 5 * sm_count();
}

size_t seg_table_bytes(const ScanArgs& a) {
    return align_up((size_t)a.dim * seg_pairs(a.dstate) * kSegTR * sizeof(float2), 256);
}

size_t seg_carry_bytes(const ScanArgs& a) {
    const size_t slots = (size_t)a.n_events / SegTile<kSegR>::TILE + (size_t)a.n_channels + 1;
    return align_up(slots * seg_pairs(a.dstate) * sizeof(float2), 256);
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
