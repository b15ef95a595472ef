// scan_v3.cu — staged depthwise scan kernels for dstate <= 64 (forward and
// backward), used when the channels of one feature d fill whole warps.
// Semantics are those of scan_fwd.cu / scan_bwd.cu (reference
// selective_scan_fwd_kernel.cuh:403-728, selective_scan_bwd_kernel.cuh:
// 635-1169, depthwise B/C); the layout is:
//
//  * warps own channels of one feature d (batch rows b..), so they share one
//    decay table per feature (rows k = 1..kKT3 for the integer gap k, row 0 =
//    identity), built once per CTA or warp with exp2 in double (correctly
//    rounded: each entry is reused by every event with that gap);
//  * events are staged 32 per channel at a time: one coalesced load per
//    channel and array brings them into registers while the previous batch is
//    processed, then a transposed shared-memory copy hands each lane its own
//    channel's events (conflict-free); padding slots past a channel's last
//    event read the identity row with u = 0, so inner loops carry no per-event
//    predicate, and a batch holding a gap outside the table (or, forward, a
//    clamping exponent of non-decaying parameters) takes a separate exact loop;
//  * forward (dw_fwd_v4): phase A runs the state recurrence with G <= 4 states
//    per lane and stores the states of the batch to shared memory; phase B
//    maps lanes to events and forms y = D*u + u*sum_s cc_s*eta_s for each
//    channel, stored coalesced;
//  * backward (dw_bwd_v3): 4 states per lane; per 2048-event chunk a forward
//    pass saves the state entering every 8-event tile, then batches, tiles and
//    events are walked last to first with the tile's states recomputed into
//    registers; per-event sums over a channel's lanes are transposed
//    reductions once per tile.
#include <stdlib.h>

#include <algorithm>

#include <mutex>
#include <type_traits>

#include "scan_common.cuh"

namespace bcm {

namespace {

int env_int(const char* name, int dflt) {
    const char* e = getenv(name);
    return e ? atoi(e) : dflt;
}

constexpr int kR3 = 32;          // events per channel per staged batch
constexpr int kKT3 = 128;        // tabulated gaps 1..kKT3
constexpr int kRows3 = kKT3 + 1; // row 0 = identity (padding slots)
static_assert(kChunkX % kR3 == 0, "chunk boundaries must fall on batch boundaries");
static_assert(kR3 % kCkpt == 0, "tiles must not straddle batches");

template <int G, int LPC>
struct V3 {
    static constexpr int NP = G * LPC;     // padded states per channel
    static constexpr int CPW = 32 / LPC;   // channels per warp
    static constexpr int P = CPW + 1;      // staging pitch (conflict-free transposes)
    static constexpr int TAB = NP * kRows3;
};

// Table layout: float4 groups of states, [s/4][row] -> a lane's G decays of
// one row are G/4 vector loads; rows of different lanes spread over banks.
// Decay of gap `row` for state s of feature d: from the per-call table when
// one was computed, else evaluated here (row 0 and padded states = 1).
template <int NP>
__device__ __forceinline__ float table_entry(const ScanArgs& a, int d, int s, int row) {
    if (a.dtab != nullptr) return a.dtab[((int64_t)d * NP + s) * kRows3 + row];
    float v = 1.f;
    if (row > 0 && s < a.dstate) {
        const float A2 = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
        v = decay_exact(event_delta(a.dt_idle[d], a.dt_active[d], row), A2);
    }
    return v;
}

template <int NP>
__device__ void build_table3(float* tab, const ScanArgs& a, int d, int lane) {
    for (int e = lane; e < kRows3 * NP; e += 32) {
        const int row = e % kRows3, s = e / kRows3;
        tab[((s >> 2) * kRows3 + row) * 4 + (s & 3)] = table_entry<NP>(a, d, s, row);
    }
    __syncwarp();
}

// Checkpoint state of G states (G = 2: one 8-byte, G >= 4: G/4 16-byte moves).
template <int G>
__device__ __forceinline__ void ck_store(float* p, const float (&v)[G]) {
    if constexpr (G == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int j = 0; j < G / 4; ++j)
            reinterpret_cast<float4*>(p)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
}

template <int G>
__device__ __forceinline__ void ck_load(const float* p, bool ok, float (&v)[G]) {
    if constexpr (G == 2) {
        const float2 t = ok ? *reinterpret_cast<const float2*>(p) : make_float2(0.f, 0.f);
        v[0] = t.x; v[1] = t.y;
    } else {
#pragma unroll
        for (int j = 0; j < G / 4; ++j) {
            const float4 t = ok ? reinterpret_cast<const float4*>(p)[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
        }
    }
}

template <int G>
__device__ __forceinline__ void tab_row3(const float* tab, int row, int q, float (&dec)[G]) {
    if constexpr (G == 2) {   // two states inside one float4 group of the table
        const int s0 = 2 * q;
        const float2 v = *reinterpret_cast<const float2*>(tab + (((s0 >> 2) * kRows3 + row) * 4 + (s0 & 3)));
        dec[0] = v.x;
        dec[1] = v.y;
        return;
    }
    const float4* t4 = reinterpret_cast<const float4*>(tab);
#pragma unroll
    for (int j = 0; j < G / 4; ++j) {
        const float4 v = t4[(q * (G / 4) + j) * kRows3 + row];
        dec[4 * j] = v.x;
        dec[4 * j + 1] = v.y;
        dec[4 * j + 2] = v.z;
        dec[4 * j + 3] = v.w;
    }
}

// One channel's batch of events -> registers: slot c of lane l holds event
// j0 + l of warp channel c (coalesced: the 32 lanes read 32 consecutive events).
template <typename T, int CPW>
__device__ __forceinline__ void fetch_f(const T* src, const int* s_base, const int* s_len, int j0,
                                        int lane, float (&r)[CPW]) {
    const int j = j0 + lane;
#pragma unroll
    for (int c = 0; c < CPW; ++c) r[c] = (j < s_len[c]) ? to_f32<T>(src[s_base[c] + j]) : 0.f;
}

template <int CPW>
__device__ __forceinline__ void fetch_k(const int32_t* src, const int* s_base, const int* s_len, int j0,
                                        int lane, int (&r)[CPW]) {
    const int j = j0 + lane;
#pragma unroll
    for (int c = 0; c < CPW; ++c) r[c] = (j < s_len[c]) ? src[s_base[c] + j] : 0;
}

template <int CPW, int P, typename V>
__device__ __forceinline__ void stage(V* s, const V (&r)[CPW], int lane) {
#pragma unroll
    for (int c = 0; c < CPW; ++c) s[lane * P + c] = r[c];
}

__device__ __forceinline__ int warp_max(int v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(kFull, v, off));
    return v;
}

__device__ __forceinline__ float warp_all_min(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fminf(v, __shfl_xor_sync(kFull, v, off));
    return v;
}

// True when some real event of the batch in registers (slot c = channel c,
// event j0 + lane; padding slots hold k = 0) needs the exact path: a gap
// outside the table, or (forward, non-decaying parameters) a delta that may
// clamp.  Warp-uniform.
template <int CPW>
__device__ __forceinline__ bool batch_needs_exact(const int (&pk)[CPW], const int* s_len, int j0, int lane,
                                                  float dti, float dta, float dlim) {
    bool miss = false;
    const int j = j0 + lane;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
        const int kk = pk[c];
        const bool bad = (unsigned)(kk - 1) >= (unsigned)kKT3 || event_delta(dti, dta, kk) > dlim;
        miss = miss || (j < s_len[c] && bad);
    }
    return __any_sync(kFull, miss);
}

// Sum v[0..CPW) over the 32 lanes so that afterwards every lane holds the
// total of its own channel (lane / LPC) in v[0].
template <int CPW>
__device__ __forceinline__ float warp_channel_sum(float (&v)[CPW], int lane) {
#pragma unroll
    for (int lvl = 0; (CPW >> lvl) > 1; ++lvl) {
        const int o = 16 >> lvl;
        const int half = (CPW >> lvl) / 2;
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < half; ++j) {
            const float send = up ? v[j] : v[j + half];
            const float recv = __shfl_xor_sync(kFull, send, o);
            v[j] = (up ? v[j + half] : v[j]) + recv;
        }
    }
    float t = v[0];
#pragma unroll
    for (int o = 32 / CPW / 2; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
    return t;
}

// =========================================================== backward ====
// Per channel and chunk of 2048 events: pass 1 runs the recurrence forward
// from the chunk's start state and saves the state entering every tile of
// kCkpt events (workspace slots as scan_bwd.cu); pass 2 walks batches, tiles
// and events last to first, recomputing each tile's states from its
// checkpoint into registers.  Per-event sums over a channel's states are
// reduced over its LPC lanes once per tile (transposed: lane q finalises
// events q*TB/LPC .. q*TB/LPC + TB/LPC - 1 of the tile).
template <typename T, int G, int LPC>
__global__ void __launch_bounds__(32)
dw_bwd_v3(ScanArgs a, int bgroups) {
    using V = V3<G, LPC>;
    constexpr int CPW = V::CPW, P = V::P, NP = V::NP;
    constexpr int TB = kCkpt;
    constexpr int EPL = TB / LPC;
    extern __shared__ __align__(16) float sm3[];
    float* tab = sm3;
    float* s_u = tab + V::TAB;
    int* s_k = reinterpret_cast<int*>(s_u + kR3 * P);
    float* s_d = reinterpret_cast<float*>(s_k + kR3 * P);
    float* s_du = s_d + kR3 * P;
    int* s_cb = reinterpret_cast<int*>(s_du + kR3 * P);   // chunk start of each channel
    int* s_len = s_cb + CPW;                               // chunk length of each channel
    int* s_beg = s_len + CPW;
    int* s_n = s_beg + CPW;

    const int lane = threadIdx.x, grp = lane / LPC, q = lane % LPC;
    // rank-major: the warps holding every feature's longest rows start first
    const int d = rank_major(a) ? blockIdx.x % a.dim : blockIdx.x / bgroups;
    const int b0 = (rank_major(a) ? blockIdx.x / a.dim : blockIdx.x % bgroups) * CPW;
    const int N = a.dstate;
    if (lane < CPW) {
        const int c = scan_row(a, d, b0 + lane) * a.dim + d;
        s_beg[lane] = a.cu[c];
        s_n[lane] = a.cu[c + 1] - a.cu[c];
    }
    build_table3<NP>(tab, a, d, lane);
    const int ch = scan_row(a, d, b0 + grp) * a.dim + d;
    const int beg = s_beg[grp], n = s_n[grp];
    const int nch = (n + kChunkX - 1) / kChunkX;
    const int nch_max = warp_max(nch);

    // states advance in fp32x2 pairs (state 2h in .x, 2h+1 in .y): the same
    // fp32 operations, in the same order, as one state at a time
    static_assert(G % 2 == 0, "state pairs");
    constexpr int H = G / 2;
    float2 cc[H], ccA[H];
#pragma unroll
    for (int h = 0; h < H; ++h) {
        float c2[2], a2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int s = q * G + 2 * h + e;
            const bool o = s < N;
            const float Ar = o ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
            c2[e] = o ? a.B[d * N + s] * a.C[d * N + s] : 0.f;
            a2[e] = c2[e] * Ar;
        }
        cc[h] = make_float2(c2[0], c2[1]);
        ccA[h] = make_float2(a2[0], a2[1]);
    }
    const float dti = a.dt_idle[d], dta = a.dt_active[d];
    const float Dv = a.D ? a.D[d] : 0.f;
    const T* u = static_cast<const T*>(a.u);
    const T* dout = static_cast<const T*>(a.dout);
    // checkpoints: the forward's (slots by event index over the whole
    // channel), else this kernel's pass 1 (slots by index inside the chunk)
    const bool fwd_ck = a.ckpt != nullptr;
    float* const ck0 = (fwd_ck ? a.ckpt : a.ws_ckpt) + ((int64_t)(beg >> 3) + ch) * NP + q * G;

    // decays of one event: table row (row 0 = identity for padding slots);
    // EXACT batches send real events outside the table to exp2 in double
    auto decays = [&](auto exact_c, int kv, bool real, float dl, float (&dec)[G]) {
        constexpr bool EXACT = decltype(exact_c)::value;
        if (!EXACT) {
            tab_row3<G>(tab, kv, q, dec);
        } else {
            const bool hit = (unsigned)(kv - 1) < (unsigned)kKT3;
            tab_row3<G>(tab, (real && hit) ? kv : 0, q, dec);
            if (real && !hit) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int s = q * G + g;
                    const float Ar = s < N ? a.A[d * a.A_sd + s * a.A_sn] : 0.f;
                    dec[g] = decay_fast(dl, (float)((double)Ar * 1.4426950408889634));
                }
            }
        }
    };

    float2 gam[H], anx[H], SA[H], SB[H], QE[H];
    float tA[G], tB[G], tQ[G];
#pragma unroll
    for (int h = 0; h < H; ++h) {
        gam[h] = make_float2(0.f, 0.f);
        anx[h] = make_float2(1.f, 1.f);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) tA[g] = tB[g] = tQ[g] = 0.f;
    float t_ddi = 0.f, t_dda = 0.f, t_dD = 0.f;

    for (int c = nch_max - 1; c >= 0; --c) {
        const int cs = c * kChunkX;
        const int len = (c < nch) ? min(n - cs, kChunkX) : 0;
        const int len_max = warp_max(len);
        __syncwarp();
        if (lane < CPW) {
            const int nl = s_n[lane];
            s_cb[lane] = s_beg[lane] + cs;
            s_len[lane] = (cs < nl) ? min(nl - cs, kChunkX) : 0;
        }
        __syncwarp();
#pragma unroll
        for (int h = 0; h < H; ++h) SA[h] = SB[h] = QE[h] = make_float2(0.f, 0.f);
        float c_ddi = 0.f, c_dda = 0.f, c_dD = 0.f;
        float* const ck = fwd_ck ? ck0 + (int64_t)(cs >> 3) * NP : ck0;

        // ---- pass 1: checkpoints of the chunk -----------------------------
        if (!fwd_ck) {
            float eta[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                eta[g] = 0.f;
                const int s = q * G + g;
                if (c < nch && c > 0 && c - 1 < a.n_chunks && s < N) {
                    const float hv = a.x[((int64_t)ch * a.n_chunks + c - 1) * 2 * N + 2 * s + 1];
                    const float wb = a.B[d * N + s];
                    eta[g] = (wb != 0.f) ? hv / wb : 0.f;
                }
            }
            float pu[CPW];
            int pk[CPW];
            fetch_f<T, CPW>(u, s_cb, s_len, 0, lane, pu);
            fetch_k<CPW>(a.k, s_cb, s_len, 0, lane, pk);
            for (int j0 = 0; j0 < len_max; j0 += kR3) {
                const bool exact = batch_needs_exact<CPW>(pk, s_len, j0, lane, dti, dta, INFINITY);
                __syncwarp();
                stage<CPW, P>(s_u, pu, lane);
                stage<CPW, P>(s_k, pk, lane);
                __syncwarp();
                if (j0 + kR3 < len_max) {
                    fetch_f<T, CPW>(u, s_cb, s_len, j0 + kR3, lane, pu);
                    fetch_k<CPW>(a.k, s_cb, s_len, j0 + kR3, lane, pk);
                }
                auto run = [&](auto exact_c) {
#pragma unroll 1
                    for (int t = 0; t < kR3 / TB; ++t) {
                        if (j0 + t * TB < len) ck_store<G>(ck + (int64_t)((j0 + t * TB) / TB) * NP, eta);
#pragma unroll
                        for (int ii = 0; ii < TB; ++ii) {
                            const int i = t * TB + ii;
                            const float uv = s_u[i * P + grp];
                            const int kv = s_k[i * P + grp];
                            const float dl = event_delta(dti, dta, kv);
                            float dec[G];
                            decays(exact_c, kv, j0 + i < len, dl, dec);
                            const float w = dl * uv * uv;
#pragma unroll
                            for (int g = 0; g < G; ++g) eta[g] = fmaf(dec[g], eta[g], w);
                        }
                    }
                };
                if (exact) run(std::true_type{}); else run(std::false_type{});
            }
        }

        // ---- pass 2: batches, tiles and events last to first --------------
        if (len_max > 0) {
            float pu[CPW], pd[CPW];
            int pk[CPW];
            const int jlast = ((len_max - 1) / kR3) * kR3;
            auto fetch_all = [&](int jb) {
                fetch_f<T, CPW>(u, s_cb, s_len, jb, lane, pu);
                fetch_k<CPW>(a.k, s_cb, s_len, jb, lane, pk);
                fetch_f<T, CPW>(dout, s_cb, s_len, jb, lane, pd);
                if (a.z != nullptr) {
                    // gate: dout * z * sigmoid(z); dz written by the one lane that holds the event
                    const int j = jb + lane;
#pragma unroll
                    for (int c2 = 0; c2 < CPW; ++c2) {
                        if (j < s_len[c2]) {
                            const int e = s_cb[c2] + j;
                            const float zv = to_f32<T>(static_cast<const T*>(a.z)[e]);
                            const float sg = 1.0f / (1.0f + expf(-zv));
                            const float ov = to_f32<T>(static_cast<const T*>(a.out_fwd)[e]);
                            static_cast<T*>(a.dz)[e] = from_f32<T>(pd[c2] * ov * sg * (1.0f + zv * (1.0f - sg)));
                            pd[c2] = pd[c2] * (zv * sg);
                        }
                    }
                }
            };
            fetch_all(jlast);
            for (int jb = jlast; jb >= 0; jb -= kR3) {
                const bool exact = batch_needs_exact<CPW>(pk, s_len, jb, lane, dti, dta, INFINITY);
                __syncwarp();
                stage<CPW, P>(s_u, pu, lane);
                stage<CPW, P>(s_k, pk, lane);
                stage<CPW, P>(s_d, pd, lane);
                __syncwarp();
                if (jb > 0) fetch_all(jb - kR3);
                float eN[G];
                {
                    const int jt = jb + (kR3 / TB - 1) * TB;
                    ck_load<G>(ck + (int64_t)(jt / TB) * NP, jt < len, eN);
                }
                auto run = [&](auto exact_c) {
#pragma unroll 1
                    for (int t = kR3 / TB - 1; t >= 0; --t) {
                        const int i0 = t * TB;
                        float2 et[H], e0[H];
#pragma unroll
                        for (int h = 0; h < H; ++h) et[h] = e0[h] = make_float2(eN[2 * h], eN[2 * h + 1]);
                        if (t > 0) {   // next (earlier) tile's checkpoint
                            const int jt = jb + i0 - TB;
                            ck_load<G>(ck + (int64_t)(jt / TB) * NP, jt < len, eN);
                        }
                        // forward recompute of the tile
                        float2 eti[TB][H];
                        float te[TB], tg[TB], ta[TB];
#pragma unroll
                        for (int ii = 0; ii < TB; ++ii) {
                            const int i = i0 + ii;
                            const float uv = s_u[i * P + grp];
                            const int kv = s_k[i * P + grp];
                            const float qv = s_d[i * P + grp] * uv;
                            const float dl = event_delta(dti, dta, kv);
                            float dec[G];
                            decays(exact_c, kv, jb + i < len, dl, dec);
                            const float w = dl * uv * uv;
                            const float2 w2 = make_float2(w, w), q2 = make_float2(qv, qv);
                            float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
                            for (int h = 0; h < H; ++h) {
                                et[h] = __ffma2_rn(make_float2(dec[2 * h], dec[2 * h + 1]), et[h], w2);
                                eti[ii][h] = et[h];
                                s2 = __ffma2_rn(cc[h], et[h], s2);
                                QE[h] = __ffma2_rn(q2, et[h], QE[h]);
                            }
                            te[ii] = s2.x + s2.y;
                        }
                        // reverse over the tile: per-lane partial sums
#pragma unroll
                        for (int ii = TB - 1; ii >= 0; --ii) {
                            const int i = i0 + ii;
                            const float uv = s_u[i * P + grp];
                            const int kv = s_k[i * P + grp];
                            const float qv = s_d[i * P + grp] * uv;
                            const float dl = event_delta(dti, dta, kv);
                            float dec[G];
                            decays(exact_c, kv, jb + i < len, dl, dec);
                            const float w = dl * uv * uv;
                            const float2 w2 = make_float2(w, w), q2 = make_float2(qv, qv), dl2 = make_float2(dl, dl);
                            float2 tg2 = make_float2(0.f, 0.f), ta2 = make_float2(0.f, 0.f);
#pragma unroll
                            for (int h = 0; h < H; ++h) {
                                const float2 dc = make_float2(dec[2 * h], dec[2 * h + 1]);
                                gam[h] = __ffma2_rn(anx[h], gam[h], q2);
                                // gam * (eta_i - w_i), formed as gam * a_i * eta_{i-1}:
                                // no cancellation when the state has decayed
                                const float2 ep = (ii > 0) ? eti[ii > 0 ? ii - 1 : 0][h] : e0[h];
                                const float2 pr = __fmul2_rn(gam[h], __fmul2_rn(dc, ep));
                                SB[h] = __ffma2_rn(gam[h], w2, SB[h]);
                                SA[h] = __ffma2_rn(pr, dl2, SA[h]);
                                ta2 = __ffma2_rn(ccA[h], pr, ta2);
                                tg2 = __ffma2_rn(cc[h], gam[h], tg2);
                                anx[h] = dc;
                            }
                            tg[ii] = tg2.x + tg2.y;
                            ta[ii] = ta2.x + ta2.y;
                        }
                        group_transpose_sum<LPC, TB>(te, q);
                        group_transpose_sum<LPC, TB>(tg, q);
                        group_transpose_sum<LPC, TB>(ta, q);
                        // this lane finalises events i0 + q*EPL + e of the tile
#pragma unroll
                        for (int e = 0; e < EPL; ++e) {
                            const int i = i0 + q * EPL + e;
                            if (jb + i < s_len[grp]) {
                                const float uv = s_u[i * P + grp];
                                const int kv = s_k[i * P + grp];
                                const float dv = s_d[i * P + grp];
                                const float dl = event_delta(dti, dta, kv);
                                s_du[i * P + grp] = fmaf(Dv, dv, fmaf(2.f * uv * dl, tg[e], dv * te[e]));
                                const float ddel = fmaf(uv * uv, tg[e], ta[e]);
                                c_ddi = fmaf(ddel, (float)(kv - 1), c_ddi);
                                c_dda += ddel;
                                c_dD = fmaf(dv, uv, c_dD);
                            }
                        }
                    }
                };
                if (exact) run(std::true_type{}); else run(std::false_type{});
                __syncwarp();
                {
                    const int j = jb + lane;
                    T* du = static_cast<T*>(a.du);
#pragma unroll 4
                    for (int c2 = 0; c2 < CPW; ++c2)
                        if (j < s_len[c2]) du[s_cb[c2] + j] = from_f32<T>(s_du[lane * P + c2]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < H; ++h) {
            tA[2 * h] += SA[h].x;
            tA[2 * h + 1] += SA[h].y;
            tB[2 * h] += SB[h].x;
            tB[2 * h + 1] += SB[h].y;
            tQ[2 * h] += QE[h].x;
            tQ[2 * h + 1] += QE[h].y;
        }
        t_ddi += c_ddi;
        t_dda += c_dda;
        t_dD += c_dD;
    }
    // the scalar sums of a channel are spread over its LPC lanes
    t_ddi = group_sum<LPC>(t_ddi);
    t_dda = group_sum<LPC>(t_dda);
    t_dD = group_sum<LPC>(t_dD);
    float* part = a.ws_part + (int64_t)ch * a.part_stride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int s = q * G + g;
        if (s < N) {
            part[s] = ((g & 1) ? cc[g / 2].y : cc[g / 2].x) * tA[g];
            part[NP + s] = a.C[d * N + s] * tB[g];
            part[2 * NP + s] = a.B[d * N + s] * tQ[g];
        }
    }
    if (q == 0) {
        part[3 * NP] = t_ddi;
        part[3 * NP + 1] = t_dda;
        part[3 * NP + 2] = t_dD;
    }
}

// ====================================================== forward, split ====
// Two phases per staged batch of 32 events:
//   A  lane (channel, state group of G states) runs the recurrence
//      eta = a*eta + w over the batch and stores every state to shared memory
//      (only the state chain is sequential; a handful of instructions per
//      event and G <= 4 states per lane give many warps);
//   B  lane = event: y = D*u + u*sum_s cc_s*eta_s read back from shared
//      memory for each of the warp's channels, stored coalesced.
// A CTA holds the WPB warps of one feature d, which share one decay table.
template <int G, int NP>
struct V4 {
    static constexpr int LPC = NP / G;
    static constexpr int CPW = 32 / LPC;
    static constexpr int P = CPW + 1;
    static constexpr int EP = CPW * NP + 4;   // floats per event row of s_eta (== 4 mod 32)
    // per-warp region, a multiple of 4 floats so every warp's float4 rows
    // (s_eta, read as float4 in phase B) stay 16-byte aligned
    static constexpr int WARP_FLOATS = (4 * kR3 * P + kR3 * EP + 2 * CPW + 3) / 4 * 4;
};
static_assert(V4<2, 64>::WARP_FLOATS % 4 == 0 && V4<1, 16>::WARP_FLOATS % 4 == 0, "warp regions");

// Decay table of a CTA: [state][row] for G < 4 (scalar reads), float4
// groups [state/4][row] (as build_table3) for G >= 4.
template <int NP, int G>
__device__ void build_table_block(float* tab, const ScanArgs& a, int d) {
    for (int e = threadIdx.x; e < kRows3 * NP; e += blockDim.x) {
        const int row = e % kRows3, s = e / kRows3;
        const float v = table_entry<NP>(a, d, s, row);
        if (G >= 4) tab[((s >> 2) * kRows3 + row) * 4 + (s & 3)] = v;
        else if (G == 2) tab[((s >> 1) * kRows3 + row) * 2 + (s & 1)] = v;
        else tab[s * kRows3 + row] = v;
    }
}

template <int G>
__device__ __forceinline__ void tab_row4(const float* tab, int row, int s0, float (&dec)[G]) {
    if constexpr (G >= 4) {
        tab_row3<G>(tab, row, s0 / G, dec);
    } else if constexpr (G == 2) {
        const float2 v = reinterpret_cast<const float2*>(tab)[(s0 >> 1) * kRows3 + row];
        dec[0] = v.x;
        dec[1] = v.y;
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) dec[g] = tab[(s0 + g) * kRows3 + row];
    }
}

template <int G>
__device__ __forceinline__ void sts_vec(float* p, const float (&v)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4)
            *reinterpret_cast<float4*>(p + g) = make_float4(v[g], v[g + 1], v[g + 2], v[g + 3]);
    } else if constexpr (G == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) p[g] = v[g];
    }
}

// widest CTA of a layout (more state per lane, or a wider cc vector for
// phase B, needs more registers: smaller CTAs)
template <int G, int NP>
constexpr int v4_max_warps() { return G >= 8 ? 2 : (NP >= 32 ? 8 : 16); }

template <typename T, int G, int NP>
__global__ void __launch_bounds__(32 * v4_max_warps<G, NP>())
dw_fwd_v4(ScanArgs a, int blocks_per_d) {
    using V = V4<G, NP>;
    constexpr int CPW = V::CPW, P = V::P, LPC = V::LPC, EP = V::EP;
    extern __shared__ __align__(16) float sm4[];
    const int nwarps = blockDim.x >> 5;
    {
        // the layout below needs this much dynamic shared memory; never touch more
        unsigned dyn;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < (size_t)(NP * kRows3 + nwarps * V::WARP_FLOATS) * sizeof(float)) return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPC, q = lane % LPC;
    // rank-major: the CTAs holding every feature's longest rows start first
    const int d = rank_major(a) ? blockIdx.x % a.dim : blockIdx.x / blocks_per_d;
    const int b0 = ((rank_major(a) ? blockIdx.x / a.dim : blockIdx.x % blocks_per_d) * nwarps + warp) * CPW;
    float* tab = sm4;
    float* wbase = sm4 + NP * kRows3 + warp * V::WARP_FLOATS;
    float* s_u = wbase;
    int* s_k = reinterpret_cast<int*>(s_u + kR3 * P);
    float2* s_wr = reinterpret_cast<float2*>(s_k + kR3 * P);   // (w, table row as bits)
    float* s_eta = reinterpret_cast<float*>(s_wr + kR3 * P);
    int* s_beg = reinterpret_cast<int*>(s_eta + kR3 * EP);
    int* s_n = s_beg + CPW;
    const int N = a.dstate;

    if (lane < CPW) {
        const int c = scan_row(a, d, b0 + lane) * a.dim + d;
        s_beg[lane] = a.cu[c];
        s_n[lane] = a.cu[c + 1] - a.cu[c];
    }
    build_table_block<NP, G>(tab, a, d);
    __syncthreads();

    const int ch = scan_row(a, d, b0 + grp) * a.dim + d;
    const int n = s_n[grp];
    const int n_max = warp_max(n);
    const int s0 = q * G;

    float A2[G], eta[G], corr[G];
    float amax = 0.f;
    bool decaying = true;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int st = s0 + g;
        const float Ar = st < N ? a.A[d * a.A_sd + st * a.A_sn] : 0.f;
        A2[g] = (float)((double)Ar * 1.4426950408889634);
        eta[g] = corr[g] = 0.f;
        amax = fmaxf(amax, fabsf(A2[g]));
        decaying = decaying && A2[g] <= 0.f;
    }
    // phase B needs cc of every state
    // as pairs (state 2h in .x, 2h+1 in .y) for the packed output sum
    float2 ccall[NP / 2];
#pragma unroll
    for (int h = 0; h < NP / 2; ++h)
        ccall[h] = make_float2(2 * h < N ? a.B[d * N + 2 * h] * a.C[d * N + 2 * h] : 0.f,
                               2 * h + 1 < N ? a.B[d * N + 2 * h + 1] * a.C[d * N + 2 * h + 1] : 0.f);
    const float dti = a.dt_idle[d], dta = a.dt_active[d];
    const float Dv = a.D ? a.D[d] : 0.f;
    decaying = decaying && dti >= 0.f && dta >= 0.f;
    const float dclamp = amax > 0.f ? 126.0f / amax : INFINITY;
    const float dlim = warp_all_min(decaying ? INFINITY : dclamp);
    float sd[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) sd[c] = 0.f;

    // chunk states past the channel's last chunk are zero (the kernel writes
    // every slot of x: no pre-zeroing)
    for (int c = (n + kChunkX - 1) / kChunkX; c < a.n_chunks; ++c) {
        float* xo = a.x + ((int64_t)ch * a.n_chunks + c) * 2 * N;
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (s0 + g < N) {
                xo[2 * (s0 + g)] = 0.f;
                xo[2 * (s0 + g) + 1] = 0.f;
            }
    }
    // checkpoints for the backward: the state entering events 0, 8, 16, ...
    // of the channel (slot j/8 of the channel's region)
    float* ckb = nullptr;
    if (a.ckpt != nullptr) {
        ckb = a.ckpt + ((int64_t)(s_beg[grp] >> 3) + ch) * NP + s0;
        if (n > 0) sts_vec<G>(ckb, eta);
    }
    const T* u = static_cast<const T*>(a.u);
    float pu[CPW];
    int pk[CPW];
    fetch_f<T, CPW>(u, s_beg, s_n, 0, lane, pu);
    fetch_k<CPW>(a.k, s_beg, s_n, 0, lane, pk);
    for (int j0 = 0; j0 < n_max; j0 += kR3) {
        const bool exact = batch_needs_exact<CPW>(pk, s_n, j0, lane, dti, dta, dlim);
        {
            const int j = j0 + lane;
#pragma unroll
            for (int c = 0; c < CPW; ++c) {
                const bool real = j < s_n[c];
                const int kk = pk[c];
                const float dl = event_delta(dti, dta, kk);
                sd[c] += real ? dl : 0.f;
                s_u[lane * P + c] = pu[c];
                s_k[lane * P + c] = kk;
                const int row = (real && (unsigned)(kk - 1) < (unsigned)kKT3) ? kk : 0;
                s_wr[lane * P + c] = make_float2(dl * pu[c] * pu[c], __int_as_float(row));
            }
        }
        __syncwarp();
        if (j0 + kR3 < n_max) {
            fetch_f<T, CPW>(u, s_beg, s_n, j0 + kR3, lane, pu);
            fetch_k<CPW>(a.k, s_beg, s_n, j0 + kR3, lane, pk);
        }
        float* erow = s_eta + grp * NP + s0;
        // ---- phase A: the state recurrence of the batch
        if (!exact) {
            float dec[G];
            const float2 wr0 = s_wr[grp];
            tab_row4<G>(tab, __float_as_int(wr0.y), s0, dec);
            float w0 = wr0.x;
            float2 wr1 = s_wr[P + grp];
#pragma unroll 8
            for (int i = 0; i < kR3; ++i) {
                const int i2 = min(i + 2, kR3 - 1);
                float dn[G];
                tab_row4<G>(tab, __float_as_int(wr1.y), s0, dn);
                const float w1 = wr1.x;
                wr1 = s_wr[i2 * P + grp];
                if constexpr (G % 2 == 0) {   // state pairs in packed fp32x2 FMAs
#pragma unroll
                    for (int h = 0; h < G / 2; ++h) {
                        const float2 r = __ffma2_rn(make_float2(dec[2 * h], dec[2 * h + 1]),
                                                    make_float2(eta[2 * h], eta[2 * h + 1]), make_float2(w0, w0));
                        eta[2 * h] = r.x;
                        eta[2 * h + 1] = r.y;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < G; ++g) eta[g] = fmaf(dec[g], eta[g], w0);
                }
                sts_vec<G>(erow + i * EP, eta);
                if (ckb != nullptr && (i & 7) == 7 && j0 + i + 1 < n)
                    sts_vec<G>(ckb + (int64_t)((j0 + i + 1) >> 3) * NP, eta);
#pragma unroll
                for (int g = 0; g < G; ++g) dec[g] = dn[g];
                w0 = w1;
            }
        } else {
#pragma unroll 1
            for (int i = 0; i < kR3; ++i) {
                const float uv = s_u[i * P + grp];
                const int kv = s_k[i * P + grp];
                const bool real = j0 + i < n;
                const float dl = event_delta(dti, dta, kv);
                const bool hit = (unsigned)(kv - 1) < (unsigned)kKT3;
                float dec[G];
                tab_row4<G>(tab, (real && hit) ? kv : 0, s0, dec);
                if (real && (!hit || dl > dlim)) {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        // tabulated gaps keep the table's value (the backward
                        // reads the same table), others take exp2f
                        if (!hit) dec[g] = decay_fast(dl, A2[g]);
                        if (dl > dclamp) {
                            const float x = dl * A2[g];
                            corr[g] += fmaxf(fminf(x, 126.0f), -126.0f) - x;
                        }
                    }
                }
                const float w = real ? dl * uv * uv : 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) eta[g] = fmaf(dec[g], eta[g], w);
                sts_vec<G>(erow + i * EP, eta);
                if (ckb != nullptr && (i & 7) == 7 && j0 + i + 1 < n)
                    sts_vec<G>(ckb + (int64_t)((j0 + i + 1) >> 3) * NP, eta);
            }
        }
        // chunk state after a chunk end or after the channel's last event
        const int jend = j0 + kR3;
        const bool xw = n > j0 && (n <= jend || jend % kChunkX == 0);
        if (__any_sync(kFull, xw)) {
            float t[CPW];
#pragma unroll
            for (int c = 0; c < CPW; ++c) t[c] = sd[c];
            const float sdel = warp_channel_sum<CPW>(t, lane);
            const int c = (min(n, jend) - 1) / kChunkX;
            if (xw && c < a.n_chunks) {
                float* xo = a.x + ((int64_t)ch * a.n_chunks + c) * 2 * N;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const int st = s0 + g;
                    if (st < N) {
                        xo[2 * st] = exp2f(fmaf(A2[g], sdel, corr[g]));
                        xo[2 * st + 1] = a.B[d * N + st] * eta[g];
                    }
                }
            }
        }
        __syncwarp();
        // ---- phase B: lane = event, one output per warp channel
        {
            const int j = j0 + lane;
            T* out = static_cast<T*>(a.out);
            const float* ev = s_eta + lane * EP;
#pragma unroll 2
            for (int c = 0; c < CPW; ++c) {
                // four running sums (states st%4 = 0..3) as two packed pairs
                float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
                for (int st = 0; st < NP; st += 4) {
                    const float4 e4 = *reinterpret_cast<const float4*>(ev + c * NP + st);
                    s01 = __ffma2_rn(ccall[st / 2], make_float2(e4.x, e4.y), s01);
                    s23 = __ffma2_rn(ccall[st / 2 + 1], make_float2(e4.z, e4.w), s23);
                }
                const float acc = (s01.x + s01.y) + (s23.x + s23.y);
                const float uv = s_u[lane * P + c];
                const float y = fmaf(Dv, uv, uv * acc);
                if (j < s_n[c]) {
                    const int e = s_beg[c] + j;
                    out[e] = from_f32<T>(y);
                    if (a.z != nullptr) {
                        const float zv = to_f32<T>(static_cast<const T*>(a.z)[e]);
                        static_cast<T*>(a.out_z)[e] = from_f32<T>(y * silu(zv));
                    }
                }
            }
        }
        __syncwarp();
    }
}

template <typename T, int G, int NP>
bcm_status launch_fwd_v4(const ScanArgs& a, cudaStream_t st) {
    using V = V4<G, NP>;
    const int bn = a.n_channels / a.dim;
    const int groups = bn / V::CPW;          // warps per feature
    const int wmax = std::min(v4_max_warps<G, NP>(), std::max(1, env_int("BCM_V4_WPB", 16)));
    int wpb = 1;
    while (wpb * 2 <= wmax && groups % (wpb * 2) == 0) wpb *= 2;
    const int blocks_per_d = groups / wpb;
    const size_t smem = (size_t)(NP * kRows3 + wpb * V::WARP_FLOATS) * sizeof(float);
    if (smem > 48 * 1024) {
        // allow this kernel the device's opt-in maximum (once per device)
        static std::mutex mu;
        static int optin[64] = {};
        int dev = 0;
        BCM_CUDA_TRY(cudaGetDevice(&dev));
        BCM_REQUIRE(dev >= 0 && dev < 64, "flat_ch fwd: device %d out of range", dev);
        std::lock_guard<std::mutex> lock(mu);
        if (optin[dev] == 0) {
            int mx = 0;
            BCM_CUDA_TRY(cudaDeviceGetAttribute(&mx, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
            BCM_CUDA_TRY(cudaFuncSetAttribute(dw_fwd_v4<T, G, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx));
            optin[dev] = mx;
        }
        if (smem > (size_t)optin[dev]) {
            set_error("flat_ch fwd: %zu bytes of shared memory exceed the device limit %d", smem, optin[dev]);
            return BCM_ERR_UNSUPPORTED;
        }
    }
    dw_fwd_v4<T, G, NP><<<a.dim * blocks_per_d, wpb * 32, smem, st>>>(a, blocks_per_d);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

template <int G, int LPC>
size_t bwd_v3_smem() {
    using V = V3<G, LPC>;
    const size_t stg = (size_t)kR3 * V::P * sizeof(float);
    return V::TAB * sizeof(float) + 4 * stg + 4 * V::CPW * sizeof(int);   // < 48 KB
}

template <typename T, int G, int LPC>
bcm_status launch_bwd_v3(const ScanArgs& a, cudaStream_t st) {
    constexpr int CPW = V3<G, LPC>::CPW;
    const int bgroups = (a.n_channels / a.dim) / CPW;
    dw_bwd_v3<T, G, LPC><<<a.dim * bgroups, 32, bwd_v3_smem<G, LPC>(), st>>>(a, bgroups);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

// States per lane of the split forward (BCM_V4_G = 1, 2 or 4 overrides the
// default 2) and channels per warp of each direction.
int fwd_g() {
    static const int g = [] {
        const int v = env_int("BCM_V4_G", 2);
        return (v == 1 || v == 2 || v == 4) ? v : 2;
    }();
    return g;
}

int padded_states(int N) { return N <= 8 ? 8 : N <= 16 ? 16 : N <= 32 ? 32 : 64; }

// Backward states per lane up to 16 states (BCM_BWD_G = 2 overrides the default 4).
int bwd_g() {
    static const int g = env_int("BCM_BWD_G", 4) == 2 ? 2 : 4;
    return g;
}

int channels_per_warp(int N, bool bwd) {
    const int NP = padded_states(N);
    if (bwd) return NP <= 16 ? 32 * bwd_g() / NP : 256 / NP;   // 8 states per lane above 16
    return NP <= 16 ? 32 * fwd_g() / NP : 64 / NP;     // 2 states per lane above 16
}

}  // namespace

// The staged kernels apply when dstate <= 64 and the channels of one feature
// fill whole warps (n_channels / dim a multiple of the channels per warp).
bool v3_supported(const ScanArgs& a, bool bwd) {
    static const int mode = env_int("BCM_SCAN_V3", 1);
    if (mode == 0 || a.dstate > 64 || a.dim <= 0 || a.n_channels % a.dim != 0) return false;
    return (a.n_channels / a.dim) % channels_per_warp(a.dstate, bwd) == 0;
}

int v3_ckpt_np(int dstate) { return padded_states(dstate); }

int64_t v3_bwd_warps(const ScanArgs& a) {
    return (int64_t)a.n_channels / channels_per_warp(a.dstate, true);
}

size_t v3_ckpt_bytes(const ScanArgs& a) {
    if (a.bc_mode != BCM_BC_DEPTHWISE || a.n_events <= 0 || !v3_supported(a, false) || !v3_supported(a, true))
        return 0;
    const size_t slots = (size_t)(a.n_events >> 3) + (size_t)a.n_channels + 1;
    return slots * (size_t)padded_states(a.dstate) * sizeof(float);
}

// Batch rows of each feature by descending event count (ties by row): one
// CTA per feature ranks its rows by counting.  Rows past 4096 per feature
// keep their order (order[b] = b).
__global__ void row_order_kernel(const int32_t* __restrict__ cu, int dim, int Bn, int* __restrict__ order) {
    extern __shared__ int s_n[];
    const int d = blockIdx.x;
    for (int b = threadIdx.x; b < Bn; b += blockDim.x) {
        const int c = b * dim + d;
        s_n[b] = cu[c + 1] - cu[c];
    }
    __syncthreads();
    for (int b = threadIdx.x; b < Bn; b += blockDim.x) {
        const int nb = s_n[b];
        int rank = 0;
        for (int b2 = 0; b2 < Bn; ++b2) {
            const int n2 = s_n[b2];
            rank += (n2 > nb || (n2 == nb && b2 < b)) ? 1 : 0;
        }
        order[d * Bn + rank] = b;
    }
}

// Decay tables of the staged kernels, [dim][NP][kKT3 + 1], once per call.
__global__ void staged_table_kernel(ScanArgs a, int NP, float* __restrict__ tab) {
    const int64_t total = (int64_t)a.dim * NP * kRows3;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i % kRows3);
        const int64_t ds = i / kRows3;
        const int s = (int)(ds % NP), d = (int)(ds / NP);
        float v = 1.f;
        if (row > 0 && s < a.dstate) {
            const float A2 = (float)((double)a.A[d * a.A_sd + s * a.A_sn] * 1.4426950408889634);
            v = decay_exact(event_delta(a.dt_idle[d], a.dt_active[d], row), A2);
        }
        tab[i] = v;
    }
}

static size_t row_order_bytes(const ScanArgs& a) {
    return align_up((size_t)a.n_channels * sizeof(int), 256);
}

size_t staged_prep_bytes(const ScanArgs& a) {
    return row_order_bytes(a) + align_up((size_t)a.dim * padded_states(a.dstate) * kRows3 * sizeof(float), 256);
}

bcm_status staged_prep_launch(ScanArgs& a, void* ws, cudaStream_t st) {
    const int Bn = a.n_channels / a.dim;
    if (Bn > 4096) {
        set_error("flat_ch: row order needs at most 4096 rows per feature, got %d", Bn);
        return BCM_ERR_UNSUPPORTED;
    }
    int* order = static_cast<int*>(ws);
    float* tab = reinterpret_cast<float*>(static_cast<char*>(ws) + row_order_bytes(a));
    const int threads = std::min(256, std::max(32, (Bn + 31) / 32 * 32));
    row_order_kernel<<<a.dim, threads, Bn * sizeof(int), st>>>(a.cu, a.dim, Bn, order);
    BCM_LAUNCH_CHECK();
    const int NP = padded_states(a.dstate);
    const int64_t total = (int64_t)a.dim * NP * kRows3;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
    staged_table_kernel<<<grid, 256, 0, st>>>(a, NP, tab);
    BCM_LAUNCH_CHECK();
    a.row_order = order;
    a.dtab = tab;
    a.rank_major = env_int("BCM_V3_RANK_MAJOR", 1) != 0;
    return BCM_OK;
}

bcm_status v3_launch(const ScanArgs& a, bcm_dtype dtype, bool bwd, cudaStream_t st) {
    const int g = fwd_g();
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        if (bwd) {
            if (a.dstate <= 8) return bwd_g() == 2 ? launch_bwd_v3<T, 2, 4>(a, st) : launch_bwd_v3<T, 4, 2>(a, st);
            if (a.dstate <= 16) return bwd_g() == 2 ? launch_bwd_v3<T, 2, 8>(a, st) : launch_bwd_v3<T, 4, 4>(a, st);
            if (a.dstate <= 32) return launch_bwd_v3<T, 8, 4>(a, st);
            return launch_bwd_v3<T, 8, 8>(a, st);
        }
        if (a.dstate > 32) return launch_fwd_v4<T, 2, 64>(a, st);
        if (a.dstate > 16) return launch_fwd_v4<T, 2, 32>(a, st);
        if (a.dstate <= 8) {
            if (g == 1) return launch_fwd_v4<T, 1, 8>(a, st);
            if (g == 4) return launch_fwd_v4<T, 4, 8>(a, st);
            return launch_fwd_v4<T, 2, 8>(a, st);
        }
        if (g == 1) return launch_fwd_v4<T, 1, 16>(a, st);
        if (g == 4) return launch_fwd_v4<T, 4, 16>(a, st);
        return launch_fwd_v4<T, 2, 16>(a, st);
    });
}

}  // namespace bcm
