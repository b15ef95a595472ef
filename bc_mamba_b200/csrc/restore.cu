// restore.cu — causal zero-order-hold restore of event values to the dense
// (B, L, D) layout, and its backward (per-event segment sums of dout).
//
// Semantics follow csrc/r_nodecay/restore_dense_fwd_kernel.cuh:38-112 and
// restore_dense_bwd_kernel.cuh:42-113: out[b,t,d] = y[e*] with e* the last
// event of channel b*D+d at or before t (0 before the first event); the
// reference's 12-step search reaches at most event 4094 of a channel, so only
// the first min(n, 4095) events are addressable and the last of them holds to
// L.  dy[e] = sum of dout over [t_e, t_{e+1}) (L for the last addressable
// event), 0 for unaddressable events, always fp32.
//
// Design (ours).  A CTA owns one batch row b, 32 consecutive features and a
// range of positions, walked in windows of kTT = 128 positions:
//   1. staging: each warp loads the window's events of 8 channels (32 events
//      per coalesced load) and builds a 128-bit event mask per channel with
//      warp OR-reductions (plus, forward, the event values in order); the
//      first batch of the next window is loaded while the current one is swept;
//   2. sweep: warp w takes positions [32w, 32w+32) of the window and lane c
//      takes channel c, so every position is one coalesced row of 32 features
//      of (B, L, D): the forward stores the held value row by row, the
//      backward loads its 32 rows up front and closes a segment sum at each
//      set bit of the mask.
// No global load sits in the sweep.  The backward combines the four
// sub-window partials of each channel in order and the CTA owning an event's
// start keeps reading past its range until the event ends, so each dy is
// summed in one fixed order (the reference uses fp32 atomics).
#include "common.cuh"

namespace bcm {
namespace {

constexpr int kDB = 32;       // features per CTA
constexpr int kTT = 128;      // positions per window
constexpr int kWarpsR = 4;    // warps per CTA; warp w sweeps positions [32w, 32w+32)
constexpr int kChPerWarp = kDB / kWarpsR;
constexpr int kCap = 4095;    // addressable events per channel (reference search limit)
constexpr int kMW = kTT / 32; // mask words per channel and window
constexpr int kMP = kMW + 1;  // padded mask pitch (conflict-free column reads)

__device__ __forceinline__ int lower_bound_i32(const int32_t* a, int n, int key) {
    int lo = 0, hi = n;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (a[mid] < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Staging of one channel's events in [t0, wend) starting at local index p:
// sets the channel's mask words, optionally stores the values in order, and
// returns the number of events taken (warp-uniform).  Events are loaded 32 at
// a time with one coalesced load per array.
// (t0_pre, v0_pre) are this lane's first-batch event time and value, loaded
// by the caller for all of a warp's channels at once so their latencies overlap.
template <typename Tin, bool VALUES>
__device__ __forceinline__ int stage_channel(const int32_t* ts, const Tin* y, int beg, int n, int p,
                                             int t0, int wend, uint32_t* mask, float* vals,
                                             int lane, float& last_val, int t_pre, float v_pre) {
    uint32_t m[kMW];
#pragma unroll
    for (int w = 0; w < kMW; ++w) m[w] = 0u;
    int taken = 0;
    int t = t_pre;
    float v = v_pre;
    while (true) {
        const bool valid = t >= t0 && t < wend && taken + lane < kTT;
        const int cnt = __popc(__ballot_sync(kFull, valid));
        const int rel = valid ? t - t0 : -1;
#pragma unroll
        for (int w = 0; w < kMW; ++w)
            m[w] |= __reduce_or_sync(kFull, (valid && (rel >> 5) == w) ? (1u << (rel & 31)) : 0u);
        if (VALUES) {
            if (valid) vals[taken + lane] = v;
            if (cnt > 0) last_val = __shfl_sync(kFull, v, cnt - 1);
        }
        taken += cnt;
        if (cnt < 32) break;
        // a dense window: the next 32 events of this channel
        const int j = p + taken + lane;
        t = (j < n) ? ts[beg + j] : INT_MAX;
        if (VALUES) v = (j < n) ? to_f32<Tin>(y[beg + j]) : 0.f;
    }
    if (lane < kMW) {
#pragma unroll
        for (int w = 0; w < kMW; ++w)
            if (lane == w) mask[w] = m[w];
    }
    return taken;
}


template <typename T>
__global__ void __launch_bounds__(kWarpsR * 32)
restore_bwd_kernel(const T* __restrict__ dout, const int32_t* __restrict__ ts,
                   const int32_t* __restrict__ cu, int D, int L, int part_len,
                   int n_dblk, float* __restrict__ dy) {
    __shared__ uint32_t s_mask[kDB][kMP];
    __shared__ float s_head[kWarpsR][kDB], s_tail[kWarpsR][kDB];
    __shared__ int s_cnt[kWarpsR][kDB];
    __shared__ int s_p[kDB];
    __shared__ int s_any;
    const int dblk = blockIdx.x % n_dblk;
    const int part = blockIdx.x / n_dblk;
    const int b = blockIdx.y;
    const int d0 = dblk * kDB;
    const int t_beg = part * part_len;
    const int t_own_end = min(L, t_beg + part_len);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    int c_beg[kChPerWarp], c_n[kChPerWarp];
#pragma unroll
    for (int ci = 0; ci < kChPerWarp; ++ci) {
        const int d = d0 + warp * kChPerWarp + ci;
        c_beg[ci] = 0; c_n[ci] = 0;
        if (d < D) {
            const int ch = b * D + d;
            c_beg[ci] = cu[ch];
            const int n_all = cu[ch + 1] - c_beg[ci];
            c_n[ci] = min(n_all, kCap);
            if (part == 0)  // events past the search cap receive no gradient
                for (int j = kCap + lane; j < n_all; j += 32) dy[c_beg[ci] + j] = 0.f;
        }
    }
    if (lane < kChPerWarp) {
        int beg = 0, n = 0;
#pragma unroll
        for (int ci = 0; ci < kChPerWarp; ++ci)
            if (ci == lane) { beg = c_beg[ci]; n = c_n[ci]; }
        s_p[warp * kChPerWarp + lane] = lower_bound_i32(ts + beg, n, t_beg);
    }
    // interval bookkeeping of channel `lane` (threads of warp 0 only):
    // open = global index of the event whose interval is running (ours), -1 none
    int open = -1;
    float open_acc = 0.f;
    int p_next[kChPerWarp];
    const int my_d = d0 + lane;
    const bool cvalid = my_d < D;
    const int my_beg = cvalid ? cu[b * D + my_d] : 0;
    __syncthreads();
    // first 32 events of every channel of the next window, loaded ahead
    int t_pre[kChPerWarp];
    auto prefetch = [&](const int (&pp)[kChPerWarp]) {
#pragma unroll
        for (int ci = 0; ci < kChPerWarp; ++ci) {
            const int j = pp[ci] + lane;
            t_pre[ci] = (j < c_n[ci]) ? ts[c_beg[ci] + j] : INT_MAX;
        }
    };
    {
        int p0[kChPerWarp];
#pragma unroll
        for (int ci = 0; ci < kChPerWarp; ++ci) p0[ci] = s_p[warp * kChPerWarp + ci];
        prefetch(p0);
    }

    for (int t0 = t_beg; t0 < L; t0 += kTT) {
        const bool owning = t0 < t_own_end;
        if (!owning) {
            if (threadIdx.x == 0) s_any = 0;
            __syncthreads();
            if (warp == 0 && open >= 0) s_any = 1;
            __syncthreads();
            if (!s_any) break;
        }
        const int wend = min(t0 + kTT, L);
        // 1. this warp's 32 rows of the window (lane = channel: each row one
        //    coalesced load of 32 features) are issued first, then the staging
        //    of event masks.  Each warp publishes the advanced pointers of its
        //    own channels from the previous window (the previous combine read
        //    the old values).
        const int tw = t0 + warp * 32;
        float v[32];
        {
            const T* col = dout + ((int64_t)b * L + tw) * D + my_d;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = (cvalid && tw + i < wend) ? to_f32<T>(col[(int64_t)i * D]) : 0.f;
        }
        if (t0 != t_beg && lane < kChPerWarp) {
#pragma unroll
            for (int ci = 0; ci < kChPerWarp; ++ci)
                if (ci == lane) s_p[warp * kChPerWarp + ci] = p_next[ci];
        }
        __syncwarp();
#pragma unroll
        for (int ci = 0; ci < kChPerWarp; ++ci) {
            const int c = warp * kChPerWarp + ci;
            float dummy = 0.f;
            const int p = s_p[c];
            p_next[ci] = p + stage_channel<T, false>(ts, nullptr, c_beg[ci], c_n[ci], p, t0, wend,
                                                     s_mask[c], nullptr, lane, dummy, t_pre[ci], 0.f);
        }
        prefetch(p_next);   // in flight during the sweep and combine
        __syncthreads();
        // 2. sweep: lane = channel, positions [32w, 32w+32) of the window
        {
            const int c = lane;
            uint32_t before = 0;
#pragma unroll
            for (int w = 0; w < kMW; ++w)
                if (w < warp) before += __popc(s_mask[c][w]);
            const uint32_t mw = s_mask[c][warp];
            const int ebase = my_beg + s_p[c] + (int)before;   // global index of this piece's first event
            float acc = 0.f, head = 0.f;
            int e = 0;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if ((mw >> i) & 1u) {
                    if (e == 0) head = acc;
                    else if (owning) dy[ebase + e - 1] = acc;   // interval inside the piece
                    acc = 0.f;
                    ++e;
                }
                acc += v[i];
            }
            if (e == 0) head = acc;
            s_head[warp][c] = head;
            s_tail[warp][c] = acc;
            s_cnt[warp][c] = e;
        }
        __syncthreads();
        // 3. ordered combine of the four pieces (warp 0, lane = channel)
        if (warp == 0 && my_d < D) {
            const int c = lane;
            int ebase = my_beg + s_p[c];
#pragma unroll
            for (int w = 0; w < kWarpsR; ++w) {
                const int cnt = s_cnt[w][c];
                if (cnt > 0) {
                    if (open >= 0) dy[open] = open_acc + s_head[w][c];
                    ebase += cnt;
                    open = owning ? ebase - 1 : -1;
                    open_acc = s_tail[w][c];
                } else {
                    open_acc += s_head[w][c];
                }
            }
        }
        __syncthreads();
    }
    // intervals still open at L end there
    if (warp == 0 && my_d < D && open >= 0) dy[open] = open_acc;
}

// ---- bitmap backward -------------------------------------------------------------
// A pre-pass marks every addressable event (the first kCap of a channel, at a
// position in [0, L)) in a bitmap [b][t/32][d]: one warp per channel, its
// sorted times combined into 32-bit words with a segmented OR over the lanes
// (a word cut by a 32-event batch is carried to the next), every word written
// once with a plain store.  The backward then needs no event times: a warp
// owns one batch row b, 32 features (lane = channel) and a range of
// positions, and per 32-row window reads one coalesced mask word per lane and
// the 32 rows (coalesced), closing a channel's interval sum at each set bit
// (in row order: deterministic); it keeps reading past its range until the
// intervals it owns have ended.
constexpr int kBU = 4;   // units (warps) per CTA

__global__ void event_bitmap_kernel(const int32_t* __restrict__ ts, const int32_t* __restrict__ cu,
                                    int64_t n_ch, int D, int L, int nw, uint32_t* __restrict__ bm) {
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= n_ch) return;
    const int lane = threadIdx.x & 31;
    const int64_t b = c / D;
    const int d = (int)(c % D);
    const int beg = cu[c];
    const int n = min(cu[c + 1] - beg, kCap);
    uint32_t* col = bm + b * nw * (int64_t)D + d;          // word w at col[w * D]
    int carry_w = -1;
    uint32_t carry_bits = 0u;
    constexpr int kPre = 16;                                  // batches whose loads are issued together
    for (int g0 = 0; g0 < n; g0 += 32 * kPre) {
    int tpre[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const int j = g0 + 32 * i + lane;
        tpre[i] = (j < n) ? ts[beg + j] : -1;
    }
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const int j0 = g0 + 32 * i;
        if (j0 >= n) break;
        const int j = j0 + lane;
        const int t = tpre[i];
        const bool ok = j < n && t >= 0 && t < L;
        const int w = ok ? (t >> 5) : -2 - lane;              // invalid lanes form their own segments
        uint32_t bits = ok ? (1u << (t & 31)) : 0u;
        if (lane == 0 && carry_w >= 0) {                      // the previous batch's last word
            if (w == carry_w) bits |= carry_bits;             // continues here
            else col[(int64_t)carry_w * D] = carry_bits;      // or is complete
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {              // inclusive segmented OR from the left
            const uint32_t ob = __shfl_up_sync(kFull, bits, off);
            const int owd = __shfl_up_sync(kFull, w, off);
            if (lane >= off && owd == w) bits |= ob;
        }
        const int w_next = __shfl_down_sync(kFull, w, 1);
        const bool last = (lane == 31);
        if (ok && !last && w_next != w) col[(int64_t)w * D] = bits;
        carry_w = __shfl_sync(kFull, w, 31);
        carry_bits = __shfl_sync(kFull, bits, 31);
        if (carry_w < 0) carry_bits = 0u;
    }
    }
    if (lane == 0 && carry_w >= 0) col[(int64_t)carry_w * D] = carry_bits;
}

struct BUnit {
    int64_t b;
    int d0, t_beg, t_end;
};

__device__ __forceinline__ BUnit bunit(int64_t unit, int n_dblk, int n_parts, int part_len, int L) {
    BUnit u;
    const int part = (int)(unit % n_parts);
    const int64_t rest = unit / n_parts;
    u.d0 = (int)(rest % n_dblk) * 32;
    u.b = rest / n_dblk;
    u.t_beg = part * part_len;
    u.t_end = min(L, u.t_beg + part_len);
    return u;
}

// k-ary lower bound: first index in [0, n) with a[i] >= key (n if none);
// each round issues 7 independent probes, so n <= 4096 takes 4 load rounds.
__device__ __forceinline__ int lower_bound8(const int32_t* __restrict__ a, int n, int key) {
    int lo = 0, hi = n;   // the answer lies in [lo, hi]
    while (hi - lo > 8) {
        const int step = (hi - lo + 7) >> 3;
        int c = 0;
#pragma unroll
        for (int k = 1; k < 8; ++k) {
            const int p = lo + step * k;
            c += (p < hi && a[p] < key) ? 1 : 0;
        }
        const int nhi = lo + step * (c + 1);
        lo = (c > 0) ? lo + step * c + 1 : lo;
        hi = min(hi, nhi);
    }
    int c = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) c += (lo + k < hi && a[lo + k] < key) ? 1 : 0;
    return lo + c;
}

// ---- sweep forward -------------------------------------------------------------
// A warp owns one batch row b, 32 features (lane = channel) and a range of
// positions [t_beg, t_end) (whole 32-position words).  Each lane finds its
// channel's first event at or after t_beg, then keeps the times and values of
// its next kQ events in registers, loaded kQ events ahead so every load has
// kQ gaps' worth of positions to arrive.  Per position the lane holds or
// replaces its value and the warp stores one coalesced row of 32 features;
// per 32 positions each lane stores its word of event bits (the bitmap the
// backward sweeps), and the unit records its lanes' first event indices.
// No shared memory and few registers, so many units run per SM.
constexpr int kQ = 4;               // events held ahead per lane
constexpr int kFU = 4;              // units (warps) per CTA
constexpr int kSweepUnitsPerSM = 48;

struct SweepLayout {
    int n_dblk, part_len, n_parts;
    int64_t n_units;
};

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kFU * 32)
restore_fwd_sweep(const Tin* __restrict__ y, const int32_t* __restrict__ ts, const int32_t* __restrict__ cu,
                  int D, int L, int nw, int part_len, int n_dblk, int n_parts, int64_t n_units,
                  Tout* __restrict__ out, uint32_t* __restrict__ bm, int32_t* __restrict__ e_start) {
    const int64_t unit = (int64_t)blockIdx.x * kFU + (threadIdx.x >> 5);
    if (unit >= n_units) return;   // warp-uniform; the kernel has no block barrier
    const int lane = threadIdx.x & 31;
    const BUnit u = bunit(unit, n_dblk, n_parts, part_len, L);
    const int d = u.d0 + lane;
    const bool valid = d < D;
    int beg = 0, n = 0;
    if (valid) {
        const int64_t c = u.b * D + d;
        beg = cu[c];
        n = min(cu[c + 1] - beg, kCap);
    }
    const int p = (u.t_beg == 0 || n <= 0) ? 0 : lower_bound8(ts + beg, n, u.t_beg);
    if (e_start != nullptr) e_start[unit * 32 + lane] = p;
    float cur = (p > 0) ? to_f32<Tin>(y[beg + p - 1]) : 0.f;
    int tq[kQ];
    float yq[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
        const int j = p + q;
        tq[q] = (j < n) ? ts[beg + j] : INT_MAX;
        yq[q] = (j < n) ? to_f32<Tin>(y[beg + j]) : 0.f;
    }
    int nxt = p + kQ;
    Tout* col = out + (u.b * L + u.t_beg) * (int64_t)D + (valid ? d : 0);
    uint32_t* mcol = (bm != nullptr) ? bm + (u.b * nw + (u.t_beg >> 5)) * (int64_t)D + d : nullptr;
    for (int t0 = u.t_beg; t0 < u.t_end; t0 += 32) {
        uint32_t m = 0u;
        const int rows = min(32, u.t_end - t0);
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            if (r >= rows) break;   // warp-uniform
            if (t0 + r == tq[0]) {
                cur = yq[0];
#pragma unroll
                for (int q = 0; q + 1 < kQ; ++q) {
                    tq[q] = tq[q + 1];
                    yq[q] = yq[q + 1];
                }
                tq[kQ - 1] = (nxt < n) ? ts[beg + nxt] : INT_MAX;
                yq[kQ - 1] = (nxt < n) ? to_f32<Tin>(y[beg + nxt]) : 0.f;
                ++nxt;
                m |= 1u << r;
            }
            if (valid) col[(int64_t)r * D] = from_f32<Tout>(cur);
        }
        if (mcol != nullptr && valid) *mcol = m;
        col += (int64_t)32 * D;
        if (mcol != nullptr) mcol += D;
    }
}

// ---- word sweep forward (bitmap first) ---------------------------------------------
// With the event bitmap built first (event_bitmap_kernel), a warp unit
// (b, 32 features, positions [t_beg, t_end), the units of the sweep layout)
// needs no event times in its sweep.  Per 32-position word each lane reads
// its mask word (one coalesced load per warp, two words ahead) and copies the
// word's event values, consecutive in its channel's stream, into its column
// of a shared-memory slot buffer by 4-byte cp.async one word ahead; row r of
// the word then holds the value of event popc(mask & bits 0..r) - 1 of the
// word, or the value held into the word when that count is 0: branch-free,
// with every row one coalesced store of 32 features.  The unit still records
// its lanes' first event indices for the backward.
constexpr int kWU = 4;   // units (warps) per CTA, as the sweep layout's kFU

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int NG>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(NG) : "memory"); }

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kWU * 32)
restore_fwd_words(const Tin* __restrict__ y, const int32_t* __restrict__ ts, const int32_t* __restrict__ cu,
                  const uint32_t* __restrict__ bm, int D, int L, int nw, int part_len, int n_dblk, int n_parts,
                  int64_t n_units, Tout* __restrict__ out, int32_t* __restrict__ e_start) {
    __shared__ float s_val[kWU][2][32][32];   // [warp][buffer][slot][lane]
    const int wi = threadIdx.x >> 5;
    const int64_t unit = (int64_t)blockIdx.x * kWU + wi;
    if (unit >= n_units) return;   // warp-uniform; the kernel has no block barrier
    const int lane = threadIdx.x & 31;
    const BUnit u = bunit(unit, n_dblk, n_parts, part_len, L);
    const int d = u.d0 + lane;
    const bool valid = d < D;
    const int dc = valid ? d : D - 1;   // lanes past D address a real column and store nothing
    int beg = 0, n = 0;
    if (valid) {
        const int64_t c = u.b * D + d;
        beg = cu[c];
        n = min(cu[c + 1] - beg, kCap);
    }
    const int p = (u.t_beg == 0 || n <= 0) ? 0 : lower_bound8(ts + beg, n, u.t_beg);
    if (e_start != nullptr) e_start[unit * 32 + lane] = p;
    float cur = (p > 0) ? to_f32<Tin>(y[beg + p - 1]) : 0.f;
    int idx = beg + p;   // the next event (global index)
    const uint32_t* mcol = bm + (u.b * nw + (u.t_beg >> 5)) * (int64_t)D + dc;
    const int nwd = (u.t_end - u.t_beg + 31) >> 5;   // words of the unit
    auto mask_at = [&](int w) -> uint32_t { return (valid && w < nwd) ? mcol[(int64_t)w * D] : 0u; };
    // the values of a word's events (from global index first) into slot buffer buf
    // (a bitmap with more bits than the channel has events, e.g. an
    // extraction mask passed with another stream, reads no further than the
    // channel's last event)
    auto fetch = [&](uint32_t m, int first, int buf) {
        const int nv = min(__popc(m), beg + n - first);
        float(*sv)[32] = s_val[wi][buf];
        for (int k = 0; k < nv; ++k) {
            if constexpr (sizeof(Tin) == 4) {
                cp_async4(&sv[k][lane], y + first + k);
            } else {
                sv[k][lane] = to_f32<Tin>(y[first + k]);
            }
        }
        cp_async_commit();
    };
    uint32_t m0 = mask_at(0), m1 = mask_at(1);
    fetch(m0, idx, 0);
    Tout* col = out + (u.b * L + u.t_beg) * (int64_t)D + dc;
    for (int w = 0; w < nwd; ++w) {
        const int buf = w & 1;
        const uint32_t m2 = mask_at(w + 2);
        const int nv0 = __popc(m0);
        fetch(m1, idx + nv0, buf ^ 1);   // the next word's values, in flight during this word's rows
        cp_async_wait<1>();
        __syncwarp();
        const float(*sv)[32] = s_val[wi][buf];
        const int rows = min(32, u.t_end - (u.t_beg + 32 * w));
        if (rows == 32) {
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const int k = __popc(m0 & ((2u << r) - 1u));
                const float v = k ? sv[k ? k - 1 : 0][lane] : cur;
                if (valid) col[(int64_t)r * D] = from_f32<Tout>(v);
            }
        } else {
            for (int r = 0; r < rows; ++r) {
                const int k = __popc(m0 & ((2u << r) - 1u));
                const float v = k ? sv[k ? k - 1 : 0][lane] : cur;
                if (valid) col[(int64_t)r * D] = from_f32<Tout>(v);
            }
        }
        cur = nv0 ? sv[nv0 ? nv0 - 1 : 0][lane] : cur;
        idx += nv0;
        col += (int64_t)32 * D;
        __syncwarp();   // this buffer is refilled by the next word's fetch
        m0 = m1;
        m1 = m2;
    }
    cp_async_wait<0>();
}

template <typename T>
__global__ void __launch_bounds__(kBU * 32)
restore_bwd_bitmap(const T* __restrict__ dout, const int32_t* __restrict__ cu, const uint32_t* __restrict__ bm,
                   const int32_t* __restrict__ e_start, int D, int L, int nw, int part_len, int n_dblk,
                   int n_parts, int64_t n_units, float* __restrict__ dy) {
    const int64_t unit = (int64_t)blockIdx.x * kBU + (threadIdx.x >> 5);
    if (unit >= n_units) return;
    const int lane = threadIdx.x & 31;
    const BUnit u = bunit(unit, n_dblk, n_parts, part_len, L);
    const int d = u.d0 + lane;
    const bool valid = d < D;
    const int dc = valid ? d : D - 1;   // lanes past D read a real column and use none of it
    int beg = 0, n_all = 0;
    if (valid) {
        const int64_t c = u.b * D + d;
        beg = cu[c];
        n_all = cu[c + 1] - beg;
    }
    const uint32_t* mcol = bm + u.b * nw * (int64_t)D + dc;
    // local index of the first event at or after t_beg: recorded by the
    // forward, else the marked events before t_beg (times lie in [0, L), so
    // the bitmap holds exactly the first min(n, kCap) events)
    int p = 0;
    if (e_start != nullptr) {
        p = valid ? e_start[unit * 32 + lane] : 0;
    } else if (valid) {
#pragma unroll 8
        for (int w = 0; w < (u.t_beg >> 5); ++w) p += __popc(mcol[(int64_t)w * D]);
    }
    if (u.t_beg == 0)
        for (int j = kCap; j < n_all; ++j) dy[beg + j] = 0.f;      // past the search cap
    int e = beg + p;        // next event (global index)
    int open = -1;          // owned event whose interval is running
    float acc = 0.f;
    const T* col = dout + (u.b * L + u.t_beg) * (int64_t)D + dc;
    for (int t0 = u.t_beg; t0 < L; t0 += 32) {
        if (t0 >= u.t_end && !__any_sync(kFull, open >= 0)) break;
        const uint32_t m0 = valid ? mcol[(int64_t)(t0 >> 5) * D] : 0u;
        float v[32];
        if (t0 + 32 <= L) {
#pragma unroll
            for (int r = 0; r < 32; ++r) v[r] = to_f32<T>(col[(int64_t)r * D]);
        } else {
#pragma unroll
            for (int r = 0; r < 32; ++r) v[r] = (t0 + r < L) ? to_f32<T>(col[(int64_t)r * D]) : 0.f;
        }
        col += (int64_t)32 * D;
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const bool hit = ((m0 >> r) & 1u) != 0u;
            if (hit && open >= 0) dy[open] = acc;   // an event starts here: the running interval ends
            open = hit ? ((t0 + r < u.t_end) ? e : -1) : open;
            e += hit ? 1 : 0;
            acc = (hit ? 0.f : acc) + v[r];
        }
    }
    if (open >= 0) dy[open] = acc;              // the interval runs to L
}

}  // namespace
}  // namespace bcm

using namespace bcm;

static int restore_part_len(int64_t n_blocks_2d, int64_t L) {
    // Enough CTAs to cover the SMs several times; whole windows per part.
    const int64_t target = (int64_t)sm_count() * 12;
    int64_t parts = std::max<int64_t>(1, target / std::max<int64_t>(1, n_blocks_2d));
    int64_t len = (L + parts - 1) / parts;
    len = std::max<int64_t>(kTT * 2, (len + kTT - 1) / kTT * kTT);
    return (int)std::min<int64_t>(len, std::max<int64_t>((L + kTT - 1) / kTT * kTT, kTT));
}

// Unit layout of the sweep forward and the bitmap backward (shared, so that
// the backward can read the forward's per-unit start indices): warp units of
// 32 features x part_len positions (whole 32-position words), about
// kSweepUnitsPerSM per SM, more only when the batch rows alone exceed that.
static SweepLayout sweep_layout(int64_t B, int64_t D, int64_t L) {
    SweepLayout s;
    s.n_dblk = (int)((D + 31) / 32);
    const int64_t cols = B * s.n_dblk;
    const int64_t target = (int64_t)sm_count() * kSweepUnitsPerSM;
    const int64_t parts = std::max<int64_t>(1, (target + cols - 1) / std::max<int64_t>(1, cols));
    int64_t len = (L + parts - 1) / parts;
    len = std::max<int64_t>(32, (len + 31) / 32 * 32);
    s.part_len = (int)len;
    s.n_parts = (int)((L + len - 1) / len);
    s.n_units = cols * s.n_parts;
    return s;
}

// The event bitmap from the extraction's threshold mask ([B*Dm, nw] words,
// base channel b*Dm + j): logical channel b*D + d (D = Dm*expand) holds the
// events of base feature j = d / expand, so its word w is mask word w of base
// channel b*Dm + j.  A 32 x 32 tile per CTA through shared memory: the reads
// run along w, the writes along d; every bitmap word is written.
__global__ void __launch_bounds__(256)
mask_bitmap_kernel(const uint32_t* __restrict__ mask, int Dm, int expand, int nw, int n_jblk, int n_wblk,
                   uint32_t* __restrict__ bm) {
    __shared__ uint32_t tile[32][33];
    const int64_t blk = blockIdx.x;
    const int wb = (int)(blk % n_wblk);
    const int64_t rest = blk / n_wblk;
    const int jb = (int)(rest % n_jblk);
    const int64_t b = rest / n_jblk;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int r = ty; r < 32; r += 8) {
        const int j = jb * 32 + r, w = wb * 32 + tx;
        tile[r][tx] = (j < Dm && w < nw) ? mask[(b * Dm + j) * (int64_t)nw + w] : 0u;
    }
    __syncthreads();
    const int64_t D = (int64_t)Dm * expand;
    const int n_j = min(32, Dm - jb * 32);
    for (int r = ty; r < 32; r += 8) {
        const int w = wb * 32 + r;
        if (w >= nw) continue;
        uint32_t* row = bm + (b * nw + w) * D + (int64_t)jb * 32 * expand;
        for (int i = tx; i < n_j * expand; i += 32) row[i] = tile[i / expand][r];
    }
}

static size_t bitmap_words_bytes(int64_t n_channels, int64_t seqlen) {
    return (size_t)n_channels * (size_t)((seqlen + 31) / 32) * sizeof(uint32_t);
}

static bcm_status restore_fwd_impl(const void* y_flat, bcm_dtype y_dtype, const int32_t* time_steps,
                                   const int32_t* cu_seqlens, int64_t n_events, int64_t n_channels,
                                   int64_t dim, int64_t seqlen, void* out, bcm_dtype out_dtype,
                                   uint32_t* bitmap, const uint32_t* base_mask, int64_t expand,
                                   cudaStream_t stream) {
    BCM_REQUIRE(dtype_ok(y_dtype) && dtype_ok(out_dtype), "restore_dense_fwd: unsupported dtype");
    BCM_REQUIRE(y_dtype == BCM_F32 || y_dtype == out_dtype,
                "restore_dense_fwd: 16-bit input only supports the same output dtype");
    BCM_REQUIRE(dim >= 1 && seqlen >= 1 && n_channels >= 1 && n_events >= 0,
                "restore_dense_fwd: bad sizes");
    BCM_REQUIRE(n_channels % dim == 0, "restore_dense_fwd: n_channels must be divisible by dim");
    BCM_REQUIRE(seqlen < (1ll << 31) - 2 * kTT, "restore_dense_fwd: seqlen too large");
    BCM_REQUIRE(out && cu_seqlens && (n_events == 0 || (y_flat && time_steps)),
                "restore_dense_fwd: null pointer");
    const int64_t B = n_channels / dim;
    const SweepLayout lay = sweep_layout(B, dim, seqlen);
    BCM_REQUIRE((lay.n_units + kFU - 1) / kFU < (1ll << 31), "restore_dense_fwd: too many units");
    const int nw = (int)((seqlen + 31) / 32);
    // the per-unit start indices follow the bitmap words
    int32_t* e_start = bitmap ? reinterpret_cast<int32_t*>(reinterpret_cast<char*>(bitmap) +
                                                           bitmap_words_bytes(n_channels, seqlen))
                              : nullptr;
    if (bitmap != nullptr && n_events > 0 && base_mask != nullptr) {
        // the bitmap transposed from the extraction's mask (every word written)
        const int Dm = (int)(dim / expand);
        const int n_jblk = (Dm + 31) / 32, n_wblk = (nw + 31) / 32;
        const int64_t grid = B * n_jblk * n_wblk;
        BCM_REQUIRE(grid < (1ll << 31), "restore_dense_fwd_mask: too many tiles");
        mask_bitmap_kernel<<<(unsigned)grid, 256, 0, stream>>>(base_mask, Dm, (int)expand, nw, n_jblk, n_wblk,
                                                               bitmap);
        BCM_LAUNCH_CHECK();
    } else if (bitmap != nullptr && n_events > 0) {
        // the bitmap first (every word written: zeros, then the words holding
        // events), then the word sweep reads it instead of the event times
        BCM_CUDA_TRY(cudaMemsetAsync(bitmap, 0, bitmap_words_bytes(n_channels, seqlen), stream));
        event_bitmap_kernel<<<(unsigned)((n_channels + 7) / 8), 256, 0, stream>>>(
            time_steps, cu_seqlens, n_channels, (int)dim, (int)seqlen, nw, bitmap);
        BCM_LAUNCH_CHECK();
    }
    auto launch = [&](auto tin, auto tout) -> bcm_status {
        using Tin = decltype(tin);
        using Tout = decltype(tout);
        if (bitmap != nullptr && n_events > 0) {
            static_assert(kWU == kFU, "the word sweep runs the sweep layout's units");
            restore_fwd_words<Tin, Tout><<<(unsigned)((lay.n_units + kWU - 1) / kWU), kWU * 32, 0, stream>>>(
                static_cast<const Tin*>(y_flat), time_steps, cu_seqlens, bitmap, (int)dim, (int)seqlen, nw,
                lay.part_len, lay.n_dblk, lay.n_parts, lay.n_units, static_cast<Tout*>(out), e_start);
        } else {
            restore_fwd_sweep<Tin, Tout><<<(unsigned)((lay.n_units + kFU - 1) / kFU), kFU * 32, 0, stream>>>(
                static_cast<const Tin*>(y_flat), time_steps, cu_seqlens, (int)dim, (int)seqlen, nw, lay.part_len,
                lay.n_dblk, lay.n_parts, lay.n_units, static_cast<Tout*>(out), bitmap, e_start);
        }
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    };
    if (y_dtype == BCM_F32) {
        if (out_dtype == BCM_F32) return launch(float{}, float{});
        if (out_dtype == BCM_F16) return launch(float{}, __half{});
        return launch(float{}, __nv_bfloat16{});
    }
    if (y_dtype == BCM_F16) return launch(__half{}, __half{});
    return launch(__nv_bfloat16{}, __nv_bfloat16{});
}

extern "C" bcm_status bcm_restore_dense_fwd(const void* y_flat, bcm_dtype y_dtype,
                                            const int32_t* time_steps, const int32_t* cu_seqlens,
                                            int64_t n_events, int64_t n_channels, int64_t dim,
                                            int64_t seqlen, void* out, bcm_dtype out_dtype,
                                            cudaStream_t stream) {
    clear_error();
    return restore_fwd_impl(y_flat, y_dtype, time_steps, cu_seqlens, n_events, n_channels, dim, seqlen,
                            out, out_dtype, nullptr, nullptr, 1, stream);
}

extern "C" bcm_status bcm_restore_dense_fwd_bitmap(const void* y_flat, bcm_dtype y_dtype,
                                                   const int32_t* time_steps, const int32_t* cu_seqlens,
                                                   int64_t n_events, int64_t n_channels, int64_t dim,
                                                   int64_t seqlen, void* out, bcm_dtype out_dtype,
                                                   uint32_t* event_bitmap, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(event_bitmap, "restore_dense_fwd_bitmap: null event_bitmap");
    return restore_fwd_impl(y_flat, y_dtype, time_steps, cu_seqlens, n_events, n_channels, dim, seqlen,
                            out, out_dtype, event_bitmap, nullptr, 1, stream);
}

extern "C" bcm_status bcm_restore_dense_fwd_mask(const void* y_flat, bcm_dtype y_dtype,
                                                 const int32_t* time_steps, const int32_t* cu_seqlens,
                                                 int64_t n_events, int64_t n_channels, int64_t dim,
                                                 int64_t seqlen, void* out, bcm_dtype out_dtype,
                                                 const uint32_t* base_mask, int64_t expand,
                                                 uint32_t* event_bitmap, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(event_bitmap && base_mask, "restore_dense_fwd_mask: null event_bitmap or base_mask");
    BCM_REQUIRE(expand >= 1 && dim % expand == 0, "restore_dense_fwd_mask: dim must be a multiple of expand");
    // the bitmap built from events marks at most kCap events per channel;
    // the mask holds them all, so the two agree only while no channel can
    // have more
    BCM_REQUIRE(seqlen <= kCap, "restore_dense_fwd_mask: seqlen above %d (use the event bitmap)", kCap);
    return restore_fwd_impl(y_flat, y_dtype, time_steps, cu_seqlens, n_events, n_channels, dim, seqlen,
                            out, out_dtype, event_bitmap, base_mask, expand, stream);
}

extern "C" size_t bcm_restore_bitmap_bytes(int64_t n_channels, int64_t dim, int64_t seqlen) {
    if (n_channels < 0 || dim < 1 || seqlen < 1 || n_channels % dim != 0) return 0;
    const SweepLayout lay = sweep_layout(n_channels / dim, dim, seqlen);
    return bitmap_words_bytes(n_channels, seqlen) + (size_t)lay.n_units * 32 * sizeof(int32_t);
}

extern "C" size_t bcm_restore_workspace_bytes(int64_t n_channels, int64_t seqlen) {
    if (n_channels < 0 || seqlen < 0) return 0;
    return align_up(bitmap_words_bytes(n_channels, seqlen), 256);
}


static bcm_status launch_bwd_bitmap(const void* dout, bcm_dtype dtype, const int32_t* cu_seqlens, int64_t B,
                                    int64_t dim, int64_t seqlen, const uint32_t* bm, const int32_t* e_start,
                                    float* dy, cudaStream_t stream) {
    const SweepLayout lay = sweep_layout(B, dim, seqlen);
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        restore_bwd_bitmap<T><<<(unsigned)((lay.n_units + kBU - 1) / kBU), kBU * 32, 0, stream>>>(
            static_cast<const T*>(dout), cu_seqlens, bm, e_start, (int)dim, (int)seqlen,
            (int)((seqlen + 31) / 32), lay.part_len, lay.n_dblk, lay.n_parts, lay.n_units, dy);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}

extern "C" bcm_status bcm_restore_dense_bwd_bitmap(const void* dout, bcm_dtype dtype,
                                                   const int32_t* time_steps, const int32_t* cu_seqlens,
                                                   int64_t n_events, int64_t n_channels, int64_t dim,
                                                   int64_t seqlen, const uint32_t* event_bitmap, float* dy,
                                                   cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "restore_dense_bwd_bitmap: unsupported dtype");
    BCM_REQUIRE(dim >= 1 && seqlen >= 1 && n_channels >= 0 && n_events >= 0,
                "restore_dense_bwd_bitmap: bad sizes");
    BCM_REQUIRE(n_channels % dim == 0, "restore_dense_bwd_bitmap: n_channels must be divisible by dim");
    BCM_REQUIRE(seqlen < (1ll << 31) - 2 * kTT, "restore_dense_bwd_bitmap: seqlen too large");
    if (n_events == 0 || n_channels == 0) return BCM_OK;
    BCM_REQUIRE(dout && time_steps && cu_seqlens && dy && event_bitmap, "restore_dense_bwd_bitmap: null pointer");
    const int32_t* e_start = reinterpret_cast<const int32_t*>(reinterpret_cast<const char*>(event_bitmap) +
                                                              bitmap_words_bytes(n_channels, seqlen));
    return launch_bwd_bitmap(dout, dtype, cu_seqlens, n_channels / dim, dim, seqlen, event_bitmap, e_start, dy,
                             stream);
}

extern "C" bcm_status bcm_restore_dense_bwd(const void* dout, bcm_dtype dtype,
                                            const int32_t* time_steps, const int32_t* cu_seqlens,
                                            int64_t n_events, int64_t n_channels, int64_t dim,
                                            int64_t seqlen, float* dy, void* workspace,
                                            size_t workspace_bytes, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "restore_dense_bwd: unsupported dtype");
    BCM_REQUIRE(dim >= 1 && seqlen >= 1 && n_channels >= 0 && n_events >= 0,
                "restore_dense_bwd: bad sizes");
    BCM_REQUIRE(n_channels % dim == 0, "restore_dense_bwd: n_channels must be divisible by dim");
    BCM_REQUIRE(seqlen < (1ll << 31) - 2 * kTT, "restore_dense_bwd: seqlen too large");
    if (n_events == 0 || n_channels == 0) return BCM_OK;
    BCM_REQUIRE(dout && time_steps && cu_seqlens && dy, "restore_dense_bwd: null pointer");
    const int64_t B = n_channels / dim;
    BCM_REQUIRE(B < 65536, "restore_dense_bwd: batch too large");
    const int n_dblk = ceil_div(dim, kDB);
    const int part_len = restore_part_len(B * n_dblk, seqlen);
    const int n_parts = ceil_div(seqlen, part_len);
    dim3 grid(n_dblk * n_parts, (unsigned)B);
    const bool use_bitmap = workspace && workspace_bytes >= bcm_restore_workspace_bytes(n_channels, seqlen);
    if (use_bitmap) {
        const int nw = (int)((seqlen + 31) / 32);
        BCM_CUDA_TRY(cudaMemsetAsync(workspace, 0, (size_t)n_channels * nw * sizeof(uint32_t), stream));
        event_bitmap_kernel<<<(unsigned)((n_channels + 7) / 8), 256, 0, stream>>>(
            time_steps, cu_seqlens, n_channels, (int)dim, (int)seqlen, nw, static_cast<uint32_t*>(workspace));
        BCM_LAUNCH_CHECK();
    }
    if (use_bitmap)
        return launch_bwd_bitmap(dout, dtype, cu_seqlens, B, dim, seqlen,
                                 static_cast<const uint32_t*>(workspace), nullptr, dy, stream);
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        restore_bwd_kernel<T><<<grid, kWarpsR * 32, 0, stream>>>(
            static_cast<const T*>(dout), time_steps, cu_seqlens, (int)dim, (int)seqlen, part_len,
            n_dblk, dy);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}
