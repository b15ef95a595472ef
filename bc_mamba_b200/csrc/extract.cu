// extract.cu — threshold → event-stream extraction, replica expansion and the
// event gather / scatter.  Semantics follow the reference extension
// csrc/extract/extract_events_cuda.cu (count_base_kernel :192-208,
// fill_base_kernel :226-312, build_logical_cu_kernel :449-467,
// expand_events_direct_kernel :482-509, gather/scatter :629-662); the design
// is our own:
//   pass 1  one warp per base channel reads the row once (coalesced 128 B
//           loads, 32 in flight per lane), ballots 32 positions at a time and
//           writes a 1-bit-per-position mask plus the channel count;
//   pass 2  one CTA scans the counts into cu_seqlens and the max;
//   pass 3  one warp per channel turns mask words into (ch, t, k): a warp
//           prefix sum places each word's events in a shared-memory list that
//           is then written out with coalesced stores.
// The row is read once (the reference reads it twice) and the fill pass reads
// L/8 bytes of mask instead of the L*sizeof(T) input row.
#include <mutex>

#include "common.cuh"

namespace bcm {
namespace {

constexpr int kCountWarps = 4;   // warps per CTA in the count pass
constexpr int kFillWarps = 4;

// ---- pass 1: threshold + bitmask + count ---------------------------------
template <typename T>
__global__ void __launch_bounds__(kCountWarps * 32)
threshold_mask_kernel(const T* __restrict__ x, int64_t n_rows, int L, int n_words,
                      float thr, uint32_t* __restrict__ mask,
                      int32_t* __restrict__ counts) {
    const int lane = lane_id();
    const int64_t row = (int64_t)blockIdx.x * kCountWarps + (threadIdx.x >> 5);
    if (row >= n_rows) return;
    const T* xr = x + row * (int64_t)L;
    uint32_t* mr = mask + row * (int64_t)n_words;
    int cnt = 0;
    for (int w0 = 0; w0 < n_words; w0 += 32) {
        // 32 words = 1024 positions per iteration; lane j keeps word w0 + j.
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int t = (w0 + j) * 32 + lane;
            v[j] = (t < L) ? to_f32<T>(xr[t]) : -INFINITY;
        }
        uint32_t mine = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            // NaN > thr is false, like the reference's float compare.
            const uint32_t b = __ballot_sync(kFull, v[j] > thr);
            if (lane == j) mine = b;
        }
        if (w0 + lane < n_words) {
            mr[w0 + lane] = mine;
            cnt += __popc(mine);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cnt += __shfl_xor_sync(kFull, cnt, off);
    if (lane == 0) counts[row] = cnt;
}

// ---- pass 1, (B, L, d_model) input ----------------------------------------
// The same mask and counts from the layout the model holds its spikes in
// (rows of d_model features per position), so callers need no transposed
// copy.  A warp owns one batch row b, 32 consecutive features (lane =
// channel) and kBldWords mask words (32 positions each): per word it issues
// the 32 row loads (each a coalesced row of 32 features) and packs the lane's
// 32 comparisons into the channel's word.  Counts are per-warp partial sums
// added with integer atomics (exact and order-independent).
constexpr int kBldWords = 2;

template <typename T>
__global__ void __launch_bounds__(kCountWarps * 32)
threshold_mask_bld_kernel(const T* __restrict__ x, int L, int Dm, int n_words, int n_dblk, int n_wparts,
                          int64_t n_units, float thr, const float* __restrict__ thr_feature,
                          uint32_t* __restrict__ mask, int32_t* __restrict__ counts) {
    const int64_t unit = (int64_t)blockIdx.x * kCountWarps + (threadIdx.x >> 5);
    if (unit >= n_units) return;
    const int lane = lane_id();
    const int wpart = (int)(unit % n_wparts);
    const int64_t rest = unit / n_wparts;
    const int dblk = (int)(rest % n_dblk);
    const int64_t b = rest / n_dblk;
    const int d = dblk * 32 + lane;
    const bool valid = d < Dm;
    // one threshold for every feature, or feature d's own
    const float th = (thr_feature != nullptr && valid) ? thr_feature[d] : thr;
    const T* col = x + b * L * (int64_t)Dm + d;
    uint32_t* mrow = mask + (b * Dm + d) * (int64_t)n_words;
    const int w_beg = wpart * kBldWords;
    const int w_end = min(n_words, w_beg + kBldWords);
    int cnt = 0;
    for (int w = w_beg; w < w_end; ++w) {
        float v[32];
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const int t = w * 32 + r;
            v[r] = (valid && t < L) ? to_f32<T>(col[(int64_t)t * Dm]) : -INFINITY;
        }
        uint32_t word = 0u;
#pragma unroll
        for (int r = 0; r < 32; ++r) word |= (v[r] > th ? 1u : 0u) << r;   // NaN > th is false
        if (valid) {
            mrow[w] = word;
            cnt += __popc(word);
        }
    }
    if (valid && cnt > 0) atomicAdd(&counts[b * Dm + d], cnt);
}

// ---- pass 2: exclusive scan of counts into cu_seqlens + max ----------------
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads)
counts_scan_kernel(const int32_t* __restrict__ counts, int64_t n,
                   int32_t* __restrict__ cu, int32_t* __restrict__ max_out,
                   int32_t* __restrict__ summary) {   // {total, max}: one copy to the host
    __shared__ int s_warp_sum[32];
    __shared__ int s_warp_max[32];
    const int tid = threadIdx.x;
    const int64_t per = (n + kScanThreads - 1) / kScanThreads;
    const int64_t beg = min((int64_t)tid * per, n);
    const int64_t end = min(beg + per, n);
    int local = 0, lmax = 0;
    for (int64_t i = beg; i < end; ++i) {
        const int c = counts[i];
        local += c;
        lmax = max(lmax, c);
    }
    // block exclusive scan of `local`
    int incl = warp_inclusive_sum(local);
    int wmax = lmax;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) wmax = max(wmax, __shfl_xor_sync(kFull, wmax, off));
    const int warp = tid >> 5, lane = tid & 31;
    if (lane == 31) s_warp_sum[warp] = incl;
    if (lane == 0) s_warp_max[warp] = wmax;
    __syncthreads();
    if (warp == 0) {
        int s = s_warp_sum[lane];
        int m = s_warp_max[lane];
        int si = warp_inclusive_sum(s);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(kFull, m, off));
        s_warp_sum[lane] = si - s;  // exclusive
        if (lane == 0) {
            *max_out = m;
            summary[1] = m;
        }
    }
    __syncthreads();
    int run = s_warp_sum[warp] + incl - local;  // exclusive prefix for this thread
    if (tid == 0) cu[0] = 0;
    for (int64_t i = beg; i < end; ++i) {
        run += counts[i];
        cu[i + 1] = run;
    }
    if (tid == kScanThreads - 1) summary[0] = run;   // the last range ends at n: the total
}

// ---- pass 3: mask words → (ch, t, k) ---------------------------------------
// One warp per channel, 1024 positions (32 words) per step: each lane expands
// its word's set bits into a shared-memory list at its warp-prefix offset,
// then the warp writes (ch, t, k) for the whole list with coalesced stores;
// k = t - t_prev reads the neighbouring list entry (first of the channel:
// t + 1, reference fill_base_kernel :294-299).
__global__ void __launch_bounds__(kFillWarps * 32)
mask_fill_kernel(const uint32_t* __restrict__ mask, const int32_t* __restrict__ cu,
                 int64_t n_rows, int L, int n_words,
                 int32_t* __restrict__ ch_ids, int32_t* __restrict__ t_steps,
                 int32_t* __restrict__ k_flat) {
    __shared__ int s_t[kFillWarps][1024 + 1];
    const int lane = lane_id();
    const int w_in = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * kFillWarps + w_in;
    if (row >= n_rows) return;
    int* st = s_t[w_in] + 1;             // st[-1] holds the previous block's last t
    const uint32_t* mr = mask + row * (int64_t)n_words;
    int pos = cu[row];
    if (lane == 0) st[-1] = -1;
    for (int w0 = 0; w0 < n_words; w0 += 32) {
        const int w = w0 + lane;
        const uint32_t word = (w < n_words) ? mr[w] : 0u;
        const int c = __popc(word);
        const int incl = warp_inclusive_sum(c);
        const int total = __shfl_sync(kFull, incl, 31);
        int o = incl - c;
        uint32_t bits = word;
        while (bits) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            st[o++] = w * 32 + b;
        }
        __syncwarp();
        for (int i = lane; i < total; i += 32) {
            const int t = st[i];
            const int prev = st[i - 1];
            ch_ids[pos + i] = (int32_t)row;
            t_steps[pos + i] = t;
            k_flat[pos + i] = (prev < 0) ? (t + 1) : (t - prev);
        }
        __syncwarp();
        if (lane == 0 && total > 0) st[-1] = st[total - 1];
        __syncwarp();
        pos += total;
    }
}

// Pass 3 writing the expanded stream directly (extraction followed by
// expansion, without the base arrays): base channel c's events are written
// `expand` times, copy r at s*expand + r*cnt + i as channel c*expand + r (the
// layout expand_events_kernel produces), and the warp also writes the
// expanded cu_seqlens entries of its channel.  With x (B, D, L) given it also
// gathers x at every expanded event (x_flat[o] = x[channel][t], what
// gather_kernel computes from the finished stream).
constexpr int kXB = 4;   // events per lane whose x loads are issued together
constexpr int kXE = 2;   // copies (expand) covered by those loads (more load in the tail)

template <typename T>
__global__ void __launch_bounds__(kFillWarps * 32, 6)
mask_fill_expand_kernel(const uint32_t* __restrict__ mask, const int32_t* __restrict__ base_cu,
                        int64_t n_rows, int n_words, int expand,
                        int32_t* __restrict__ ch_ids, int32_t* __restrict__ t_steps,
                        int32_t* __restrict__ k_flat, int32_t* __restrict__ cu,
                        const T* __restrict__ x, int L, T* __restrict__ x_flat, int64_t cap) {
    __shared__ int s_t[kFillWarps][1024 + 1];
    const int lane = lane_id();
    const int w_in = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * kFillWarps + w_in;
    if (row >= n_rows) return;
    int* st = s_t[w_in] + 1;             // st[-1] holds the previous block's last t
    const uint32_t* mr = mask + row * (int64_t)n_words;
    const int s = base_cu[row];
    const int cnt = base_cu[row + 1] - s;
    const int64_t out0 = (int64_t)s * expand;
    for (int r = lane; r < expand; r += 32) cu[row * expand + r] = (int32_t)(out0 + (int64_t)r * cnt);
    if (row == n_rows - 1 && lane == 0) cu[n_rows * expand] = (int32_t)((int64_t)base_cu[n_rows] * expand);
    int local = 0;
    if (lane == 0) st[-1] = -1;
    for (int w0 = 0; w0 < n_words; w0 += 32) {
        const int w = w0 + lane;
        const uint32_t word = (w < n_words) ? mr[w] : 0u;
        const int c = __popc(word);
        const int incl = warp_inclusive_sum(c);
        const int total = __shfl_sync(kFull, incl, 31);
        int o = incl - c;
        uint32_t bits = word;
        while (bits) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            st[o++] = w * 32 + b;
        }
        __syncwarp();
        // kXB events per lane at a time: their x loads (copies r < kXE) are
        // all issued before any store, so the latencies overlap
        for (int i0 = 0; i0 < total; i0 += 32 * kXB) {
            int tv[kXB], kv[kXB];
            T xv[kXB][kXE];
#pragma unroll
            for (int u = 0; u < kXB; ++u) {
                const int i = i0 + u * 32 + lane;
                const bool in = i < total;
                const int t = in ? st[i] : 0;
                const int prev = in ? st[i - 1] : 0;
                tv[u] = t;
                kv[u] = (prev < 0) ? (t + 1) : (t - prev);
#pragma unroll
                for (int r = 0; r < kXE; ++r)
                    xv[u][r] = (x != nullptr && in && r < expand) ? x[(row * expand + r) * L + t] : T{};
            }
#pragma unroll
            for (int u = 0; u < kXB; ++u) {
                const int i = i0 + u * 32 + lane;
                if (i >= total) continue;
                auto put = [&](int r, T xr) {
                    const int64_t o2 = out0 + (int64_t)r * cnt + local + i;
                    if (o2 >= cap) return;   // outputs sized below the total: the caller fills again
                    ch_ids[o2] = (int32_t)(row * expand + r);
                    t_steps[o2] = tv[u];
                    k_flat[o2] = kv[u];
                    if (x != nullptr) x_flat[o2] = xr;
                };
#pragma unroll
                for (int r = 0; r < kXE; ++r)
                    if (r < expand) put(r, xv[u][r]);
                for (int r = kXE; r < expand; ++r)   // copies past kXE load here
                    put(r, x != nullptr ? x[(row * expand + r) * L + tv[u]] : T{});
            }
        }
        __syncwarp();
        if (lane == 0 && total > 0) st[-1] = st[total - 1];
        __syncwarp();
        local += total;
    }
}

// ---- expansion ---------------------------------------------------------------
__global__ void build_logical_cu_kernel(const int32_t* __restrict__ base_cu, int64_t n_base,
                                        int expand, int32_t* __restrict__ cu,
                                        int32_t* __restrict__ max_out) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int cnt = 0;
    if (c < n_base) {
        const int s = base_cu[c];
        cnt = base_cu[c + 1] - s;
        for (int r = 0; r < expand; ++r) cu[c * expand + r] = s * expand + r * cnt;
    } else if (c == n_base) {
        cu[n_base * expand] = base_cu[n_base] * expand;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cnt = max(cnt, __shfl_xor_sync(kFull, cnt, off));
    if (lane_id() == 0 && cnt > 0) atomicMax(max_out, cnt);
}

__global__ void expand_events_kernel(const int32_t* __restrict__ bch, const int32_t* __restrict__ bt,
                                     const int32_t* __restrict__ bk, const int32_t* __restrict__ base_cu,
                                     int64_t n_base_events, int64_t n_base, int expand,
                                     int32_t* __restrict__ ch, int32_t* __restrict__ t,
                                     int32_t* __restrict__ k) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_base_events; i += stride) {
        const int c = bch[i];
        if (c < 0 || c >= n_base) continue;  // malformed stream: skip, never fault
        const int tv = bt[i], kv = bk[i];
        const int s = base_cu[c];
        const int cnt = base_cu[c + 1] - s;
        const int64_t local = i - s;
        if (local < 0 || local >= cnt) continue;  // stream inconsistent with cu_seqlens
        for (int r = 0; r < expand; ++r) {
            const int64_t o = (int64_t)s * expand + (int64_t)r * cnt + local;
            ch[o] = c * expand + r;
            t[o] = tv;
            k[o] = kv;
        }
    }
}

// ---- gather / scatter -----------------------------------------------------
template <typename T>
__global__ void gather_kernel(const T* __restrict__ x, int64_t n_ch, int L,
                              const int32_t* __restrict__ ch, const int32_t* __restrict__ ts,
                              int64_t n_events, T* __restrict__ out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_events; e += stride) {
        const int c = ch[e], t = ts[e];
        T v = from_f32<T>(0.f);
        if (c >= 0 && c < n_ch && t >= 0 && t < L) v = x[(int64_t)c * L + t];
        out[e] = v;
    }
}

// ---- gather backward --------------------------------------------------------
// Pass A: row boundaries of a channel-sorted stream (row_start[r] = first event
// of row r, row_start[NC] = E) and an order check: channel_ids must be
// non-decreasing and inside [0, NC); otherwise *flag = 1.
__global__ void row_bounds_kernel(const int32_t* __restrict__ ch, int64_t n_events, int64_t n_ch,
                                  int32_t* __restrict__ row_start, int32_t* __restrict__ flag) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e <= n_events; e += stride) {
        const int64_t c = (e < n_events) ? (int64_t)ch[e] : n_ch;
        const int64_t prev = (e > 0) ? (int64_t)ch[e - 1] : -1;
        if ((e < n_events && (c < 0 || c >= n_ch)) || c < prev || prev >= n_ch) {
            *flag = 1;
            continue;
        }
        for (int64_t r = prev + 1; r <= c; ++r) row_start[r] = (int32_t)e;
    }
}

// Pass B: one warp per row.  The row's events are loaded first (coalesced,
// up to kRowPre*32 at a time, all loads independent), the row is zeroed with
// 16-byte stores while they are in flight, and the events are then written
// into it (same warp, ordered after the zeros by __syncwarp; L2 merges the
// writes, so the row reaches DRAM once).  A row whose times are not strictly
// increasing inside [0, L) is rewritten by its own warp: zeros, then its
// events in stream order (flag_out, when given, is raised as well).
constexpr int kRowWarps = 8;
constexpr int kRowPre = 16;

template <typename T, bool VEC>
__global__ void __launch_bounds__(kRowWarps * 32)
dense_rows_direct_kernel(const T* __restrict__ g, const int32_t* __restrict__ ts,
                         const int32_t* __restrict__ row_start, const int32_t* __restrict__ flag_in,
                         int64_t n_ch, int L, T* __restrict__ dx, int32_t* __restrict__ flag_out) {
    constexpr int V = 16 / sizeof(T);
    if (flag_in != nullptr && *flag_in) return;
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    if (r >= n_ch) return;
    T* row = dx + r * (int64_t)L;
    const int e_beg = row_start[r];
    const int e_end = row_start[r + 1];
    bool bad = false;
    int prev = -1;   // time of the last event of the previous 32 (order check)
    bool zeroed = false;
    for (int b0 = e_beg; b0 < e_end || !zeroed; b0 += kRowPre * 32) {
        int t[kRowPre];
        T v[kRowPre];
#pragma unroll
        for (int i = 0; i < kRowPre; ++i) {
            const int j = b0 + i * 32 + lane;
            const bool in = j < e_end;
            t[i] = in ? ts[j] : INT_MAX;
            v[i] = in ? g[j] : from_f32<T>(0.f);
        }
        if (!zeroed) {
            if (VEC) {
                for (int p = lane * V; p < L; p += 32 * V) *reinterpret_cast<uint4*>(row + p) = make_uint4(0, 0, 0, 0);
            } else {
                for (int p = lane; p < L; p += 32) row[p] = from_f32<T>(0.f);
            }
            zeroed = true;
            __syncwarp();
        }
#pragma unroll
        for (int i = 0; i < kRowPre; ++i) {
            const int j = b0 + i * 32 + lane;
            int tp = __shfl_up_sync(kFull, t[i], 1);
            if (lane == 0) tp = prev;
            prev = __shfl_sync(kFull, t[i], 31);
            if (j < e_end) {
                if (t[i] < 0 || t[i] >= L || t[i] <= tp) bad = true;
                else row[t[i]] = v[i];
            }
        }
    }
    if (__any_sync(kFull, bad)) {
        __syncwarp();
        for (int p = lane; p < L; p += 32) row[p] = from_f32<T>(0.f);
        __syncwarp();
        if (lane == 0) {
            for (int j = e_beg; j < e_end; ++j) {
                const int t = ts[j];
                if (t >= 0 && t < L) row[t] = g[j];
            }
            if (flag_out != nullptr) atomicExch(flag_out, 1);
        }
    }
}

// Fallback for any other event order (runs only when *flag is set):
// zero-fill, then scatter in stream order (reference
// extract_events_cuda.cu:649-662, 731).
template <typename T>
__global__ void fallback_zero_kernel(const int32_t* __restrict__ flag, T* __restrict__ dx, int64_t n) {
    if (!*flag) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        dx[i] = from_f32<T>(0.f);
}

template <typename T>
__global__ void fallback_scatter_kernel(const int32_t* __restrict__ flag, const T* __restrict__ g,
                                        const int32_t* __restrict__ ch, const int32_t* __restrict__ ts,
                                        int64_t n_events, int64_t n_ch, int L, T* __restrict__ dx) {
    if (!*flag) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_events; e += stride) {
        const int c = ch[e], t = ts[e];
        if (c >= 0 && c < n_ch && t >= 0 && t < L) dx[(int64_t)c * L + t] = g[e];
    }
}

// Pass B launch (16-byte row stores when L and dx allow).
template <typename T>
bcm_status launch_dense_rows(const T* g, const int32_t* ts, const int32_t* row_start, const int32_t* flag_in,
                             int64_t n_ch, int64_t L, T* dx, int32_t* flag_out, cudaStream_t stream) {
    constexpr int V = 16 / sizeof(T);
    const bool vec = (L % V == 0) && (reinterpret_cast<uintptr_t>(dx) % 16 == 0);
    const int64_t grid = (n_ch + kRowWarps - 1) / kRowWarps;
    BCM_REQUIRE(grid < (1ll << 31), "gather_events_bwd: too many rows");
    if (vec)
        dense_rows_direct_kernel<T, true><<<(unsigned)grid, kRowWarps * 32, 0, stream>>>(
            g, ts, row_start, flag_in, n_ch, (int)L, dx, flag_out);
    else
        dense_rows_direct_kernel<T, false><<<(unsigned)grid, kRowWarps * 32, 0, stream>>>(
            g, ts, row_start, flag_in, n_ch, (int)L, dx, flag_out);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

inline int grid_for(int64_t n, int threads) {
    const int64_t want = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 16;
    return (int)std::max<int64_t>(1, std::min(want, cap));
}

}  // namespace
}  // namespace bcm

using namespace bcm;

// counts -> cu_seqlens and max on the device, then the event total to the
// host (the one synchronisation the reference API implies: outputs are sized
// by it).
// Bytes of the extraction workspace taken by the event bit mask; the
// {total, max} summary of the count scan follows it.
static size_t mask_region_bytes(int64_t n_base_channels, int64_t seqlen) {
    const int64_t words = (seqlen + 31) / 32;
    return align_up((size_t)(n_base_channels * words * sizeof(uint32_t)), 256);
}

// A small pinned host buffer per host thread for the summary copy (a copy to
// pageable memory is staged by the driver); nullptr if pinning fails.
static int32_t* pinned_summary() {
    thread_local int32_t* buf = nullptr;
    thread_local bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        if (cudaHostAlloc(&p, 2 * sizeof(int32_t), cudaHostAllocPortable) == cudaSuccess)
            buf = static_cast<int32_t*>(p);
        else
            (void)cudaGetLastError();
    }
    return buf;
}

// A timing-free event per host thread and device marking the summary copy.
static cudaError_t summary_event(cudaEvent_t* out) {
    constexpr int kDev = 64;
    thread_local cudaEvent_t ev[kDev] = {};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kDev) return cudaErrorInvalidDevice;
    if (ev[dev] == nullptr) {
        err = cudaEventCreateWithFlags(&ev[dev], cudaEventDisableTiming);
        if (err != cudaSuccess) return err;
    }
    *out = ev[dev];
    return cudaSuccess;
}

// `before_sync` enqueues more work after the summary copy (work that needs
// cu_seqlens on the device but not the total on the host); the host then
// waits for the copy only, so the GPU keeps running that work meanwhile.
template <typename Hook>
static bcm_status scan_counts_and_sync(const int32_t* counts, int64_t n_base_channels, int32_t* cu_seqlens,
                                       int32_t* max_seqlen, void* workspace, int64_t seqlen,
                                       int64_t* n_events_host, int32_t* max_host, cudaStream_t stream,
                                       Hook&& before_sync) {
    int32_t* summary = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) +
                                                  mask_region_bytes(n_base_channels, seqlen));
    counts_scan_kernel<<<1, kScanThreads, 0, stream>>>(counts, n_base_channels, cu_seqlens, max_seqlen, summary);
    BCM_LAUNCH_CHECK();
    int32_t pageable[2] = {0, 0};
    int32_t* host = pinned_summary();
    if (host == nullptr) host = pageable;
    BCM_CUDA_TRY(cudaMemcpyAsync(host, summary, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
    cudaEvent_t copied = nullptr;
    BCM_CUDA_TRY(summary_event(&copied));
    BCM_CUDA_TRY(cudaEventRecord(copied, stream));
    const bcm_status hs = before_sync();
    if (hs != BCM_OK) return hs;
    BCM_CUDA_TRY(cudaEventSynchronize(copied));
    *n_events_host = host[0];
    if (max_host) *max_host = host[1];
    return BCM_OK;
}

extern "C" size_t bcm_extract_workspace_bytes(int64_t n_base_channels, int64_t seqlen) {
    if (n_base_channels < 0 || seqlen < 0) return 0;
    return mask_region_bytes(n_base_channels, seqlen) + 256;
}

template <typename Hook>
static bcm_status count_base_impl(const void* base_input, bcm_dtype dtype, int64_t n_base_channels,
                                  int64_t seqlen, float threshold, int32_t* counts, int32_t* cu_seqlens,
                                  int32_t* max_seqlen, void* workspace, size_t workspace_bytes,
                                  int64_t* n_events_host, int32_t* max_seqlen_host, cudaStream_t stream,
                                  Hook&& before_sync) {
    BCM_REQUIRE(dtype_ok64(dtype), "extract_base_events: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(n_base_channels >= 0 && seqlen >= 0, "extract_base_events: negative size");
    BCM_REQUIRE(seqlen < (1ll << 31) && n_base_channels * seqlen < (1ll << 31) * 64,
                "extract_base_events: sizes exceed int32 event indexing");
    BCM_REQUIRE(cu_seqlens && max_seqlen && n_events_host, "extract_base_events: null output");
    const size_t need = bcm_extract_workspace_bytes(n_base_channels, seqlen);
    if (workspace_bytes < need || (need > 0 && !workspace)) {
        set_error("extract_base_events: workspace of %zu bytes < required %zu",
                  workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    if (n_base_channels == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(max_seqlen, 0, sizeof(int32_t), stream));
        BCM_CUDA_TRY(cudaMemsetAsync(cu_seqlens, 0, sizeof(int32_t), stream));
        BCM_CUDA_TRY(cudaStreamSynchronize(stream));
        *n_events_host = 0;
        if (max_seqlen_host) *max_seqlen_host = 0;
        return BCM_OK;
    }
    BCM_REQUIRE(base_input && counts, "extract_base_events: null pointer");
    const int L = (int)seqlen;
    const int n_words = (L + 31) / 32;
    uint32_t* mask = static_cast<uint32_t*>(workspace);
    if (L == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * n_base_channels, stream));
    } else {
        const int grid = ceil_div(n_base_channels, kCountWarps);
        bcm_status st = dispatch_dtype64(dtype, [&](auto tag) -> bcm_status {
            using T = decltype(tag);
            threshold_mask_kernel<T><<<grid, kCountWarps * 32, 0, stream>>>(
                static_cast<const T*>(base_input), n_base_channels, L, n_words, threshold,
                mask, counts);
            BCM_LAUNCH_CHECK();
            return BCM_OK;
        });
        if (st != BCM_OK) return st;
    }
    return scan_counts_and_sync(counts, n_base_channels, cu_seqlens, max_seqlen, workspace, seqlen,
                                n_events_host, max_seqlen_host, stream, before_sync);
}

template <typename Hook>
static bcm_status count_bld_impl(const void* input_bld, bcm_dtype dtype, int64_t batch, int64_t seqlen,
                                 int64_t d_model, float threshold, const float* thr_feature,
                                 int32_t* counts, int32_t* cu_seqlens,
                                 int32_t* max_seqlen, void* workspace, size_t workspace_bytes,
                                 int64_t* n_events_host, int32_t* max_seqlen_host, cudaStream_t stream,
                                 Hook&& before_sync) {
    BCM_REQUIRE(dtype_ok64(dtype), "extract_base_events_bld: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(batch >= 0 && seqlen >= 0 && d_model >= 0, "extract_base_events_bld: negative size");
    const int64_t n_base_channels = batch * d_model;
    BCM_REQUIRE(seqlen < (1ll << 31) && n_base_channels * seqlen < (1ll << 31) * 64,
                "extract_base_events_bld: sizes exceed int32 event indexing");
    BCM_REQUIRE(cu_seqlens && max_seqlen && n_events_host, "extract_base_events_bld: null output");
    const size_t need = bcm_extract_workspace_bytes(n_base_channels, seqlen);
    if (workspace_bytes < need || (need > 0 && !workspace)) {
        set_error("extract_base_events_bld: workspace of %zu bytes < required %zu", workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    if (n_base_channels == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(max_seqlen, 0, sizeof(int32_t), stream));
        BCM_CUDA_TRY(cudaMemsetAsync(cu_seqlens, 0, sizeof(int32_t), stream));
        BCM_CUDA_TRY(cudaStreamSynchronize(stream));
        *n_events_host = 0;
        if (max_seqlen_host) *max_seqlen_host = 0;
        return BCM_OK;
    }
    BCM_REQUIRE(input_bld && counts, "extract_base_events_bld: null pointer");
    BCM_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * n_base_channels, stream));
    const int L = (int)seqlen;
    if (L > 0) {
        const int n_words = (L + 31) / 32;
        const int n_dblk = (int)((d_model + 31) / 32);
        const int n_wparts = (n_words + kBldWords - 1) / kBldWords;
        const int64_t n_units = batch * n_dblk * n_wparts;
        const int64_t grid = (n_units + kCountWarps - 1) / kCountWarps;
        BCM_REQUIRE(grid < (1ll << 31), "extract_base_events_bld: too many rows");
        bcm_status st = dispatch_dtype64(dtype, [&](auto tag) -> bcm_status {
            using T = decltype(tag);
            threshold_mask_bld_kernel<T><<<(unsigned)grid, kCountWarps * 32, 0, stream>>>(
                static_cast<const T*>(input_bld), L, (int)d_model, n_words, n_dblk, n_wparts, n_units, threshold,
                thr_feature, static_cast<uint32_t*>(workspace), counts);
            BCM_LAUNCH_CHECK();
            return BCM_OK;
        });
        if (st != BCM_OK) return st;
    }
    return scan_counts_and_sync(counts, n_base_channels, cu_seqlens, max_seqlen, workspace, seqlen,
                                n_events_host, max_seqlen_host, stream, before_sync);
}

static bcm_status no_hook() { return BCM_OK; }

extern "C" bcm_status bcm_extract_base_count(const void* base_input, bcm_dtype dtype,
                                             int64_t n_base_channels, int64_t seqlen,
                                             float threshold, int32_t* counts,
                                             int32_t* cu_seqlens, int32_t* max_seqlen,
                                             void* workspace, size_t workspace_bytes,
                                             int64_t* n_events_host, int32_t* max_seqlen_host,
                                             cudaStream_t stream) {
    clear_error();
    return count_base_impl(base_input, dtype, n_base_channels, seqlen, threshold, counts, cu_seqlens, max_seqlen,
                           workspace, workspace_bytes, n_events_host, max_seqlen_host, stream, no_hook);
}

extern "C" bcm_status bcm_extract_base_count_bld(const void* input_bld, bcm_dtype dtype, int64_t batch,
                                                 int64_t seqlen, int64_t d_model, float threshold,
                                                 int32_t* counts, int32_t* cu_seqlens, int32_t* max_seqlen,
                                                 void* workspace, size_t workspace_bytes,
                                                 int64_t* n_events_host, int32_t* max_seqlen_host,
                                                 cudaStream_t stream) {
    clear_error();
    return count_bld_impl(input_bld, dtype, batch, seqlen, d_model, threshold, nullptr, counts, cu_seqlens,
                          max_seqlen, workspace, workspace_bytes, n_events_host, max_seqlen_host, stream, no_hook);
}

extern "C" bcm_status bcm_extract_base_fill(int64_t n_base_channels, int64_t seqlen,
                                            const int32_t* cu_seqlens, const void* workspace,
                                            size_t workspace_bytes, int32_t* ch_ids,
                                            int32_t* t_steps, int32_t* k_flat,
                                            cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(n_base_channels >= 0 && seqlen >= 0, "extract_base_events: negative size");
    if (n_base_channels == 0 || seqlen == 0) return BCM_OK;
    const size_t need = bcm_extract_workspace_bytes(n_base_channels, seqlen);
    if (workspace_bytes < need || !workspace) {
        set_error("extract_base_events: workspace of %zu bytes < required %zu",
                  workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    BCM_REQUIRE(cu_seqlens && ch_ids && t_steps && k_flat, "extract_base_events: null pointer");
    const int L = (int)seqlen;
    const int n_words = (L + 31) / 32;
    const int grid = ceil_div(n_base_channels, kFillWarps);
    mask_fill_kernel<<<grid, kFillWarps * 32, 0, stream>>>(
        static_cast<const uint32_t*>(workspace), cu_seqlens, n_base_channels, L, n_words,
        ch_ids, t_steps, k_flat);
    BCM_LAUNCH_CHECK();
    return BCM_OK;
}

static bcm_status launch_expand_fill(int64_t n_base_channels, int64_t seqlen, const int32_t* base_cu,
                                     const void* workspace, int64_t expand, int32_t* ch_ids, int32_t* t_steps,
                                     int32_t* k_flat, int32_t* cu_seqlens, const void* x, bcm_dtype x_dtype,
                                     void* x_flat, int64_t cap, cudaStream_t stream) {
    const int L = (int)seqlen;
    const int n_words = (L + 31) / 32;
    const int grid = ceil_div(n_base_channels, kFillWarps);
    if (x == nullptr) {
        mask_fill_expand_kernel<float><<<grid, kFillWarps * 32, 0, stream>>>(
            static_cast<const uint32_t*>(workspace), base_cu, n_base_channels, n_words, (int)expand,
            ch_ids, t_steps, k_flat, cu_seqlens, nullptr, L, nullptr, cap);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    }
    BCM_REQUIRE(dtype_ok64(x_dtype), "extract_expand_fill: unsupported x dtype %d", (int)x_dtype);
    return dispatch_dtype64(x_dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        mask_fill_expand_kernel<T><<<grid, kFillWarps * 32, 0, stream>>>(
            static_cast<const uint32_t*>(workspace), base_cu, n_base_channels, n_words, (int)expand,
            ch_ids, t_steps, k_flat, cu_seqlens, static_cast<const T*>(x), L, static_cast<T*>(x_flat), cap);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}

extern "C" bcm_status bcm_extract_expand_fill(int64_t n_base_channels, int64_t seqlen,
                                              const int32_t* base_cu_seqlens, const void* workspace,
                                              size_t workspace_bytes, int64_t expand, int32_t* ch_ids,
                                              int32_t* t_steps, int32_t* k_flat, int32_t* cu_seqlens,
                                              const void* x, bcm_dtype x_dtype, void* x_flat,
                                              cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(n_base_channels >= 0 && seqlen >= 0, "extract_expand_fill: negative size");
    BCM_REQUIRE(expand >= 1 && n_base_channels * expand < (1ll << 31), "extract_expand_fill: bad expand");
    if (n_base_channels == 0) return BCM_OK;
    BCM_REQUIRE(base_cu_seqlens && cu_seqlens, "extract_expand_fill: null pointer");
    const size_t need = bcm_extract_workspace_bytes(n_base_channels, seqlen);
    if (workspace_bytes < need || !workspace) {
        set_error("extract_expand_fill: workspace of %zu bytes < required %zu", workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    BCM_REQUIRE(seqlen == 0 || (ch_ids && t_steps && k_flat), "extract_expand_fill: null pointer");
    BCM_REQUIRE((x == nullptr) == (x_flat == nullptr), "extract_expand_fill: x and x_flat go together");
    return launch_expand_fill(n_base_channels, seqlen, base_cu_seqlens, workspace, expand, ch_ids, t_steps, k_flat,
                              cu_seqlens, x, x_dtype, x_flat, INT64_MAX, stream);
}

static bcm_status extract_expanded_impl(const void* input, bcm_dtype dtype, int32_t input_layout, int64_t batch,
                                        int64_t d_model, int64_t seqlen, float threshold, const float* thr_feature,
                                        int64_t expand, int32_t* counts, int32_t* base_cu_seqlens,
                                        int32_t* max_seqlen, void* workspace, size_t workspace_bytes,
                                        int64_t capacity, int32_t* ch_ids, int32_t* t_steps, int32_t* k_flat,
                                        int32_t* cu_seqlens, const void* x, bcm_dtype x_dtype, void* x_flat,
                                        int64_t* n_events_host, int32_t* max_seqlen_host, cudaStream_t stream) {
    BCM_REQUIRE(input_layout == 0 || input_layout == 1, "extract_expanded: input_layout must be 0 or 1");
    BCM_REQUIRE(batch >= 0 && d_model >= 0 && seqlen >= 0 && capacity >= 0, "extract_expanded: negative size");
    BCM_REQUIRE(expand >= 1 && batch * d_model * expand < (1ll << 31), "extract_expanded: bad expand");
    BCM_REQUIRE(cu_seqlens && n_events_host, "extract_expanded: null output");
    BCM_REQUIRE((x == nullptr) == (x_flat == nullptr), "extract_expanded: x and x_flat go together");
    BCM_REQUIRE(capacity == 0 || (ch_ids && t_steps && k_flat), "extract_expanded: null stream outputs");
    const int64_t NCb = batch * d_model;
    if (NCb == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(cu_seqlens, 0, sizeof(int32_t), stream));
        if (max_seqlen) BCM_CUDA_TRY(cudaMemsetAsync(max_seqlen, 0, sizeof(int32_t), stream));
        BCM_CUDA_TRY(cudaStreamSynchronize(stream));
        *n_events_host = 0;
        if (max_seqlen_host) *max_seqlen_host = 0;
        return BCM_OK;
    }
    // the fill goes in before the host waits: it needs the offsets on the
    // device, not the total on the host
    auto fill = [&]() -> bcm_status {
        return launch_expand_fill(NCb, seqlen, base_cu_seqlens, workspace, expand, ch_ids, t_steps, k_flat,
                                  cu_seqlens, x, x_dtype, x_flat, capacity, stream);
    };
    if (input_layout == 0)
        return count_base_impl(input, dtype, NCb, seqlen, threshold, counts, base_cu_seqlens, max_seqlen, workspace,
                               workspace_bytes, n_events_host, max_seqlen_host, stream, fill);
    return count_bld_impl(input, dtype, batch, seqlen, d_model, threshold, thr_feature, counts, base_cu_seqlens,
                          max_seqlen, workspace, workspace_bytes, n_events_host, max_seqlen_host, stream, fill);
}

extern "C" bcm_status bcm_extract_expanded(const void* input, bcm_dtype dtype, int32_t input_layout,
                                           int64_t batch, int64_t d_model, int64_t seqlen, float threshold,
                                           int64_t expand, int32_t* counts, int32_t* base_cu_seqlens,
                                           int32_t* max_seqlen, void* workspace, size_t workspace_bytes,
                                           int64_t capacity, int32_t* ch_ids, int32_t* t_steps, int32_t* k_flat,
                                           int32_t* cu_seqlens, const void* x, bcm_dtype x_dtype, void* x_flat,
                                           int64_t* n_events_host, int32_t* max_seqlen_host,
                                           cudaStream_t stream) {
    clear_error();
    return extract_expanded_impl(input, dtype, input_layout, batch, d_model, seqlen, threshold, nullptr, expand,
                                 counts, base_cu_seqlens, max_seqlen, workspace, workspace_bytes, capacity, ch_ids,
                                 t_steps, k_flat, cu_seqlens, x, x_dtype, x_flat, n_events_host, max_seqlen_host,
                                 stream);
}

extern "C" bcm_status bcm_extract_expanded_ft(const void* input_bld, bcm_dtype dtype, int64_t batch,
                                              int64_t d_model, int64_t seqlen, const float* feature_thresholds,
                                              int64_t expand, int32_t* counts, int32_t* base_cu_seqlens,
                                              int32_t* max_seqlen, void* workspace, size_t workspace_bytes,
                                              int64_t capacity, int32_t* ch_ids, int32_t* t_steps,
                                              int32_t* k_flat, int32_t* cu_seqlens, const void* x,
                                              bcm_dtype x_dtype, void* x_flat, int64_t* n_events_host,
                                              int32_t* max_seqlen_host, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(feature_thresholds != nullptr, "extract_expanded_ft: null feature thresholds");
    return extract_expanded_impl(input_bld, dtype, 1, batch, d_model, seqlen, 0.f, feature_thresholds, expand,
                                 counts, base_cu_seqlens, max_seqlen, workspace, workspace_bytes, capacity, ch_ids,
                                 t_steps, k_flat, cu_seqlens, x, x_dtype, x_flat, n_events_host, max_seqlen_host,
                                 stream);
}

extern "C" bcm_status bcm_expand_base_events(const int32_t* base_ch_ids,
                                             const int32_t* base_t_steps,
                                             const int32_t* base_k_flat,
                                             const int32_t* base_cu_seqlens,
                                             int64_t n_base_events, int64_t n_base_channels,
                                             int64_t expand, int32_t* ch_ids,
                                             int32_t* t_steps, int32_t* k_flat,
                                             int32_t* cu_seqlens, int32_t* max_seqlen,
                                             cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(n_base_events >= 0 && n_base_channels >= 0, "expand_base_events: negative size");
    BCM_REQUIRE(expand >= 1, "expand_base_events: expand must be >= 1");
    BCM_REQUIRE(n_base_events * expand < (1ll << 31) && n_base_channels * expand < (1ll << 31),
                "expand_base_events: sizes exceed int32 indexing");
    BCM_REQUIRE(cu_seqlens && max_seqlen, "expand_base_events: null output");
    BCM_CUDA_TRY(cudaMemsetAsync(max_seqlen, 0, sizeof(int32_t), stream));
    if (n_base_events == 0) {
        // Reference returns zero cu_seqlens and a zero max when nothing fires.
        BCM_CUDA_TRY(cudaMemsetAsync(cu_seqlens, 0,
                                     sizeof(int32_t) * (n_base_channels * expand + 1), stream));
        return BCM_OK;
    }
    BCM_REQUIRE(base_ch_ids && base_t_steps && base_k_flat && base_cu_seqlens && ch_ids &&
                    t_steps && k_flat,
                "expand_base_events: null pointer");
    {
        const int threads = 256;
        const int grid = ceil_div(n_base_channels + 1, threads);
        build_logical_cu_kernel<<<grid, threads, 0, stream>>>(base_cu_seqlens, n_base_channels,
                                                              (int)expand, cu_seqlens, max_seqlen);
        BCM_LAUNCH_CHECK();
    }
    {
        const int threads = 256;
        expand_events_kernel<<<grid_for(n_base_events, threads), threads, 0, stream>>>(
            base_ch_ids, base_t_steps, base_k_flat, base_cu_seqlens, n_base_events,
            n_base_channels, (int)expand, ch_ids, t_steps, k_flat);
        BCM_LAUNCH_CHECK();
    }
    return BCM_OK;
}

extern "C" bcm_status bcm_gather_events_fwd(const void* x, bcm_dtype dtype, int64_t n_channels,
                                            int64_t seqlen, const int32_t* channel_ids,
                                            const int32_t* time_steps, int64_t n_events,
                                            void* out, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok64(dtype), "gather_events_fwd: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(n_events >= 0 && n_channels >= 0 && seqlen >= 0, "gather_events_fwd: negative size");
    if (n_events == 0) return BCM_OK;
    BCM_REQUIRE(x && channel_ids && time_steps && out, "gather_events_fwd: null pointer");
    const int threads = 256;
    return dispatch_dtype64(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        gather_kernel<T><<<grid_for(n_events, threads), threads, 0, stream>>>(
            static_cast<const T*>(x), n_channels, (int)seqlen, channel_ids, time_steps, n_events,
            static_cast<T*>(out));
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}

extern "C" size_t bcm_gather_bwd_workspace_bytes(int64_t n_channels) {
    if (n_channels < 0) return 0;
    return align_up((size_t)(n_channels + 1 + 64) * sizeof(int32_t), 256);
}

extern "C" bcm_status bcm_gather_events_bwd(const void* grad, bcm_dtype dtype,
                                            const int32_t* channel_ids,
                                            const int32_t* time_steps, int64_t n_events,
                                            int64_t n_channels, int64_t seqlen, void* dx,
                                            void* workspace, size_t workspace_bytes,
                                            cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok64(dtype), "gather_events_bwd: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(n_events >= 0 && n_channels >= 0 && seqlen >= 0, "gather_events_bwd: negative size");
    BCM_REQUIRE(n_events < (1ll << 31) && seqlen < (1ll << 31), "gather_events_bwd: sizes exceed int32");
    const size_t bytes = (size_t)n_channels * (size_t)seqlen * dtype_size(dtype);
    if (bytes == 0) return BCM_OK;
    BCM_REQUIRE(dx, "gather_events_bwd: null dx");
    if (n_events == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(dx, 0, bytes, stream));
        return BCM_OK;
    }
    BCM_REQUIRE(grad && channel_ids && time_steps, "gather_events_bwd: null pointer");
    const size_t need = bcm_gather_bwd_workspace_bytes(n_channels);
    if (!workspace || workspace_bytes < need) {
        set_error("gather_events_bwd: workspace of %zu bytes < required %zu", workspace_bytes, need);
        return BCM_ERR_WORKSPACE;
    }
    // workspace: [flag][pad to 256 B][row_start[NC + 1]]
    int32_t* flag = static_cast<int32_t*>(workspace);
    int32_t* row_start = flag + 64;
    BCM_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int32_t), stream));
    const int threads = 256;
    row_bounds_kernel<<<grid_for(n_events + 1, threads), threads, 0, stream>>>(
        channel_ids, n_events, n_channels, row_start, flag);
    BCM_LAUNCH_CHECK();
    return dispatch_dtype64(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        const bcm_status st = launch_dense_rows<T>(static_cast<const T*>(grad), time_steps, row_start, flag,
                                                   n_channels, seqlen, static_cast<T*>(dx), flag, stream);
        if (st != BCM_OK) return st;
        const int fb_grid = sm_count() * 2;
        fallback_zero_kernel<T><<<fb_grid, threads, 0, stream>>>(flag, static_cast<T*>(dx),
                                                                 (int64_t)n_channels * seqlen);
        BCM_LAUNCH_CHECK();
        fallback_scatter_kernel<T><<<fb_grid, threads, 0, stream>>>(
            flag, static_cast<const T*>(grad), channel_ids, time_steps, n_events, n_channels,
            (int)seqlen, static_cast<T*>(dx));
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}

extern "C" bcm_status bcm_gather_events_bwd_rows(const void* grad, bcm_dtype dtype,
                                                 const int32_t* time_steps, const int32_t* cu_seqlens,
                                                 int64_t n_events, int64_t n_channels, int64_t seqlen,
                                                 void* dx, void* workspace, size_t workspace_bytes,
                                                 cudaStream_t stream) {
    clear_error();
    (void)workspace;        // kept for the ABI; a row with unsorted times is fixed by its own warp
    (void)workspace_bytes;
    BCM_REQUIRE(dtype_ok64(dtype), "gather_events_bwd_rows: unsupported dtype %d", (int)dtype);
    BCM_REQUIRE(n_events >= 0 && n_channels >= 0 && seqlen >= 0, "gather_events_bwd_rows: negative size");
    BCM_REQUIRE(n_events < (1ll << 31) && seqlen < (1ll << 31), "gather_events_bwd_rows: sizes exceed int32");
    const size_t bytes = (size_t)n_channels * (size_t)seqlen * dtype_size(dtype);
    if (bytes == 0) return BCM_OK;
    BCM_REQUIRE(dx, "gather_events_bwd_rows: null dx");
    if (n_events == 0) {
        BCM_CUDA_TRY(cudaMemsetAsync(dx, 0, bytes, stream));
        return BCM_OK;
    }
    BCM_REQUIRE(grad && time_steps && cu_seqlens, "gather_events_bwd_rows: null pointer");
    return dispatch_dtype64(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        return launch_dense_rows<T>(static_cast<const T*>(grad), time_steps, cu_seqlens, nullptr, n_channels,
                                    seqlen, static_cast<T*>(dx), nullptr, stream);
    });
}

// ---- gather backward without allocation -------------------------------------
// Callers that may not allocate device memory (an FFI host whose device memory
// is carved from its own arena up front; code where cudaMalloc/cudaFree would
// stall or synchronise the GPU) get the same backward with its scratch in a
// fixed array: the order flag, 63 ints of padding and row_start[NC + 1], i.e.
// the layout bcm_gather_events_bwd expects of its workspace.  Every GPU that
// loads this library holds the array (about 1 MiB) until the process exits.
namespace bcm {
namespace {
constexpr int64_t kNoallocScratchInts =
    ((64 + BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS + 1) + 63) / 64 * 64;
static __device__ __align__(256) int32_t g_gather_bwd_scratch[kNoallocScratchInts];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  Host code may
// not use g_gather_bwd_scratch as a pointer (it names a host-side stand-in),
// so the address is looked up once per device and cached.  With lazy module
// loading the first lookup on a device loads this library's module there,
// which is when the array is allocated.  The cache lives as long as the
// process: after a cudaDeviceReset() the cached address is stale, so the
// library must not be used across a device reset.
bcm_status noalloc_scratch(void** out) {
    int dev = -1;
    BCM_CUDA_TRY(cudaGetDevice(&dev));
    BCM_REQUIRE(dev >= 0 && dev < kMaxDevices, "gather_events_bwd_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_gather_bwd_scratch);
        if (err != cudaSuccess || !p) {
            set_error("gather_events_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                      cudaGetErrorString(err));
            return BCM_ERR_CUDA;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return BCM_OK;
}
}  // namespace
}  // namespace bcm

extern "C" bcm_status bcm_gather_events_bwd_noalloc(const void* grad, bcm_dtype dtype,
                                                    const int32_t* channel_ids,
                                                    const int32_t* time_steps, int64_t n_events,
                                                    int64_t n_channels, int64_t seqlen, void* dx,
                                                    cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(n_channels <= BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS,
                "gather_events_bwd_noalloc: n_channels %lld exceeds the fixed scratch limit of %d "
                "channels; use bcm_gather_events_bwd with a workspace",
                (long long)n_channels, BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS);
    void* scratch = nullptr;
    const bcm_status st = noalloc_scratch(&scratch);
    if (st != BCM_OK) return st;
    // bcm_gather_events_bwd clears the flag word itself and rewrites every
    // row_start entry it reads, so nothing left from the previous call leaks.
    static_assert(sizeof(g_gather_bwd_scratch) >= 4 * (64 + BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS + 1),
                  "scratch smaller than the workspace of the largest allowed call");
    return bcm_gather_events_bwd(grad, dtype, channel_ids, time_steps, n_events, n_channels, seqlen, dx,
                                 scratch, sizeof(g_gather_bwd_scratch), stream);
}
