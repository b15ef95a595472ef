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
// Design (ours): a CTA owns one batch row b, 32 consecutive features d and a
// range of positions.  It walks that range in windows of kTT positions.  For
// each window, every channel's events are loaded 32 at a time by a warp
// (coalesced) and each lane fills / sums its event's hold interval in a
// shared-memory tile [kTT][33]; the tile is exchanged with HBM row by row so
// every global access is a contiguous 32-feature row of (B, L, D).  This
// replaces the reference's per-(t,d) binary search and its strided stores, and
// the backward's fp32 atomics with a deterministic ordered sum: the CTA that
// owns an event's start keeps reading past its range until the event ends.
#include "common.cuh"

namespace bcm {
namespace {

constexpr int kDB = 32;       // features per CTA
constexpr int kTT = 64;       // positions per window
constexpr int kWarpsR = 4;    // warps per CTA (8 channels per warp)
constexpr int kChPerWarp = kDB / kWarpsR;
constexpr int kCap = 4095;    // addressable events per channel (reference search limit)

__device__ __forceinline__ int lower_bound_i32(const int32_t* a, int n, int key) {
    int lo = 0, hi = n;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (a[mid] < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(kWarpsR * 32)
restore_fwd_kernel(const Tin* __restrict__ y, const int32_t* __restrict__ ts,
                   const int32_t* __restrict__ cu, int D, int L, int part_len,
                   int n_dblk, Tout* __restrict__ out) {
    __shared__ float tile[kTT][kDB + 1];
    __shared__ int s_ptr[kDB];     // next event (local index) with t >= window start
    __shared__ int s_n[kDB];       // addressable events
    __shared__ int s_beg[kDB];     // global index of the channel's first event
    __shared__ float s_carry[kDB]; // value held at the window start

    const int dblk = blockIdx.x % n_dblk;
    const int part = blockIdx.x / n_dblk;
    const int b = blockIdx.y;
    const int d0 = dblk * kDB;
    const int t_beg = part * part_len;
    const int t_end = min(L, t_beg + part_len);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid < kDB) {
        const int d = d0 + tid;
        int beg = 0, n = 0, p = 0;
        float carry = 0.f;
        if (d < D) {
            const int ch = b * D + d;
            beg = cu[ch];
            n = min(cu[ch + 1] - beg, kCap);
            p = lower_bound_i32(ts + beg, n, t_beg);
            if (p > 0) carry = to_f32<Tin>(y[beg + p - 1]);
        }
        s_ptr[tid] = p; s_n[tid] = n; s_beg[tid] = beg; s_carry[tid] = carry;
    }
    __syncthreads();

    for (int t0 = t_beg; t0 < t_end; t0 += kTT) {
        const int wend = min(t0 + kTT, t_end);
        for (int ci = 0; ci < kChPerWarp; ++ci) {
            const int c = warp * kChPerWarp + ci;
            if (d0 + c >= D) break;
            const int n = s_n[c], beg = s_beg[c];
            int p = s_ptr[c];
            float carry = s_carry[c];
            int fill_from = t0;
            while (true) {
                const int j = p + lane;
                const int tj = (j < n) ? ts[beg + j] : INT_MAX;
                const bool valid = tj < wend;
                const unsigned vm = __ballot_sync(kFull, valid);
                const int cnt = __popc(vm);
                const int first_t = cnt ? __shfl_sync(kFull, tj, 0) : wend;
                // hold the carried value up to the first event of this batch
                for (int t = max(fill_from, t0) + lane; t < first_t; t += 32) tile[t - t0][c] = carry;
                if (cnt == 0) break;
                const float yj = valid ? to_f32<Tin>(y[beg + j]) : 0.f;
                int tn = __shfl_down_sync(kFull, tj, 1);
                if (lane == 31) tn = (p + 32 < n) ? ts[beg + p + 32] : INT_MAX;
                const int seg_end = min(tn, wend);
                if (valid)
                    for (int t = max(tj, t0); t < seg_end; ++t) tile[t - t0][c] = yj;
                carry = __shfl_sync(kFull, yj, cnt - 1);
                const int last_end = __shfl_sync(kFull, seg_end, cnt - 1);
                p += cnt;
                fill_from = last_end;
                if (cnt < 32 || last_end >= wend) break;
            }
            if (lane == 0) { s_ptr[c] = p; s_carry[c] = carry; }
        }
        __syncthreads();
        const int rows = wend - t0;
        for (int idx = tid; idx < rows * kDB; idx += kWarpsR * 32) {
            const int r = idx / kDB, c = idx % kDB;
            if (d0 + c < D)
                out[((int64_t)b * L + t0 + r) * D + d0 + c] = from_f32<Tout>(tile[r][c]);
        }
        __syncthreads();
    }
}

template <typename T>
__global__ void __launch_bounds__(kWarpsR * 32)
restore_bwd_kernel(const T* __restrict__ dout, const int32_t* __restrict__ ts,
                   const int32_t* __restrict__ cu, int D, int L, int part_len,
                   int n_dblk, float* __restrict__ dy) {
    // Per channel: p = next event (local index) whose start is not processed,
    // open = event whose hold interval is running (-1: none of ours), acc = its
    // partial sum.  Events starting in [t_beg, t_own_end) are owned here; the
    // CTA keeps reading past t_own_end until each owned interval has ended.
    __shared__ float tile[kTT][kDB + 1];
    __shared__ int s_ptr[kDB];
    __shared__ int s_n[kDB];
    __shared__ int s_beg[kDB];
    __shared__ int s_open[kDB];
    __shared__ float s_acc[kDB];
    __shared__ int s_any_open;

    const int dblk = blockIdx.x % n_dblk;
    const int part = blockIdx.x / n_dblk;
    const int b = blockIdx.y;
    const int d0 = dblk * kDB;
    const int t_beg = part * part_len;
    const int t_own_end = min(L, t_beg + part_len);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid < kDB) {
        const int d = d0 + tid;
        int beg = 0, n = 0, p = 0;
        if (d < D) {
            const int ch = b * D + d;
            beg = cu[ch];
            const int n_all = cu[ch + 1] - beg;
            n = min(n_all, kCap);
            p = lower_bound_i32(ts + beg, n, t_beg);
            if (part == 0)  // events past the search cap receive no gradient
                for (int j = kCap; j < n_all; ++j) dy[beg + j] = 0.f;
        }
        s_ptr[tid] = p; s_n[tid] = n; s_beg[tid] = beg;
        s_open[tid] = -1;
        s_acc[tid] = 0.f;
    }
    __syncthreads();

    for (int t0 = t_beg; t0 < L; t0 += kTT) {
        const bool owning = t0 < t_own_end;
        const int wend = min(t0 + kTT, owning ? t_own_end : L);
        if (!owning) {
            if (tid == 0) {
                int any = 0;
                for (int c = 0; c < kDB; ++c) any |= (s_open[c] >= 0);
                s_any_open = any;
            }
            __syncthreads();
            if (!s_any_open) break;
        }
        const int rows = wend - t0;
        for (int idx = tid; idx < rows * kDB; idx += kWarpsR * 32) {
            const int r = idx / kDB, c = idx % kDB;
            tile[r][c] = (d0 + c < D) ? to_f32<T>(dout[((int64_t)b * L + t0 + r) * D + d0 + c]) : 0.f;
        }
        __syncthreads();
        for (int ci = 0; ci < kChPerWarp; ++ci) {
            const int c = warp * kChPerWarp + ci;
            if (d0 + c >= D) break;
            const int n = s_n[c], beg = s_beg[c];
            int p = s_ptr[c];
            int open = s_open[c];
            float acc = s_acc[c];
            if (!owning) {
                if (open >= 0) {
                    const int tn = (open + 1 < n) ? ts[beg + open + 1] : INT_MAX;
                    const int stop = min(tn, wend);
                    float s = 0.f;
                    for (int t = t0 + lane; t < stop; t += 32) s += tile[t - t0][c];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(kFull, s, off);
                    acc += s;
                    if (tn <= wend) {
                        if (lane == 0) dy[beg + open] = acc;
                        open = -1;
                        acc = 0.f;
                    }
                }
            } else {
                int from = t0;
                while (true) {
                    const int j = p + lane;
                    const int tj = (j < n) ? ts[beg + j] : INT_MAX;
                    const bool valid = tj < wend;
                    const int cnt = __popc(__ballot_sync(kFull, valid));
                    const int first_t = cnt ? __shfl_sync(kFull, tj, 0) : wend;
                    // [from, first_t) still belongs to the open interval
                    float s = 0.f;
                    for (int t = max(from, t0) + lane; t < first_t; t += 32) s += tile[t - t0][c];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(kFull, s, off);
                    acc += s;
                    if (cnt == 0) break;
                    if (open >= 0 && lane == 0) dy[beg + open] = acc;  // next event ended it
                    // each valid lane owns [tj, tn)
                    int tn = __shfl_down_sync(kFull, tj, 1);
                    if (lane == 31) tn = (p + 32 < n) ? ts[beg + p + 32] : INT_MAX;
                    const int seg_end = min(tn, wend);
                    float v = 0.f;
                    if (valid)
                        for (int t = max(tj, t0); t < seg_end; ++t) v += tile[t - t0][c];
                    if (valid && tn <= wend) dy[beg + j] = v;
                    const int tn_last = __shfl_sync(kFull, tn, cnt - 1);
                    const float v_last = __shfl_sync(kFull, v, cnt - 1);
                    p += cnt;
                    if (tn_last <= wend) {
                        open = -1;
                        acc = 0.f;
                        from = tn_last;
                        if (cnt < 32 || tn_last >= wend) break;
                    } else {
                        open = p - 1;
                        acc = v_last;
                        break;
                    }
                }
            }
            if (lane == 0) { s_ptr[c] = p; s_open[c] = open; s_acc[c] = acc; }
        }
        __syncthreads();
    }
    // intervals still open at L end there
    if (tid < kDB && d0 + tid < D && s_open[tid] >= 0)
        dy[s_beg[tid] + s_open[tid]] = s_acc[tid];
}

}  // namespace
}  // namespace bcm

using namespace bcm;

static int restore_part_len(int64_t n_blocks_2d, int64_t L) {
    // Enough CTAs to cover the SMs several times, windows of kTT positions.
    const int64_t target = (int64_t)sm_count() * 8;
    int64_t parts = std::max<int64_t>(1, target / std::max<int64_t>(1, n_blocks_2d));
    int64_t len = (L + parts - 1) / parts;
    len = std::max<int64_t>(kTT * 4, (len + kTT - 1) / kTT * kTT);
    return (int)std::min<int64_t>(len, std::max<int64_t>(L, 1));
}

extern "C" bcm_status bcm_restore_dense_fwd(const void* y_flat, bcm_dtype y_dtype,
                                            const int32_t* time_steps, const int32_t* cu_seqlens,
                                            int64_t n_events, int64_t n_channels, int64_t dim,
                                            int64_t seqlen, void* out, bcm_dtype out_dtype,
                                            cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(y_dtype) && dtype_ok(out_dtype), "restore_dense_fwd: unsupported dtype");
    BCM_REQUIRE(y_dtype == BCM_F32 || y_dtype == out_dtype,
                "restore_dense_fwd: 16-bit input only supports the same output dtype");
    BCM_REQUIRE(dim >= 1 && seqlen >= 1 && n_channels >= 1 && n_events >= 0,
                "restore_dense_fwd: bad sizes");
    BCM_REQUIRE(n_channels % dim == 0, "restore_dense_fwd: n_channels must be divisible by dim");
    BCM_REQUIRE(seqlen < (1ll << 31) - 64, "restore_dense_fwd: seqlen too large");
    BCM_REQUIRE(out && cu_seqlens && (n_events == 0 || (y_flat && time_steps)),
                "restore_dense_fwd: null pointer");
    const int64_t B = n_channels / dim;
    const int n_dblk = ceil_div(dim, kDB);
    const int part_len = restore_part_len(B * n_dblk, seqlen);
    const int n_parts = ceil_div(seqlen, part_len);
    BCM_REQUIRE(B < 65536, "restore_dense_fwd: batch too large");
    dim3 grid(n_dblk * n_parts, (unsigned)B);
    auto launch = [&](auto tin, auto tout) -> bcm_status {
        using Tin = decltype(tin);
        using Tout = decltype(tout);
        restore_fwd_kernel<Tin, Tout><<<grid, kWarpsR * 32, 0, stream>>>(
            static_cast<const Tin*>(y_flat), time_steps, cu_seqlens, (int)dim, (int)seqlen,
            part_len, n_dblk, static_cast<Tout*>(out));
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

extern "C" bcm_status bcm_restore_dense_bwd(const void* dout, bcm_dtype dtype,
                                            const int32_t* time_steps, const int32_t* cu_seqlens,
                                            int64_t n_events, int64_t n_channels, int64_t dim,
                                            int64_t seqlen, float* dy, cudaStream_t stream) {
    clear_error();
    BCM_REQUIRE(dtype_ok(dtype), "restore_dense_bwd: unsupported dtype");
    BCM_REQUIRE(dim >= 1 && seqlen >= 1 && n_channels >= 0 && n_events >= 0,
                "restore_dense_bwd: bad sizes");
    BCM_REQUIRE(n_channels % dim == 0, "restore_dense_bwd: n_channels must be divisible by dim");
    if (n_events == 0 || n_channels == 0) return BCM_OK;
    BCM_REQUIRE(dout && time_steps && cu_seqlens && dy, "restore_dense_bwd: null pointer");
    const int64_t B = n_channels / dim;
    BCM_REQUIRE(B < 65536, "restore_dense_bwd: batch too large");
    const int n_dblk = ceil_div(dim, kDB);
    const int part_len = restore_part_len(B * n_dblk, seqlen);
    const int n_parts = ceil_div(seqlen, part_len);
    dim3 grid(n_dblk * n_parts, (unsigned)B);
    return dispatch_dtype(dtype, [&](auto tag) -> bcm_status {
        using T = decltype(tag);
        restore_bwd_kernel<T><<<grid, kWarpsR * 32, 0, stream>>>(
            static_cast<const T*>(dout), time_steps, cu_seqlens, (int)dim, (int)seqlen, part_len,
            n_dblk, dy);
        BCM_LAUNCH_CHECK();
        return BCM_OK;
    });
}
