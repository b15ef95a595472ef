// scan_common.cuh — layout and helpers shared by the flat-channel scan kernels.
//
// Thread mapping (both directions): a CTA of kScanThreads threads covers
// kScanThreads / LPC logical channels; the LPC consecutive lanes of a channel
// ("group") each own G of the channel's states, so LPC * G >= dstate.  Events
// of a channel are walked sequentially (a register recurrence per state,
// fully independent across states), so there is no block-wide scan and no
// barrier in the inner loop; the per-event sum over states is a shuffle
// reduction inside the group.  Parallelism comes from channels x state groups.
#pragma once

#include "common.cuh"

namespace bcm {

constexpr int kScanThreads = 128;
constexpr int kChunkX = 2048;   // events per saved chunk state (x layout)
constexpr int kCkpt = 8;        // events per backward recompute tile
constexpr float kLog2e = 1.4426950408889634f;

// Arguments shared by the scan kernels (device-visible copy of the C ABI args).
struct ScanArgs {
    int n_channels, dim, dstate, n_chunks, n_events;
    int bc_mode, b_variable, c_variable, tile_cs, n_tiles;
    const void* u; const int32_t* k; const int32_t* cu;
    const float* dt_idle; const float* dt_active;
    const float* A; int64_t A_sd, A_sn;
    const float* B; const float* C;      // depthwise: effective W_B/W_C [dim, N]
    const float* D; const void* z; const int32_t* tile_off;
    void* out; float* x; void* out_z;
    const void* dout; const void* out_fwd;
    void* du; float* dB_ev; float* dC_ev;  // per-event dB/dC (flat variable / tiled)
    void* dz;
    float* ws_ckpt;   // backward: recompute checkpoints
    float* ckpt;      // staged kernels: the forward writes the checkpoints here and the
                      // backward reads them instead of recomputing (nullable)
    float* ws_part;   // backward: per-channel parameter-gradient partials
    int part_stride;  // floats per channel in ws_part
    const int* row_order;  // staged kernels (nullable): batch rows of each feature d in
                           // descending event count, [dim][n_channels/dim], so the rows a
                           // warp walks in lockstep have similar lengths
    const float* dtab;     // staged kernels (nullable): decay tables computed once per call,
                           // [dim][padded dstate][kKT3 + 1], copied by each CTA instead of
                           // evaluating exp2 in double per CTA
    int rank_major;        // staged kernels: CTA i walks row group i / dim of feature
                           // i % dim (set with row_order: every feature's longest rows
                           // are dispatched first), else feature-major
};

// Batch row of slot b of feature d in the staged kernels' walk.
__device__ __forceinline__ int scan_row(const ScanArgs& a, int d, int b) {
    return a.row_order ? a.row_order[d * (a.n_channels / a.dim) + b] : b;
}

__device__ __forceinline__ bool rank_major(const ScanArgs& a) { return a.rank_major != 0; }

// Decay factor exp2(clamp(delta*A2, -126, 126)) with the accurate exp2f
// (as the reference): with long-memory states (a close to 1) a biased
// approximation would compound over ~1/(1-a) events.
__device__ __forceinline__ float decay_fast(float delta, float A2) {
    return exp2f(fmaxf(fminf(delta * A2, 126.0f), -126.0f));
}

// Same decay, correctly rounded to fp32 (exp2 evaluated in double).  The
// depthwise path tabulates decays per integer gap, so each rounded value is
// reused by every event with that gap; rounding it correctly keeps the
// coherent error of long-memory states (a close to 1) at the fp32 limit.
// Gaps past a table take decay_fast, the reference's exp2f: they are rare and
// their values hardly repeat, and a double-precision exp2 per event and state
// would make a sparse channel cost hundreds of times a dense one.
__device__ __forceinline__ float decay_exact(float delta, float A2) {
    const float x = fmaxf(fminf(delta * A2, 126.0f), -126.0f);
    return (float)exp2((double)x);
}

// delta of an event with gap k: dt_idle*(k-1) + dt_active (one rounding, as
// the reference's contracted expression).
__device__ __forceinline__ float event_delta(float dt_idle, float dt_active, int k) {
    return fmaf(dt_idle, (float)(k - 1), dt_active);
}

// Sum over the LPC lanes of a group (groups are aligned to LPC lanes).
template <int LPC>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int off = LPC / 2; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
    return v;
}

template <int LPC>
__device__ __forceinline__ int group_max_warp(int v) {
    // max over the whole warp (all groups), used for warp-uniform trip counts
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(kFull, v, off));
    return v;
}

// Sum v[0..NE) over the LPC lanes of a group.  Afterwards lane q holds the
// totals of events q*(NE/LPC) + j in v[j], j < NE/LPC.
template <int LPC, int NE>
__device__ __forceinline__ void group_transpose_sum(float (&v)[NE], int q) {
#pragma unroll
    for (int lvl = 0; (LPC >> lvl) > 1; ++lvl) {
        const int o = (LPC >> lvl) / 2;
        const int half = (NE >> lvl) / 2;
        const bool up = (q & o) != 0;
#pragma unroll
        for (int j = 0; j < half; ++j) {
            const float send = up ? v[j] : v[j + half];
            const float recv = __shfl_xor_sync(kFull, send, o);
            v[j] = (up ? v[j + half] : v[j]) + recv;
        }
    }
}

__device__ __forceinline__ float silu(float z) { return z / (1.0f + expf(-z)); }

// Reference event-chunk size for the tiled B/C layout: the forward kernel's
// kNThreads*kNItems picked from max_seqlen
// (selective_scan_fwd_kernel.cuh:771-785).
inline int ref_chunk_size(int64_t max_seqlen) {
    if (max_seqlen <= 128) return 128;
    if (max_seqlen <= 256) return 256;
    if (max_seqlen <= 512) return 512;
    if (max_seqlen <= 1024) return 1024;
    return 2048;
}

inline int n_chunks_for(int64_t max_seqlen) {
    int64_t n = (max_seqlen + kChunkX - 1) / kChunkX;
    return (int)(n < 1 ? 1 : n);
}

// Lanes per channel and states per lane for dstate N.
inline void pick_layout(int N, int& G, int& LPC) {
    if (N <= 128) {
        G = 4;
        int l = (N + 3) / 4;
        LPC = 1;
        while (LPC < l) LPC <<= 1;
    } else {
        G = 8;
        LPC = 32;
    }
}

// Depthwise fast path (scan_dw.cu), used for dstate <= 64.
bool dw_fast_supported(int dstate);
int dw_fast_np(int dstate);
bcm_status dw_fast_launch(const ScanArgs& a, bcm_dtype dtype, bool bwd, cudaStream_t st);

// Staged lane-group kernels (scan_v3.cu) for dstate <= 64 when the channels
// of one feature fill whole warps; dw_fast_launch prefers them.
bool v3_supported(const ScanArgs& a, bool bwd);
bcm_status v3_launch(const ScanArgs& a, bcm_dtype dtype, bool bwd, cudaStream_t st);
// Floats per checkpoint slot of the staged kernels (dstate padded), and the
// checkpoint buffer size shared by their forward and backward (0 when either
// does not apply, in which case ScanArgs::ckpt must be null).
int v3_ckpt_np(int dstate);
// Warps of the staged backward for these arguments (its lane groups hold
// whole channels).
int64_t v3_bwd_warps(const ScanArgs& a);
size_t v3_ckpt_bytes(const ScanArgs& a);

// Event-parallel kernels (scan_seg.cu): depthwise, no gate, dstate <= 64.
// The forward needs a decay-table workspace of seg_table_bytes and writes the
// state entering every tile into the checkpoint buffer (seg_carry_bytes);
// the backward needs the same table, the carries (from the forward, or it
// writes them into carry_ws itself) and seg_part_rows partial rows.
bool seg_supported(const ScanArgs& a);
// Whether the dispatch runs the event-parallel kernels for these arguments
// (BCM_SCAN_SEG: 0 never, 1 where the staged kernels do not apply (default),
// 2 wherever supported).
bool seg_selected(const ScanArgs& a);
// Staged kernels: per-call preparation in a workspace of staged_prep_bytes:
// the row order (scan_row) of every feature and the decay tables (dtab);
// staged_prep_launch fills it and points a.row_order / a.dtab at it.
size_t staged_prep_bytes(const ScanArgs& a);
bcm_status staged_prep_launch(ScanArgs& a, void* ws, cudaStream_t st);
size_t seg_table_bytes(const ScanArgs& a);
size_t seg_carry_bytes(const ScanArgs& a);
int seg_part_rows(const ScanArgs& a);
bcm_status seg_fwd_launch(const ScanArgs& a, bcm_dtype dtype, float* table_ws, float* carries, cudaStream_t st);
bcm_status seg_bwd_launch(const ScanArgs& a, bcm_dtype dtype, float* table_ws, const float* fwd_carries,
                          float* carry_ws, cudaStream_t st);

}  // namespace bcm
