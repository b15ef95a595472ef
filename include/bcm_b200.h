/*
 * bcm_b200.h — C ABI of the B200 (sm_100a) event-scan pipeline.
 *
 * One shared library (libbcm_b200.so) exports every entry point below with
 * plain pointers, sizes and a cudaStream_t.  No torch types cross this line.
 * Each entry point replaces one binding of the reference's pybind11
 * extensions; the reference location it replaces is cited beside it.  The
 * caller owns and allocates every buffer (outputs and workspaces); the library
 * allocates nothing, keeps no state between calls, and is re-entrant — with
 * one exception, bcm_gather_events_bwd_noalloc, which keeps its scratch in a
 * fixed per-device array inside the library (so its calls must not overlap
 * on the GPU; see its block below).
 *
 * Conventions
 *   - Every function returns a bcm_status.  BCM_OK (0) means success; any
 *     other value leaves a thread-local message readable with bcm_last_error().
 *   - Device pointers must belong to the current CUDA device; kernels are
 *     launched on `stream` (0 = legacy default stream).
 *   - Index tensors are int32.  Event streams are channel-major: the events of
 *     logical channel c occupy [cu_seqlens[c], cu_seqlens[c+1]) in ascending t.
 *   - Workspaces are opaque device scratch of at least the size the matching
 *     *_workspace_bytes() query returns; they need no initialisation.
 */
#ifndef BCM_B200_H_
#define BCM_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BCM_ABI_VERSION 1

#if defined(__GNUC__)
#define BCM_API __attribute__((visibility("default")))
#else
#define BCM_API
#endif

typedef enum bcm_status {
    BCM_OK = 0,
    BCM_ERR_INVALID_ARGUMENT = 1, /* shape/dtype/size/pointer contract violated   */
    BCM_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed          */
    BCM_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required    */
    BCM_ERR_UNSUPPORTED = 4       /* valid request this build does not implement   */
} bcm_status;

/* Element type of the floating-point event / dense tensors.  BCM_F64 is
 * accepted only by the extraction input and the gather entry points (the
 * reference dispatches those on double as well). */
typedef enum bcm_dtype {
    BCM_F32 = 0,
    BCM_F16 = 1,
    BCM_BF16 = 2,
    BCM_F64 = 3
} bcm_dtype;

/* Thread-local description of the last failure on this thread ("" if none). */
BCM_API const char* bcm_last_error(void);
BCM_API int bcm_abi_version(void);

/* ------------------------------------------------------------------------- *
 * Event extraction.
 * Replaces extract_events_cuda.extract_base_events
 *   (reference csrc/extract/extract_events_cuda.cu:324-418).
 * Split in two calls because the output length E_base is data dependent:
 *   1. bcm_extract_base_count thresholds base_input[NCb, L] (strictly
 *      float(x) > threshold), writes counts[NCb], cu_seqlens[NCb+1],
 *      max_seqlen[1] (device, int32) and a bitmask into the workspace, then
 *      copies E_base to *n_events_host and, when max_seqlen_host is not
 *      NULL, the maximum count to it (one synchronisation of `stream`).
 *   2. bcm_extract_base_fill writes ch_ids/t_steps/k_flat[E_base] from the
 *      workspace bitmask (k = t - t_prev, first event of a channel k = t + 1).
 * ------------------------------------------------------------------------- */
BCM_API size_t bcm_extract_workspace_bytes(int64_t n_base_channels, int64_t seqlen);

BCM_API bcm_status bcm_extract_base_count(const void* base_input, bcm_dtype dtype,
                                  int64_t n_base_channels, int64_t seqlen,
                                  float threshold,
                                  int32_t* counts, int32_t* cu_seqlens,
                                  int32_t* max_seqlen,
                                  void* workspace, size_t workspace_bytes,
                                  int64_t* n_events_host, int32_t* max_seqlen_host,
                                  cudaStream_t stream);

BCM_API bcm_status bcm_extract_base_fill(int64_t n_base_channels, int64_t seqlen,
                                 const int32_t* cu_seqlens,
                                 const void* workspace, size_t workspace_bytes,
                                 int32_t* ch_ids, int32_t* t_steps,
                                 int32_t* k_flat, cudaStream_t stream);

/* Count pass of the same extraction from the (B, L, d_model) layout the model
 * keeps its spikes in, for base channel b*d_model + d: replaces the transposed
 * copy Mamba.extract_events_1d makes before extract_base_events
 * (reference spike_mamba/e_model.py:376).  Outputs, workspace and the
 * synchronisation are those of bcm_extract_base_count; bcm_extract_base_fill
 * completes it unchanged. */
BCM_API bcm_status bcm_extract_base_count_bld(const void* input_bld, bcm_dtype dtype,
                                  int64_t batch, int64_t seqlen, int64_t d_model,
                                  float threshold,
                                  int32_t* counts, int32_t* cu_seqlens,
                                  int32_t* max_seqlen,
                                  void* workspace, size_t workspace_bytes,
                                  int64_t* n_events_host, int32_t* max_seqlen_host,
                                  cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Expansion of the base stream into `expand` logical replicas per channel
 * (repeat_interleave order: logical channel = base channel * expand + r).
 * Replaces extract_events_cuda.expand_base_events
 *   (reference csrc/extract/extract_events_cuda.cu:529-603).
 * Outputs: ch_ids/t_steps/k_flat[E_base*expand], cu_seqlens[NCb*expand+1],
 * max_seqlen[1] = max per-channel count.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_expand_base_events(const int32_t* base_ch_ids,
                                  const int32_t* base_t_steps,
                                  const int32_t* base_k_flat,
                                  const int32_t* base_cu_seqlens,
                                  int64_t n_base_events, int64_t n_base_channels,
                                  int64_t expand,
                                  int32_t* ch_ids, int32_t* t_steps,
                                  int32_t* k_flat, int32_t* cu_seqlens,
                                  int32_t* max_seqlen, cudaStream_t stream);

/* Extraction fill and expansion in one pass: after bcm_extract_base_count (or
 * _bld) on the same workspace, writes the stream bcm_expand_base_events would
 * make from the base stream — ch_ids/t_steps/k_flat[E_base*expand] and
 * cu_seqlens[NCb*expand+1] — without writing the base stream; the maximum
 * per-channel count is the count pass's.  With x (B, NCb*expand/B, seqlen)
 * in x_dtype (fp32/fp16/bf16/fp64) it also writes x_flat[E_base*expand] =
 * bcm_gather_events_fwd of x at that stream; x and x_flat are both NULL
 * otherwise.  Interface path of Mamba.extract_events_1d (reference
 * spike_mamba/e_model.py:371-390, 167-193), which keeps only the expanded
 * stream and the gathered x_conv. */
BCM_API bcm_status bcm_extract_expand_fill(int64_t n_base_channels, int64_t seqlen,
                                  const int32_t* base_cu_seqlens,
                                  const void* workspace, size_t workspace_bytes,
                                  int64_t expand, int32_t* ch_ids,
                                  int32_t* t_steps, int32_t* k_flat,
                                  int32_t* cu_seqlens,
                                  const void* x, bcm_dtype x_dtype, void* x_flat,
                                  cudaStream_t stream);

/* Count + fill + optional gather in one call with its one synchronisation:
 * the fill is enqueued before the host waits for the event total (the host
 * waits for that total's copy only), into outputs of `capacity` expanded
 * events (E_base*expand of them are written when they fit; any beyond
 * capacity are skipped).  input_layout 0 is the (B, d_model, L) input of
 * bcm_extract_base_count, 1 the (B, L, d_model) one of
 * bcm_extract_base_count_bld; counts / base_cu_seqlens / max_seqlen and the
 * workspace are theirs.  On return *n_events_host = E_base; if
 * E_base*expand > capacity the caller runs bcm_extract_expand_fill with
 * outputs of the full size (the workspace and base_cu_seqlens still hold the
 * mask and offsets).  cu_seqlens[NCb*expand+1] is always written in full.
 * Interface path of Mamba.extract_events_1d (reference
 * spike_mamba/e_model.py:371-390, 167-193). */
BCM_API bcm_status bcm_extract_expanded(const void* input, bcm_dtype dtype,
                                  int32_t input_layout, int64_t batch,
                                  int64_t d_model, int64_t seqlen,
                                  float threshold, int64_t expand,
                                  int32_t* counts, int32_t* base_cu_seqlens,
                                  int32_t* max_seqlen,
                                  void* workspace, size_t workspace_bytes,
                                  int64_t capacity, int32_t* ch_ids,
                                  int32_t* t_steps, int32_t* k_flat,
                                  int32_t* cu_seqlens,
                                  const void* x, bcm_dtype x_dtype, void* x_flat,
                                  int64_t* n_events_host, int32_t* max_seqlen_host,
                                  cudaStream_t stream);

/* bcm_extract_expanded on the (B, L, d_model) layout with a threshold per
 * feature: input[b, t, j] fires when float(input[b, t, j]) >
 * feature_thresholds[j] (device, d_model floats).  No reference binding
 * (the reference thresholds with one scalar); a stack of event blocks that
 * carries its membrane without per-feature offsets extracts with it. */
BCM_API bcm_status bcm_extract_expanded_ft(const void* input_bld, bcm_dtype dtype,
                                  int64_t batch, int64_t d_model, int64_t seqlen,
                                  const float* feature_thresholds, int64_t expand,
                                  int32_t* counts, int32_t* base_cu_seqlens,
                                  int32_t* max_seqlen,
                                  void* workspace, size_t workspace_bytes,
                                  int64_t capacity, int32_t* ch_ids,
                                  int32_t* t_steps, int32_t* k_flat,
                                  int32_t* cu_seqlens,
                                  const void* x, bcm_dtype x_dtype, void* x_flat,
                                  int64_t* n_events_host, int32_t* max_seqlen_host,
                                  cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Event gather of x[NC, L] at (channel_ids, time_steps) and its transpose.
 * Replaces extract_events_cuda.gather_events_fwd / gather_events_bwd
 *   (reference csrc/extract/extract_events_cuda.cu:670-708, 717-754).
 * bcm_gather_events_bwd writes all of dx[NC, L]: zeros, then grad at events.
 * It takes a workspace of bcm_gather_bwd_workspace_bytes(NC) bytes; streams
 * in extraction order (channel_ids non-decreasing, time_steps increasing
 * within a channel) are written row by row in one pass, any other order
 * falls back to zero-fill + scatter on the device.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_gather_events_fwd(const void* x, bcm_dtype dtype,
                                 int64_t n_channels, int64_t seqlen,
                                 const int32_t* channel_ids,
                                 const int32_t* time_steps, int64_t n_events,
                                 void* out, cudaStream_t stream);

BCM_API size_t bcm_gather_bwd_workspace_bytes(int64_t n_channels);

BCM_API bcm_status bcm_gather_events_bwd(const void* grad, bcm_dtype dtype,
                                 const int32_t* channel_ids,
                                 const int32_t* time_steps, int64_t n_events,
                                 int64_t n_channels, int64_t seqlen,
                                 void* dx, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* Gather backward of a stream in extraction order with its cu_seqlens: the
 * events of channel c are [cu_seqlens[c], cu_seqlens[c+1]) (channel_ids is
 * not read), so the row-bounds pass of bcm_gather_events_bwd is skipped.
 * Results equal bcm_gather_events_bwd's for such streams; a channel whose
 * times are not strictly increasing inside [0, seqlen) has its row rewritten
 * (zeros, then that row's events in stream order).  The workspace arguments
 * are not used (NULL is fine; BCM_GATHER_BWD_ROWS_WORKSPACE is kept for
 * callers that size one).  Used by the interface's gather
 * autograd function (reference GatherEventsFn.backward,
 * spike_mamba/e_model.py:179-193), which holds cu_seqlens from extraction. */
#define BCM_GATHER_BWD_ROWS_WORKSPACE 256

BCM_API bcm_status bcm_gather_events_bwd_rows(const void* grad, bcm_dtype dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens, int64_t n_events,
                                 int64_t n_channels, int64_t seqlen,
                                 void* dx, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Gather backward that allocates nothing.  No counterpart in the reference:
 * the reference's gather_events_bwd always gets its memory from PyTorch.
 *
 * For callers that may not allocate device memory on the hot path: hosts
 * binding this library over FFI whose device memory is all carved out of
 * their own arena up front, and code that runs where cudaMalloc/cudaFree
 * would block or synchronise the device (cudaFree waits for all work on
 * the GPU).  They pass grad, the event stream and dx, and nothing else.
 *
 * Results are identical to bcm_gather_events_bwd.  Its scratch (the order
 * flag and the row table) lives in a fixed array that every GPU which loads
 * this library holds until the process exits, about 1 MiB, so n_channels is
 * limited to BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS; larger calls fail with
 * BCM_ERR_INVALID_ARGUMENT.  The array is shared by every call on a device:
 * calls that can overlap on the GPU (on different streams without ordering
 * between them) race on it and must not be issued.  The first call on each
 * device looks up the array's device address (the device must be current)
 * and should come before any stream capture; with CUDA's lazy module loading
 * that first lookup is also when the library's module is loaded on the device
 * and the array is allocated, so the first call can allocate while later
 * calls do not.  The address is cached per device for the life of the
 * process: do not keep using the library across a cudaDeviceReset().
 * ------------------------------------------------------------------------- */
#define BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS 262144

BCM_API bcm_status bcm_gather_events_bwd_noalloc(const void* grad, bcm_dtype dtype,
                                 const int32_t* channel_ids,
                                 const int32_t* time_steps, int64_t n_events,
                                 int64_t n_channels, int64_t seqlen,
                                 void* dx, cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Causal depthwise convolution + SiLU evaluated only at the events.
 * Replaces the dense x_conv = silu(conv1d(x))[..., :L] of Mamba.forward
 *   (reference spike_mamba/e_model.py:306-313, 442-451) followed by the
 *   event gather of x_conv (e_model.py:167-193): nothing else reads x_conv.
 * x[B, dim, L] in dtype; weight[dim, K] and bias[dim] (may be NULL) fp32;
 * K <= 8.  Forward: out[e] = silu(bias[d] + sum_j weight[d,j] *
 * x[b, d, t_e-K+1+j]) with zeros before position 0.  Backward writes all of
 * dx[B, dim, L] (zeros where no event reaches), dweight[dim, K] and dbias[dim]
 * (if not NULL); it needs the events sorted by time within each channel and
 * cu_seqlens[B*dim+1] (the extraction order), and a workspace of
 * bcm_conv_events_bwd_workspace_bytes(B*dim, K) bytes.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_conv_events_fwd(const void* x, bcm_dtype dtype,
                                 int64_t batch, int64_t dim, int64_t seqlen,
                                 const float* weight, const float* bias,
                                 int64_t kernel_size,
                                 const int32_t* channel_ids,
                                 const int32_t* time_steps, int64_t n_events,
                                 void* out, cudaStream_t stream);

BCM_API size_t bcm_conv_events_bwd_workspace_bytes(int64_t n_channels, int64_t kernel_size);

BCM_API bcm_status bcm_conv_events_bwd(const void* x, bcm_dtype dtype,
                                 int64_t batch, int64_t dim, int64_t seqlen,
                                 const float* weight, const float* bias,
                                 int64_t kernel_size,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens, int64_t n_events,
                                 const void* grad, void* dx,
                                 float* dweight, float* dbias,
                                 void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Flat per-channel sparse selective scan with inter-spike decay.
 * Replaces selective_scan_cuda.fwd_flat_ch / bwd_flat_ch
 *   (reference csrc/selective_scan/selective_scan.cpp:674-884, 890-1153).
 *
 * Per logical channel c (feature d = c % dim) and event i of that channel:
 *   delta_i = dt_idle[d]*(k_i - 1) + dt_active[d]
 *   a_i,s   = exp2(clamp(delta_i*A[d,s]*log2(e), -126, 126))
 *   h_i,s   = a_i,s*h_{i-1},s + delta_i*u_i*B_i,s          (h_{-1} = 0)
 *   y_i     = D[d]*u_i + sum_s h_i,s*C_i,s ; out_z = y*silu(z) when z given
 * B/C modes (bc_mode):
 *   BCM_BC_DEPTHWISE : B_i,s = u_i*W_B[d,s], C_i,s = u_i*W_C[d,s]; B,C [dim,N];
 *                      optional pw_B/pw_C [dim,dim] mix W first
 *                      (W_eff[d,s] = sum_d' pw[d,d']*W[d',s]).
 *   BCM_BC_FLAT      : B and C independently either per event [N, E]
 *                      (b_variable / c_variable = 1) or per feature [N, dim].
 *   BCM_BC_TILED     : B,C [n_tiles, N, chunk] addressed through
 *                      tile_offsets[c] + event/chunk, chunk chosen from
 *                      max_seqlen (128/256/512/1024/2048).
 * x[c, j, 2s] / x[c, j, 2s+1] = (prod of a, h) of state s after the last event
 * of 2048-event chunk j of channel c; x has n_chunks = max(1, ceil(max_seqlen /
 * 2048)) chunks per channel and must be zeroed by the caller.
 * ------------------------------------------------------------------------- */
enum {
    BCM_BC_DEPTHWISE = 0,
    BCM_BC_FLAT = 1,
    BCM_BC_TILED = 2
};

typedef struct bcm_flat_ch_args {
    /* sizes */
    int64_t n_events;     /* E                                   */
    int64_t n_channels;   /* NC = len(cu_seqlens) - 1            */
    int64_t dim;          /* D (features; channel c uses c % D)  */
    int64_t dstate;       /* N, 1..256                           */
    int64_t max_seqlen;   /* max events of one channel           */
    bcm_dtype dtype;      /* u / out / z / dout / du / dz        */
    int32_t bc_mode;      /* BCM_BC_*                            */
    int32_t b_variable;   /* BCM_BC_FLAT: B is [N,E] (1) or [N,dim] (0) */
    int32_t c_variable;   /* BCM_BC_FLAT: C is [N,E] (1) or [N,dim] (0) */
    /* forward inputs (A is [dim, N] with the given strides, in elements) */
    const void* u;
    const int32_t* k;
    const int32_t* cu_seqlens;
    const float* dt_idle;
    const float* dt_active;
    const float* A;
    int64_t A_stride_d;
    int64_t A_stride_n;
    const float* B;
    const float* C;
    const float* D;             /* nullable */
    const void* z;              /* nullable */
    const int32_t* tile_offsets;/* BCM_BC_TILED only */
    int64_t n_tiles;            /* BCM_BC_TILED: leading size of B/C (bounds check) */
    const float* pw_B;          /* nullable, depthwise only */
    const float* pw_C;
    /* forward outputs */
    void* out;                  /* [E] ungated output                 */
    float* x;                   /* [NC, n_chunks, 2N], written in full (zeros past a channel's chunks) */
    void* out_z;                /* [E] gated output when z != NULL    */
    /* backward inputs / outputs (ignored by the forward) */
    const void* dout;           /* [E] gradient of the primary output */
    const void* out_fwd;        /* [E] ungated forward output, needed with z */
    void* du;                   /* [E]                                */
    float* dA;                  /* [dim, N] contiguous                */
    float* dB;                  /* depthwise: dW_B [dim,N]; else same shape as B */
    float* dC;
    float* ddt_idle;            /* [dim] */
    float* ddt_active;          /* [dim] */
    float* dD;                  /* [dim] or NULL */
    void* dz;                   /* [E] or NULL   */
    float* dpw_B;               /* [dim,dim] or NULL */
    float* dpw_C;
    /* scratch */
    void* workspace;
    size_t workspace_bytes;
    /* nullable: state checkpoints, bcm_flat_ch_ckpt_bytes(args) bytes: the
     * normalised state entering every 8th event of a channel (staged
     * kernels) or entering every 256-event tile of a warp's events
     * (event-parallel kernels; which family runs depends on the shape and on
     * BCM_SCAN_SEG, read on every call).  The forward writes them, a backward
     * given the same buffer and settings reads them instead of re-running
     * the forward recurrence; ignored when that size is 0. */
    float* ckpt;
} bcm_flat_ch_args;

/* Bytes of the checkpoint buffer for these arguments: nonzero where the
 * staged kernels (depthwise, dstate <= 64, each feature's batch rows in
 * whole warps) or the event-parallel kernels (depthwise, no gate,
 * dstate <= 64) run, 0 where the buffer would not be used. */
BCM_API size_t bcm_flat_ch_ckpt_bytes(const bcm_flat_ch_args* args);
BCM_API size_t bcm_flat_ch_fwd_workspace_bytes(const bcm_flat_ch_args* args);
BCM_API size_t bcm_flat_ch_bwd_workspace_bytes(const bcm_flat_ch_args* args);
BCM_API bcm_status bcm_flat_ch_fwd(const bcm_flat_ch_args* args, cudaStream_t stream);
BCM_API bcm_status bcm_flat_ch_bwd(const bcm_flat_ch_args* args, cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Causal zero-order-hold restore to the dense (B, L, D) layout and its
 * backward (segment sums of dout over each event's hold interval, fp32 out).
 * Replaces restore_dense_cuda_nodecay.restore_dense_fwd / restore_dense_bwd
 *   (reference csrc/r_nodecay/restore_dense.cpp:41-123, 131-201; kernels
 *   restore_dense_fwd_kernel.cuh:38-112, restore_dense_bwd_kernel.cuh:42-113).
 * Event selection follows the reference search exactly: at most the first
 * 4095 events of a channel are addressable (index capped at 4094).
 * The times of a channel are strictly increasing and lie in [0, seqlen), as
 * extraction produces them.
 * out (fwd) and dy (bwd) are written in full; no pre-zeroing needed.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_restore_dense_fwd(const void* y_flat, bcm_dtype y_dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens,
                                 int64_t n_events, int64_t n_channels,
                                 int64_t dim, int64_t seqlen,
                                 void* out, bcm_dtype out_dtype,
                                 cudaStream_t stream);

/* Forward that also writes, for bcm_restore_dense_bwd_bitmap, the event
 * bitmap (uint32 words [b][t/32][d], bit t%32 set where channel b*dim+d has
 * an addressable event at t) followed by the local index of the first event
 * of each work unit of the sweep (int32, one per unit and lane); the buffer
 * is bcm_restore_bitmap_bytes bytes for the current device, every byte
 * written, no pre-zeroing.  The autograd pair keeps it between the two
 * passes so the backward needs neither the event times nor a search. */
BCM_API size_t bcm_restore_bitmap_bytes(int64_t n_channels, int64_t dim, int64_t seqlen);
BCM_API bcm_status bcm_restore_dense_fwd_bitmap(const void* y_flat, bcm_dtype y_dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens,
                                 int64_t n_events, int64_t n_channels,
                                 int64_t dim, int64_t seqlen,
                                 void* out, bcm_dtype out_dtype,
                                 uint32_t* event_bitmap, cudaStream_t stream);
/* bcm_restore_dense_fwd_bitmap for a stream that bcm_extract_expanded[_ft]
 * produced: the event bitmap is transposed from that call's threshold mask
 * (the first words of its workspace, [B*d_model][ceil(seqlen/32)]) instead of
 * being built from the event times; dim = d_model*expand.  base_mask must be
 * the mask of the extraction that produced time_steps / cu_seqlens (a
 * mismatch gives wrong values, not out-of-range reads).  seqlen <= 4095, the
 * per-channel event limit of the bitmap; the same outputs as
 * bcm_restore_dense_fwd_bitmap.  No reference binding. */
BCM_API bcm_status bcm_restore_dense_fwd_mask(const void* y_flat, bcm_dtype y_dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens,
                                 int64_t n_events, int64_t n_channels,
                                 int64_t dim, int64_t seqlen,
                                 void* out, bcm_dtype out_dtype,
                                 const uint32_t* base_mask, int64_t expand,
                                 uint32_t* event_bitmap, cudaStream_t stream);
BCM_API bcm_status bcm_restore_dense_bwd_bitmap(const void* dout, bcm_dtype dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens,
                                 int64_t n_events, int64_t n_channels,
                                 int64_t dim, int64_t seqlen,
                                 const uint32_t* event_bitmap, float* dy,
                                 cudaStream_t stream);

/* The backward's workspace (one bit per channel and position) is optional:
 * with it an event bitmap is built first and the row sweep needs no event
 * loads; with NULL the windowed kernel runs.  Both sum each interval in a
 * fixed order (run-to-run identical); they differ only in fp32 rounding, as
 * the windowed kernel adds 32-row partials. */
BCM_API size_t bcm_restore_workspace_bytes(int64_t n_channels, int64_t seqlen);

BCM_API bcm_status bcm_restore_dense_bwd(const void* dout, bcm_dtype dtype,
                                 const int32_t* time_steps,
                                 const int32_t* cu_seqlens,
                                 int64_t n_events, int64_t n_channels,
                                 int64_t dim, int64_t seqlen,
                                 float* dy, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* ------------------------------------------------------------------------- *
 * Decode: the event path one token at a time.  Replaces Mamba.step
 *   (reference spike_mamba/e_model.py:508-568), which cannot run as written
 *   (it reads self.pw_B / self.pw_C, undefined in Mamba) and would update
 *   every channel at every token; this step is the training path itself
 *   token by token, so decoding a sequence reproduces, bit for bit, what
 *   extraction -> flat-channel scan (depthwise) -> restore compute for it.
 * Channel c = b*dim + d.  x [batch, dim] in dtype: the token's u (x_conv), or
 * with conv_state [batch, dim, kernel_size] (dtype; rolled in place) the conv
 * input, passed through silu(conv_bias + sum_j conv_weight[d, j] * state)
 * first (conv_weight fp32 [dim, kernel_size], kernel_size <= 8, conv_bias
 * fp32 [dim] or NULL).  spikes [batch, d_model] in dtype; channel (b, d)
 * fires when spikes[b, d / (dim/d_model)] > threshold (extraction's compare).
 * A [dim, dstate] fp32 with element strides; W_B / W_C [dim, dstate] fp32
 * (effective weights: pw_B @ W_B when point-wise mixing is used); D [dim] or
 * NULL.  State, zeroed before the first token: eta [batch*dim, dstate] fp32,
 * counters [batch*dim, 2] int32 {tokens since the last event, events so
 * far}, held [batch*dim] fp32.  y [batch, dim] in dtype: the output of the
 * channel's latest event among its first 4095 (the restore's hold and search
 * cap), 0 before its first event.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_event_decode_step(const void* x, const void* spikes, bcm_dtype dtype,
                                 int64_t batch, int64_t dim, int64_t d_model,
                                 int64_t dstate, float threshold,
                                 const float* dt_idle, const float* dt_active,
                                 const float* A, int64_t A_stride_d, int64_t A_stride_n,
                                 const float* W_B, const float* W_C, const float* D,
                                 void* conv_state, const float* conv_weight,
                                 const float* conv_bias, int64_t kernel_size,
                                 float* eta, int32_t* counters, float* held,
                                 void* y, cudaStream_t stream);

/* -------------------------------------------------------------------------
 * Dense selective scan (Mamba's S6) — replaces selective_scan_cuda.fwd / .bwd
 * (reference csrc/selective_scan/selective_scan.cpp:403-669, kernels
 * selective_scan_fwd_kernel.cuh:84-326 and selective_scan_bwd_kernel.cuh:
 * 31-500), real weights.
 *
 * u, delta, z, out, out_z, dout, du, ddelta, dz [batch, dim, seqlen] in dtype
 * (u and delta with the batch / dim strides below and unit position stride,
 * the others contiguous); A [dim, dstate] fp32 (strides);
 * B, C either fixed [dim, dstate] fp32 (strides) or variable
 * [batch, n_groups, dstate, seqlen] in dtype (contiguous), channel d reading
 * group d / (dim / n_groups); D, delta_bias [dim] fp32 or NULL.
 * delta' = delta + delta_bias, then softplus (log1p(exp), identity above 20)
 * when delta_softplus; h_s = exp2(clamp(delta'*A_s*log2(e), +-126)) * h_s +
 * (B variable ? B_s : 1) * delta' * u; y = sum_s C'_s * h_s + D * u with
 * C'_s = (C variable ? C_s : C_s) * (B fixed ? B_s : 1); out_z = y * silu(z).
 * x [batch, dim, ceil(seqlen/2048), 2*dstate] fp32: after each 2048-position
 * chunk, (product of the decays since position 0, h_s) per state.
 * Backward: du, ddelta in dtype; dA [dim, dstate], dB / dC (fixed: [dim,
 * dstate]; variable: [batch, n_groups, dstate, seqlen]), dD, ddelta_bias
 * fp32, all ACCUMULATED into (the caller zeroes them); dz when z is given
 * (needs `out`, the ungated forward output), out_z recomputed when non-NULL.
 * The backward re-runs the recurrence from position 0 (x is not read) and
 * needs bcm_s6_bwd_workspace_bytes of workspace.
 * ------------------------------------------------------------------------- */
typedef struct bcm_s6_args {
    int64_t batch, dim, seqlen, dstate, n_groups;
    bcm_dtype dtype;
    int is_variable_B, is_variable_C, delta_softplus;
    const void* u; int64_t u_stride_b, u_stride_d;
    const void* delta; int64_t delta_stride_b, delta_stride_d;
    const float* A; int64_t A_stride_d, A_stride_n;
    const void* B; int64_t B_stride_d, B_stride_n;   /* strides: fixed B only */
    const void* C; int64_t C_stride_d, C_stride_n;   /* strides: fixed C only */
    const float* D;
    const float* delta_bias;
    const void* z;
    /* forward outputs */
    void* out; void* out_z; float* x;
    /* backward */
    const void* dout; const void* out_fwd;
    void* du; void* ddelta; float* dA; float* dB; float* dC; float* dD; float* ddelta_bias;
    void* dz;
    void* workspace; size_t workspace_bytes;
} bcm_s6_args;

BCM_API bcm_status bcm_s6_fwd(const bcm_s6_args* args, cudaStream_t stream);
BCM_API size_t bcm_s6_bwd_workspace_bytes(const bcm_s6_args* args);
BCM_API bcm_status bcm_s6_bwd(const bcm_s6_args* args, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Event-block parameter transforms.  No reference binding: the reference
 * computes them with PyTorch ops in Mamba.forward (spike_mamba/e_model.py:463
 * A = -exp(A_log); :475-476 W_B / W_C = the halves of W_BC; :210-230
 * TwoLevelDelta dt_idle / dt_active = softplus(a0 / a1) + eps), eight small
 * kernels per direction; here one launch each way.
 * A_log, A, W_B, W_C, dA, dW_B, dW_C [dim, dstate]; W_BC, dW_BC [dim,
 * 2*dstate]; a0, a1, dt_*, da0, da1 [dim]; all fp32, contiguous.
 * softplus: x above 20 passes through (torch.nn.functional.softplus).
 * Backward: the gradient pointers dA, dW_B, dW_C, ddt_idle, ddt_active may
 * each be NULL (a zero gradient); every output is written, not accumulated.
 * ------------------------------------------------------------------------- */
BCM_API bcm_status bcm_event_params_fwd(const float* A_log, const float* W_BC, const float* a0,
                                        const float* a1, int64_t dim, int64_t dstate, float eps,
                                        float* A, float* W_B, float* W_C, float* dt_idle,
                                        float* dt_active, cudaStream_t stream);
BCM_API bcm_status bcm_event_params_bwd(const float* A, const float* a0, const float* a1,
                                        const float* dA, const float* dW_B, const float* dW_C,
                                        const float* ddt_idle, const float* ddt_active, int64_t dim,
                                        int64_t dstate, float* dA_log, float* dW_BC, float* da0,
                                        float* da1, cudaStream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* BCM_B200_H_ */
