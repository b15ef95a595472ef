"""Autograd boundary of the event pipeline, identical in signature to the
reference's Python layer so callers switch without edits:

* ``SelectiveScanFlatChFn`` / ``selective_scan_flat_ch_fn``
  (spike_mamba/selective_scan_interface.py:1015-1237)
* ``RestoreDenseFn`` / ``restore_dense_fn``  (spike_mamba/e_model.py:123-161)
* ``GatherEventsFn`` / ``gather_events``       (spike_mamba/e_model.py:167-193)
* ``extract_events_1d``                        (spike_mamba/e_model.py:361-409)
* ``EventParamsFn`` / ``event_params``          (the parameter transforms of
  Mamba.forward, spike_mamba/e_model.py:210-230, 463, 475-476, in one kernel)

All device work goes through the native shim (``bc_mamba_b200._native``);
there is no Python or CPU fallback.  ``install_shim()`` puts the drop-in
modules ``selective_scan_cuda``, ``extract_events_cuda`` and
``restore_dense_cuda_nodecay`` on ``sys.path`` so the reference's own
``e_model.py`` / ``lra_impl.py`` import them unchanged.
"""
from __future__ import annotations

import contextlib
import sys
from pathlib import Path

import torch

from ._native import load_ops

SHIM_DIR = Path(__file__).resolve().parent / "shim"


def install_shim() -> None:
    """Make ``import selective_scan_cuda`` (and the other two) resolve here."""
    p = str(SHIM_DIR)
    if p not in sys.path:
        sys.path.insert(0, p)


_stage_log = None   # list of (name, start, end) CUDA events while stage_timing() is open


@contextlib.contextmanager
def stage_timing():
    """Record a CUDA event pair on the launching stream around every
    cuda_stage entered while the context is open (autograd's backward thread
    included).  Yields the list of (name, start_event, end_event); read the
    times after a synchronize."""
    global _stage_log
    prev, _stage_log = _stage_log, []
    try:
        yield _stage_log
    finally:
        _stage_log = prev


@contextlib.contextmanager
def cuda_stage(name: str):
    """NVTX range named like the reference's profiling stages
    (spike_mamba/runtime_breakdown.py:12-15), timed with CUDA events while
    stage_timing() is open."""
    if torch.cuda.is_available():
        log = _stage_log
        torch.cuda.nvtx.range_push(name)
        if log is not None:
            start = torch.cuda.Event(enable_timing=True)
            start.record()
        try:
            yield
        finally:
            if log is not None:
                end = torch.cuda.Event(enable_timing=True)
                end.record()
                log.append((name, start, end))
            torch.cuda.nvtx.range_pop()
    else:
        yield


class SelectiveScanFlatChFn(torch.autograd.Function):
    """Flat per-channel selective scan over event streams.

    Forward inputs (positional): u_flat, k_flat, cu_seqlens, dt_idle,
    dt_active, A, B, C, D, z, max_seqlen, tile_offsets, tile_chunk_size,
    is_depthwise_bc, pw_B, pw_C.  Returns (out, x) where x holds the chunk
    boundary states (non-differentiable); out is gated by silu(z) if z given.
    """

    @staticmethod
    def forward(ctx, u_flat, k_flat, cu_seqlens, dt_idle, dt_active, A, B, C, D, z,
                max_seqlen, tile_offsets, tile_chunk_size, is_depthwise_bc, pw_B, pw_C):
        ops = load_ops()
        u_flat = u_flat.contiguous()
        k_flat = k_flat.contiguous()
        cu_seqlens = cu_seqlens.contiguous()
        dt_idle = dt_idle.contiguous()
        dt_active = dt_active.contiguous()
        A, B, C = A.contiguous(), B.contiguous(), C.contiguous()
        D = D.contiguous() if D is not None else None
        z = z.contiguous() if z is not None else None
        tile_offsets = tile_offsets.contiguous() if tile_offsets is not None else None
        pw_B = pw_B.contiguous() if pw_B is not None else None
        pw_C = pw_C.contiguous() if pw_C is not None else None
        with cuda_stage("sparse_scan_forward"):
            # the forward also keeps the state every 8 events (where the
            # staged kernels run) so the backward does not re-run the recurrence
            res = ops.fwd_flat_ch_ckpt(u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle, dt_active,
                                       A, B, C, D, z, tile_offsets, tile_chunk_size,
                                       is_depthwise_bc, pw_B, pw_C)
        out, x, ckpt = res[0], res[1], res[-1]
        ctx.has_D = D is not None
        ctx.has_z = z is not None
        ctx.has_tiles = tile_offsets is not None
        ctx.has_pw = pw_B is not None
        ctx.max_seqlen = max_seqlen
        ctx.tile_chunk_size = tile_chunk_size
        ctx.is_depthwise_bc = is_depthwise_bc
        saved = [u_flat, k_flat, cu_seqlens, dt_idle, dt_active, A, B, C, x]
        if ctx.has_D:
            saved.append(D)
        if ctx.has_z:
            saved += [z, out]
        if ctx.has_tiles:
            saved.append(tile_offsets)
        if ctx.has_pw:
            saved += [pw_B, pw_C]
        saved.append(ckpt)
        ctx.save_for_backward(*saved)
        ctx.mark_non_differentiable(x)
        # x takes no gradient: without this autograd fills a zero tensor for it
        ctx.set_materialize_grads(False)
        return (res[2] if ctx.has_z else out), x

    @staticmethod
    def backward(ctx, dout, _dx):
        ops = load_ops()
        if dout is None:        # the output was not used in the loss
            return (None,) * 16
        if dout.stride(-1) != 1:
            dout = dout.contiguous()
        it = iter(ctx.saved_tensors)
        u_flat, k_flat, cu_seqlens, dt_idle, dt_active, A, B, C, x = (next(it) for _ in range(9))
        D = next(it) if ctx.has_D else None
        z, out = (next(it), next(it)) if ctx.has_z else (None, None)
        tile_offsets = next(it) if ctx.has_tiles else None
        pw_B, pw_C = (next(it), next(it)) if ctx.has_pw else (None, None)
        ckpt = next(it)
        with cuda_stage("sparse_scan_backward"):
            res = ops.bwd_flat_ch(u_flat, k_flat, cu_seqlens, ctx.max_seqlen, dt_idle, dt_active,
                                  A, B, C, dout, x, D, z, out, tile_offsets,
                                  ctx.tile_chunk_size, ctx.is_depthwise_bc, pw_B, pw_C,
                                  ckpt if ckpt.numel() > 0 else None)
        du, dA, dB, dC, ddt_idle, ddt_active = res[:6]
        rest = iter(res[6:])
        dD = next(rest) if ctx.has_D else None
        dz = next(rest) if ctx.has_z else None
        dpw_B, dpw_C = (next(rest), next(rest)) if ctx.has_pw else (None, None)
        return (du, None, None, ddt_idle, ddt_active, dA, dB, dC, dD, dz,
                None, None, None, None, dpw_B, dpw_C)


def selective_scan_flat_ch_fn(u_flat, k_flat, cu_seqlens, max_seqlen, dt_idle, dt_active, A, B, C,
                              D=None, z=None, tile_offsets=None, tile_chunk_size=0,
                              is_depthwise_bc=False, pw_B=None, pw_C=None):
    """Autograd-enabled flat per-channel selective scan; returns (out, x)."""
    return SelectiveScanFlatChFn.apply(u_flat, k_flat, cu_seqlens, dt_idle, dt_active, A, B, C,
                                       D, z, max_seqlen, tile_offsets, tile_chunk_size,
                                       is_depthwise_bc, pw_B, pw_C)


class RestoreDenseFn(torch.autograd.Function):
    """Zero-order-hold restore: (E,) event values -> (B, L, D) dense."""

    @staticmethod
    def forward(ctx, y_flat, time_steps_i32, cu_seqlens, dim: int, seqlen: int, base_mask=None, expand: int = 1):
        # the forward also writes the event bitmap (one bit per channel and
        # position) that the backward sweeps instead of the event times;
        # base_mask: the extraction's threshold mask of this stream, which the
        # bitmap is transposed from instead
        with cuda_stage("dense_restoration_forward"):
            out, bitmap = load_ops().restore_dense_fwd_bitmap(y_flat, time_steps_i32, cu_seqlens, dim, seqlen,
                                                              base_mask=base_mask, expand=expand)
        ctx.save_for_backward(time_steps_i32, cu_seqlens, bitmap)
        ctx.dim = dim
        ctx.seqlen = seqlen
        return out

    @staticmethod
    def backward(ctx, dout):
        time_steps_i32, cu_seqlens, bitmap = ctx.saved_tensors
        with cuda_stage("restore_backward"):
            dy = load_ops().restore_dense_bwd_bitmap(dout.contiguous(), time_steps_i32, cu_seqlens, bitmap,
                                                     ctx.dim, ctx.seqlen)
        return dy, None, None, None, None, None, None


# the bitmap of the restore holds at most this many events per channel; up to
# it the extraction's mask gives the same bitmap
MASK_RESTORE_MAX_SEQLEN = 4095


def restore_dense_fn(y_flat, time_steps_i32, cu_seqlens, dim: int, seqlen: int, base_mask=None, expand: int = 1):
    """base_mask (optional): the mask buffer extract_events_1d(...,
    return_mask=True) returned for this stream (seqlen <= 4095)."""
    return RestoreDenseFn.apply(y_flat, time_steps_i32, cu_seqlens, dim, seqlen, base_mask, int(expand))


class EventParamsFn(torch.autograd.Function):
    """An event block's parameter transforms in one launch each way
    (spike_mamba/e_model.py:463 A = -exp(A_log); :475-476 W_B, W_C = the
    halves of W_BC; :210-230 dt_idle / dt_active = softplus(a0 / a1) + eps):
    the same values and gradients as those PyTorch ops, with one kernel and
    one autograd node instead of eight of each."""

    @staticmethod
    def forward(ctx, A_log, W_BC, a0, a1, eps: float):
        A, W_B, W_C, dt_idle, dt_active = load_ops().event_params_fwd(A_log, W_BC, a0, a1, float(eps))
        ctx.save_for_backward(A, a0, a1)
        ctx.set_materialize_grads(False)   # an output without a gradient reaches the kernel as NULL
        return A, W_B, W_C, dt_idle, dt_active

    @staticmethod
    def backward(ctx, dA, dW_B, dW_C, ddt_idle, ddt_active):
        A, a0, a1 = ctx.saved_tensors
        c = lambda t: None if t is None else t.contiguous()
        dA_log, dW_BC, da0, da1 = load_ops().event_params_bwd(A, a0, a1, c(dA), c(dW_B), c(dW_C), c(ddt_idle),
                                                              c(ddt_active))
        return dA_log, dW_BC, da0, da1, None


def event_params(A_log, W_BC, a0, a1, eps: float = 1e-6):
    """(A, W_B, W_C, dt_idle, dt_active) of one event block's parameters."""
    return EventParamsFn.apply(A_log, W_BC, a0, a1, eps)


class GatherEventsFn(torch.autograd.Function):
    """u_flat[e] = x_conv[b, d, t] at (channel_ids[e] = b*D + d, time_steps[e])."""

    @staticmethod
    def forward(ctx, x_conv, channel_ids_i32, time_steps_i32, cu_seqlens=None):
        x_c = x_conv.contiguous()
        with cuda_stage("active_gather_forward"):
            out_x = load_ops().gather_events_fwd(x_c, channel_ids_i32, time_steps_i32)[0]
        # with the extraction's cu_seqlens the backward reads each channel's
        # rows from it instead of recovering them from channel_ids
        if cu_seqlens is not None:
            ctx.save_for_backward(channel_ids_i32, time_steps_i32, cu_seqlens)
        else:
            ctx.save_for_backward(channel_ids_i32, time_steps_i32)
        ctx.shape = x_c.shape
        return out_x

    @staticmethod
    def backward(ctx, grad_x):
        saved = ctx.saved_tensors
        channel_ids_i32, time_steps_i32 = saved[0], saved[1]
        B, D, L = ctx.shape
        with cuda_stage("gather_scatter_backward"):
            if len(saved) == 3:
                dx = load_ops().gather_events_bwd_rows(grad_x.contiguous(), time_steps_i32, saved[2], B * D, L)
            else:
                dx = load_ops().gather_events_bwd(grad_x.contiguous(), channel_ids_i32,
                                                  time_steps_i32, B * D, L)[0]
        return dx.view(B, D, L), None, None, None


class ConvEventsFn(torch.autograd.Function):
    """silu(causal depthwise conv1d(x) + bias) evaluated only at the events:
    replaces the dense ``x_conv = act(conv1d(x))[..., :L]`` of Mamba.forward
    followed by ``GatherEventsFn`` (spike_mamba/e_model.py:442-451, 404-406),
    whose result is read nowhere else.  ``weight`` is the conv1d weight
    ([D, 1, K] or [D, K]); ``cu_seqlens`` must describe the stream (events of a
    channel contiguous and time-ordered, as extraction produces them)."""

    @staticmethod
    def forward(ctx, x, weight, bias, channel_ids_i32, time_steps_i32, cu_seqlens):
        with cuda_stage("active_gather_forward"):
            u_flat = load_ops().conv_events_fwd(x, weight, bias, channel_ids_i32, time_steps_i32)[0]
        ctx.save_for_backward(x, weight, bias if bias is not None else torch.empty(0), time_steps_i32,
                              cu_seqlens)
        ctx.has_bias = bias is not None
        return u_flat

    @staticmethod
    def backward(ctx, grad_u):
        x, weight, bias, time_steps_i32, cu_seqlens = ctx.saved_tensors
        with cuda_stage("gather_scatter_backward"):
            dx, dw, db = load_ops().conv_events_bwd(x, weight, bias if ctx.has_bias else None,
                                                    time_steps_i32, cu_seqlens, grad_u.contiguous())
        dw = dw.view(weight.shape).to(weight.dtype)
        db = db.to(bias.dtype) if ctx.has_bias else None
        return dx, dw, db, None, None, None


def conv_events(x, weight, bias, channel_ids_i32, time_steps_i32, cu_seqlens):
    return ConvEventsFn.apply(x, weight, bias, channel_ids_i32, time_steps_i32, cu_seqlens)


class ExtractGatherFn(torch.autograd.Function):
    """Extraction + expansion + gather of x_conv in one fill pass: the
    forward of extract_base_events -> expand_base_events -> GatherEventsFn
    (reference spike_mamba/e_model.py:371-390, 167-193) with the same outputs;
    only x_flat is differentiable (w.r.t. x_conv), and its backward is the
    gather backward from the stream's rows."""

    @staticmethod
    def forward(ctx, x_conv, spikes, threshold, expand, bld, max_out, keep_mask):
        x_c = x_conv.contiguous()
        # threshold: one float, or a tensor with one threshold per feature
        ft = threshold if isinstance(threshold, torch.Tensor) else None
        with cuda_stage("routing_index_extraction"):
            # the maximum count arrives on the host with the event total (one
            # synchronisation); expansion copies counts, so it is max_seqlen
            # of the expanded stream too
            res, max_seqlen = load_ops().extract_expanded_events(
                spikes, 0.0 if ft is not None else threshold, expand, bld=bld, x_conv=x_c, feature_thresholds=ft,
                keep_mask=keep_mask)
        ch, ts, kf, cu, _mx, x_flat = res[:6]
        max_out.append(int(max_seqlen))
        ctx.save_for_backward(ts, cu)
        ctx.shape = x_c.shape
        ctx.mark_non_differentiable(ch, ts, kf, cu, *res[6:])
        ctx.set_materialize_grads(False)
        # keep_mask: also the buffer holding the threshold mask (restore_dense_fn's base_mask)
        return (x_flat, ch, ts, kf, cu, res[6]) if keep_mask else (x_flat, ch, ts, kf, cu)

    @staticmethod
    def backward(ctx, grad_x, *_):
        if grad_x is None:
            return (None,) * 7
        ts, cu = ctx.saved_tensors
        B, D, L = ctx.shape
        with cuda_stage("gather_scatter_backward"):
            dx = load_ops().gather_events_bwd_rows(grad_x.contiguous(), ts, cu, B * D, L)
        return dx.view(B, D, L), None, None, None, None, None, None


def gather_events(x_conv, channel_ids_i32, time_steps_i32, cu_seqlens=None):
    """cu_seqlens (optional): the stream's channel offsets when it is in
    extraction order, as extraction returns it."""
    return GatherEventsFn.apply(x_conv, channel_ids_i32, time_steps_i32, cu_seqlens)


def extract_events_base(base_input, x_conv, threshold: float, expand: int):
    """Extraction from the (B, d_model, L) layout extract_base_events takes
    (what Mamba.extract_events_1d builds by transposing hidden_states), then
    expansion and the gather of x_conv (B, D, L).

    Returns (channel_ids, time_steps, k_flat, cu_seqlens, max_seqlen, x_conv_flat).
    """
    # extraction, expansion and the gather of x_conv in one fill pass (the
    # base stream is never written)
    mx = []
    x_flat, ch, ts, kf, cu = ExtractGatherFn.apply(x_conv, base_input.contiguous(), float(threshold), int(expand),
                                                   False, mx, False)
    return ch, ts, kf, cu, mx[0], x_flat


def extract_events_1d(hidden_states, x_conv, threshold, expand: int, return_mask: bool = False):
    """Threshold (B, L, d_model) spikes into the expanded event stream and
    gather x_conv (B, D, L) at the events, like Mamba.extract_events_1d.
    `threshold` is a float as in the reference, or a contiguous float32
    (d_model,) tensor on the spikes' device: feature j fires above
    threshold[j].

    Returns (channel_ids, time_steps, k_flat, cu_seqlens, max_seqlen, x_conv_flat), and with
    return_mask=True also the buffer holding the threshold mask (for
    restore_dense_fn's base_mask).
    """
    # straight from the (B, L, d_model) layout (the reference first makes a
    # transposed (B, d_model, L) copy, e_model.py:376); extraction, expansion
    # and the gather of x_conv in one fill pass, the maximum count back with
    # the event total (one synchronisation, no .item())
    mx = []
    thr = threshold if isinstance(threshold, torch.Tensor) else float(threshold)
    outs = ExtractGatherFn.apply(x_conv, hidden_states.contiguous(), thr, int(expand), True, mx, bool(return_mask))
    x_flat, ch, ts, kf, cu = outs[:5]
    if return_mask:
        return ch, ts, kf, cu, mx[0], x_flat, outs[5]
    return ch, ts, kf, cu, mx[0], x_flat


class EventDecoder:
    """The event path one token at a time, in place of Mamba.step
    (reference spike_mamba/e_model.py:508-568, which reads self.pw_B /
    self.pw_C that Mamba does not define).  Each step runs extraction's
    compare on the token's spikes, the depthwise scan update of the channels
    that fire and the restore's hold, so decoding a sequence gives exactly the
    outputs extract_events_* -> selective_scan_flat_ch_fn (depthwise) ->
    restore_dense_fn give for it.  With kernel_size > 0 the token's x is the
    conv input and passes the causal depthwise conv + SiLU first (the
    conv_state of e_model.py:512-518, kept here).

    State per channel (B*D of them): eta [B*D, N] (normalised scan state),
    counters [B*D, 2] (tokens since the last event, events so far), held
    [B*D] (latest output), conv_state [B, D, K]."""

    def __init__(self, batch: int, dim: int, dstate: int, device, dtype=torch.float32, kernel_size: int = 0):
        nc = batch * dim
        self.eta = torch.zeros(nc, dstate, dtype=torch.float32, device=device)
        self.counters = torch.zeros(nc, 2, dtype=torch.int32, device=device)
        self.held = torch.zeros(nc, dtype=torch.float32, device=device)
        self.conv_state = (torch.zeros(batch, dim, kernel_size, dtype=dtype, device=device)
                           if kernel_size > 0 else None)

    def step(self, x, spikes, threshold: float, dt_idle, dt_active, A, W_B, W_C, D=None,
             conv_weight=None, conv_bias=None):
        """x [B, D] (u, or the conv input with a conv state), spikes [B, d_model]
        -> y [B, D].  W_B / W_C are the effective [D, N] weights."""
        return load_ops().event_decode_step(x.contiguous(), spikes.contiguous(), float(threshold),
                                            dt_idle.contiguous(), dt_active.contiguous(), A, W_B.contiguous(),
                                            W_C.contiguous(), D, self.eta, self.counters, self.held,
                                            self.conv_state, conv_weight, conv_bias)
