"""Event-path decode restated in numpy float64 (test oracle).

The reference's Mamba.step (spike_mamba/e_model.py:508-568) cannot run as
written (it reads self.pw_B / self.pw_C, which Mamba does not define), so
decode is specified as the training path evaluated one token at a time:
extraction's compare (`spikes > threshold`, extract_events_cuda.cu:117-179)
on the expanded channel (repeat_interleave, e_model.py:543-546), the
depthwise flat-channel scan update of one event (oracle/scan.py, reference
selective_scan_fwd_kernel.cuh:545-652: delta = dt_idle*(k-1) + dt_active,
a = exp2(clamp(delta*A*log2e, +-126)), h = a*h + delta*u*B with
B = u*W_B, y = D*u + sum h*C with C = u*W_C) and the restore's hold of the
latest addressable event (oracle/restore.py: the first 4095 events), plus
the optional conv-state update of e_model.py:512-518 (roll, depthwise conv,
SiLU).  `decode_sequence` runs it over a whole sequence; the tests compare it
with extraction -> scan -> restore on the same inputs.
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
RESTORE_CAP = 4095


class DecodeState:
    """Per-channel state of B*D channels: h [NC, N], tokens since the last
    event, events so far, held output, optional conv window [NC, K]."""

    def __init__(self, n_channels: int, dstate: int, kernel_size: int = 0):
        self.h = np.zeros((n_channels, dstate))
        self.gap = np.zeros(n_channels, dtype=np.int64)
        self.n_ev = np.zeros(n_channels, dtype=np.int64)
        self.held = np.zeros(n_channels)
        self.conv = np.zeros((n_channels, kernel_size)) if kernel_size else None


def decode_step(st: DecodeState, x, spikes, threshold, dt_idle, dt_active, A, W_B, W_C, D=None,
                conv_weight=None, conv_bias=None):
    """x [B, dim], spikes [B, d_model] -> y [B, dim]; st is updated."""
    x = np.asarray(x, dtype=np.float64)
    B, dim = x.shape
    d_model = np.asarray(spikes).shape[1]
    expand = dim // d_model
    d = np.tile(np.arange(dim), B)
    u = x.reshape(-1)
    if st.conv is not None:
        st.conv = np.roll(st.conv, -1, axis=1)
        st.conv[:, -1] = u
        pre = np.sum(st.conv * np.asarray(conv_weight, np.float64)[d], axis=1)
        if conv_bias is not None:
            pre = pre + np.asarray(conv_bias, np.float64)[d]
        u = pre / (1.0 + np.exp(-pre))
    s = np.repeat(np.asarray(spikes, np.float32), expand, axis=1).reshape(-1)
    fire = s > np.float32(threshold)
    k = st.gap + 1
    delta = np.asarray(dt_idle, np.float64)[d] * (k - 1) + np.asarray(dt_active, np.float64)[d]
    a = np.exp2(np.clip(delta[:, None] * np.asarray(A, np.float64)[d] * LOG2E, -126.0, 126.0))
    Wb = np.asarray(W_B, np.float64)[d]
    Wc = np.asarray(W_C, np.float64)[d]
    h_new = a * st.h + (delta * u * u)[:, None] * Wb
    y = np.sum(h_new * (u[:, None] * Wc), axis=1)
    if D is not None:
        y = y + np.asarray(D, np.float64)[d] * u
    st.h = np.where(fire[:, None], h_new, st.h)
    st.gap = np.where(fire, 0, k)
    st.n_ev = st.n_ev + fire
    hold = fire & (st.n_ev <= RESTORE_CAP)
    st.held = np.where(hold, y, st.held)
    return st.held.reshape(B, dim).copy()


def decode_sequence(xs, spikes, threshold, dt_idle, dt_active, A, W_B, W_C, D=None, conv_weight=None,
                    conv_bias=None):
    """xs [B, dim, L], spikes [B, d_model, L] -> y [B, L, dim] (the restore layout)."""
    xs = np.asarray(xs)
    B, dim, L = xs.shape
    K = 0 if conv_weight is None else np.asarray(conv_weight).shape[-1]
    st = DecodeState(B * dim, np.asarray(A).shape[1], K)
    out = np.zeros((B, L, dim))
    for t in range(L):
        out[:, t, :] = decode_step(st, xs[:, :, t], np.asarray(spikes)[:, :, t], threshold, dt_idle, dt_active,
                                   A, W_B, W_C, D, conv_weight, conv_bias)
    return out
