"""CPU restatement (float64) of the causal depthwise convolution + SiLU that
feeds the event gather, evaluated at the events.  Test infrastructure only.

Reference semantics: Mamba.forward computes x_conv = act(conv1d(x))[..., :L]
with nn.Conv1d(groups=D, kernel_size=K, padding=K-1) and SiLU
(spike_mamba/e_model.py:306-313, 442-451; causal_conv1d_fn when installed,
the same function), then gathers x_conv at the events (e_model.py:167-193,
404-406).  So u[e] = silu(bias[d] + sum_j w[d, j] * x[b, d, t_e - K + 1 + j])
with x = 0 before position 0.
"""
from __future__ import annotations

import numpy as np


def _silu(v):
    return v / (1.0 + np.exp(-v))


def _pre(x, w, bias, ch, t):
    B, D, L = x.shape
    K = w.shape[1]
    x2 = np.asarray(x, np.float64).reshape(B * D, L)
    w = np.asarray(w, np.float64)
    ch = np.asarray(ch, np.int64)
    t = np.asarray(t, np.int64)
    d = ch % D
    pre = np.zeros(ch.size) if bias is None else np.asarray(bias, np.float64)[d].copy()
    for j in range(K):
        tt = t - (K - 1) + j
        ok = tt >= 0
        vals = np.zeros(ch.size)
        vals[ok] = x2[ch[ok], tt[ok]]
        pre += w[d, j] * vals
    return pre


def conv_events_fwd(x, w, bias, ch, t):
    """u[E] (float64)."""
    return _silu(_pre(x, w, bias, ch, t))


def conv_events_bwd(x, w, bias, ch, t, g):
    """(dx[B, D, L], dw[D, K], dbias[D]) for upstream gradient g[E] (float64)."""
    B, D, L = x.shape
    K = w.shape[1]
    pre = _pre(x, w, bias, ch, t)
    s = 1.0 / (1.0 + np.exp(-pre))
    dpre = np.asarray(g, np.float64) * s * (1.0 + pre * (1.0 - s))
    x2 = np.asarray(x, np.float64).reshape(B * D, L)
    w = np.asarray(w, np.float64)
    ch = np.asarray(ch, np.int64)
    t = np.asarray(t, np.int64)
    d = ch % D
    dx = np.zeros((B * D, L))
    dw = np.zeros((D, K))
    for j in range(K):
        tt = t - (K - 1) + j
        ok = tt >= 0
        np.add.at(dx, (ch[ok], tt[ok]), w[d[ok], j] * dpre[ok])
        np.add.at(dw[:, j], d[ok], dpre[ok] * x2[ch[ok], tt[ok]])
    db = np.zeros(D)
    np.add.at(db, d, dpre)
    return dx.reshape(B, D, L), dw, db
