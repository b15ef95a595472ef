"""Dense selective scan (Mamba's S6), restated in float64 numpy — TEST
INFRASTRUCTURE ONLY (the GPU parity checker of bcm_s6_fwd / bcm_s6_bwd).

Forward: the reference's ``selective_scan_ref``
(spike_mamba/selective_scan_interface.py:708-774) with the CUDA binding's
details (csrc/selective_scan/selective_scan.cpp:403-497,
selective_scan_fwd_kernel.cuh:164-276): delta' = delta + delta_bias, then
softplus (identity above 20); decay exp2(clamp(delta'*A*log2(e), +-126));
h = decay*h + b'*delta'*u with b' = B for variable B, 1 for fixed B (fixed B
then multiplies the output weight); y = sum_s C'_s h_s + D*u; out_z =
y*silu(z); chunk states x[b, d, c] = (product of the decays since position 0,
h) after every 2048 positions and after the last one.
Backward: the explicit reverse-mode derivative of that forward (the gradients
selective_scan_bwd_kernel.cuh:31-500 computes): dh_t = C'_t dy_t +
a_{t+1} dh_{t+1}; dA = sum delta' dh h_{t-1} a_t; ddelta' = sum_s (dh h_{t-1}
a_t A + dh b' u); du = sum_s dh b' delta' + D dy; dB, dC summed over the
channels of a group (variable) or over batch and positions (fixed);
ddelta_bias = sum of ddelta; dz from the ungated output.
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
CHUNK = 2048


def _prep(u, delta, A, B, C, delta_bias, delta_softplus):
    u = np.asarray(u, np.float64)
    raw = np.asarray(delta, np.float64)
    if delta_bias is not None:
        raw = raw + np.asarray(delta_bias, np.float64)[None, :, None]
    dl = np.where(raw <= 20.0, np.log1p(np.exp(np.minimum(raw, 20.0))), raw) if delta_softplus else raw
    A = np.asarray(A, np.float64)
    var_b, var_c = np.ndim(B) >= 3, np.ndim(C) >= 3
    bsz, dim, L = u.shape

    def per_channel(X):  # (b, g, n, l) -> (b, d, n, l)
        X = np.asarray(X, np.float64)
        return np.repeat(X, dim // X.shape[1], axis=1)

    Bv = per_channel(B) if var_b else np.asarray(B, np.float64)
    Cv = per_channel(C) if var_c else np.asarray(C, np.float64)
    return u, raw, dl, A, Bv, Cv, var_b, var_c


def _decay(dl_t, A):  # (b, d), (d, n) -> (b, d, n)
    e = np.clip(dl_t[:, :, None] * A[None] * LOG2E, -126.0, 126.0)
    return np.exp2(e)


def _weights(Bv, Cv, var_b, var_c, t):
    """b' (b, d, n) or 1, and the output weight C' (b, d, n) at position t."""
    bb = Bv[:, :, :, t] if var_b else 1.0
    cw = Cv[:, :, :, t] if var_c else Cv[None]
    if not var_b:
        cw = cw * Bv[None]
    return bb, cw


def s6_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    """Returns (out, x, out_z or None, hs) with hs the state after every
    position (b, d, l, n)."""
    u, raw, dl, A, Bv, Cv, var_b, var_c = _prep(u, delta, A, B, C, delta_bias, delta_softplus)
    bsz, dim, L = u.shape
    N = A.shape[1]
    nch = (L + CHUNK - 1) // CHUNK
    h = np.zeros((bsz, dim, N))
    P = np.ones((bsz, dim, N))
    x = np.zeros((bsz, dim, nch, 2 * N))
    y = np.zeros((bsz, dim, L))
    hs = np.zeros((bsz, dim, L, N))
    for t in range(L):
        a = _decay(dl[:, :, t], A)
        bb, cw = _weights(Bv, Cv, var_b, var_c, t)
        h = a * h + bb * (dl[:, :, t] * u[:, :, t])[:, :, None]
        P = P * a
        hs[:, :, t] = h
        y[:, :, t] = (cw * h).sum(-1)
        if (t + 1) % CHUNK == 0 or t + 1 == L:
            x[:, :, t // CHUNK, 0::2] = P
            x[:, :, t // CHUNK, 1::2] = h
    out = y if D is None else y + u * np.asarray(D, np.float64)[None, :, None]
    out_z = None
    if z is not None:
        zz = np.asarray(z, np.float64)
        out_z = out * zz / (1.0 + np.exp(-zz))
    return out, x, out_z, hs


def s6_bwd(u, delta, A, B, C, dout, D=None, z=None, delta_bias=None, delta_softplus=False):
    """Returns dict du, ddelta, dA, dB, dC, dD, ddelta_bias, dz (None where
    the input is absent)."""
    out, _x, _oz, hs = s6_fwd(u, delta, A, B, C, D, z, delta_bias, delta_softplus)
    u, raw, dl, A, Bv, Cv, var_b, var_c = _prep(u, delta, A, B, C, delta_bias, delta_softplus)
    bsz, dim, L = u.shape
    N = A.shape[1]
    dy = np.asarray(dout, np.float64).copy()
    dz = None
    if z is not None:
        zz = np.asarray(z, np.float64)
        sg = 1.0 / (1.0 + np.exp(-zz))
        dz = dy * out * sg * (1.0 + zz * (1.0 - sg))
        dy = dy * zz * sg
    du = np.zeros_like(u)
    ddl = np.zeros_like(u)
    dA = np.zeros_like(A)
    dBv = np.zeros((bsz, dim, N, L)) if var_b else np.zeros((dim, N))
    dCv = np.zeros((bsz, dim, N, L)) if var_c else np.zeros((dim, N))
    dh = np.zeros((bsz, dim, N))
    a_next = np.zeros((bsz, dim, N))
    Bfix = 1.0 if var_b else Bv[None]
    for t in range(L - 1, -1, -1):
        a = _decay(dl[:, :, t], A)
        bb, cw = _weights(Bv, Cv, var_b, var_c, t)
        hp = hs[:, :, t - 1] if t > 0 else np.zeros((bsz, dim, N))
        ht = hs[:, :, t]
        dh = a_next * dh + cw * dy[:, :, t][:, :, None]
        pr = dh * hp * a
        dA += (pr * dl[:, :, t][:, :, None]).sum(0)
        ddl[:, :, t] = (pr * A[None]).sum(-1) + (dh * bb).sum(-1) * u[:, :, t]
        du[:, :, t] = (dh * bb).sum(-1) * dl[:, :, t]
        cv = Cv[:, :, :, t] if var_c else Cv[None]
        if var_b:
            dBv[:, :, :, t] = dh * (dl[:, :, t] * u[:, :, t])[:, :, None]
        else:
            dBv += (dy[:, :, t][:, :, None] * cv * ht).sum(0)
        if var_c:
            dCv[:, :, :, t] = dy[:, :, t][:, :, None] * ht * Bfix
        else:
            dCv += (dy[:, :, t][:, :, None] * ht * Bfix).sum(0)
        a_next = a
    dD = None
    if D is not None:
        du = du + np.asarray(D, np.float64)[None, :, None] * dy
        dD = (dy * u).sum((0, 2))
    if delta_softplus:
        fac = np.where(raw <= 20.0, 1.0 / (1.0 + np.exp(-np.minimum(raw, 20.0))), 1.0)
        ddelta = ddl * fac
    else:
        ddelta = ddl
    ddelta_bias = ddelta.sum((0, 2)) if delta_bias is not None else None

    def group_sum(X, like):  # (b, d, n, l) -> (b, g, n, l)
        g = np.shape(like)[1]
        return X.reshape(bsz, g, dim // g, N, L).sum(2)

    dB = group_sum(dBv, B) if var_b else dBv
    dC = group_sum(dCv, C) if var_c else dCv
    return dict(du=du, ddelta=ddelta, dA=dA, dB=dB, dC=dC, dD=dD, ddelta_bias=ddelta_bias, dz=dz)
