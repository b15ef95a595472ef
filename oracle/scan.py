"""Flat-channel sparse selective scan restated in numpy float64 (test oracle).

Forward follows csrc/selective_scan/selective_scan_fwd_kernel.cuh:403-728 and
the host entry selective_scan.cpp:674-884:
  delta_i = dt_idle[d]*(k_i-1) + dt_active[d]                         (:545)
  a_i,s   = exp2(clamp(delta_i*A[d,s]*log2e, -126, 126))         (:559, :650)
  h_i,s   = a_i,s*h_{i-1},s + delta_i*u_i*B_i,s                 (:651-652)
  y_i     = D[d]*u_i + sum_s h_i,s*C_i,s ; out_z = y*silu(z)   (:547, :680-711)
  x[c, chunk, 2s:2s+2] = (prod a, h) at each chunk end           (:666-677)
with B/C per mode: depthwise u*W (optionally W mixed by pw, :492-510,
:568-611), per event [N,E] (:589-591, :620-622), per feature [N,dim], or the
tiled [T,N,chunk] layout (:580-587) with the chunk of the size dispatch
(:771-785).  Backward is the exact reverse-mode derivative the reference
kernel computes (selective_scan_bwd_kernel.cuh:761-1168): the reverse
recurrence g_i = dout_i*C_i + a_{i+1}*g_{i+1}, then du, dA, dB/dC (or
dW_B/dW_C, dpw), ddt_idle/ddt_active, dD and dz, written out explicitly here
(no autograd).  Clamping is treated as identity in the derivative, as there.
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634
CHUNK_X = 2048


def ref_chunk_size(max_seqlen: int) -> int:
    for lim in (128, 256, 512, 1024):
        if max_seqlen <= lim:
            return lim
    return 2048


def n_chunks_for(max_seqlen: int) -> int:
    return max(1, (max_seqlen + CHUNK_X - 1) // CHUNK_X)


def _silu(z):
    return z / (1.0 + np.exp(-z))


class _Pad:
    """Channel-padded view of a jagged event stream."""

    def __init__(self, cu: np.ndarray, dim: int):
        cu = np.asarray(cu, dtype=np.int64)
        self.NC = cu.size - 1
        self.n = cu[1:] - cu[:-1]
        self.Lmax = int(self.n.max()) if self.NC else 0
        j = np.arange(self.Lmax)
        self.mask = j[None, :] < self.n[:, None]
        self.idx = np.where(self.mask, cu[:-1, None] + j[None, :], 0)
        self.d = np.arange(self.NC) % dim
        self.cu = cu

    def pad(self, v, fill=0.0):
        v = np.asarray(v)
        out = v[self.idx].astype(np.float64)
        out[~self.mask] = fill
        return out


def _mode(B, E, tile_offsets, is_depthwise_bc):
    if tile_offsets is not None:
        return "tiled"
    if is_depthwise_bc:
        return "depthwise"
    return "flat"


def _bc_pad(P: _Pad, W, mode, var, u_pad, toff, cs, N):
    """Per (channel, event, state) B or C values, (NC, Lmax, N)."""
    if mode == "depthwise":
        return u_pad[:, :, None] * np.asarray(W, np.float64)[P.d][:, None, :]
    if mode == "tiled":
        W = np.asarray(W, np.float64)
        j = np.arange(P.Lmax)
        tile = np.asarray(toff, np.int64)[:, None] + j[None, :] // cs
        pos = j % cs
        tile = np.where(P.mask, tile, 0)
        out = W[tile, :, pos[None, :]]  # (NC, Lmax, N)
        out[~P.mask] = 0.0
        return out
    W = np.asarray(W, np.float64)
    if var:
        out = W[:, P.idx].transpose(1, 2, 0).copy()  # (NC, Lmax, N)
        out[~P.mask] = 0.0
        return out
    return np.broadcast_to(W.T[P.d][:, None, :], (P.NC, P.Lmax, N)).copy()


def _prepare(u, k, cu, max_seqlen, dt_idle, dt_active, A, B, C, tile_offsets, is_depthwise_bc,
             pw_B, pw_C, fp32_decay=False):
    u = np.asarray(u)
    E = u.size
    A = np.asarray(A, np.float64)
    dim, N = A.shape
    P = _Pad(cu, dim)
    mode = _mode(B, E, tile_offsets, is_depthwise_bc)
    B = np.asarray(B, np.float64)
    C = np.asarray(C, np.float64)
    if mode == "depthwise" and pw_B is not None:
        B = np.asarray(pw_B, np.float64) @ B
        C = np.asarray(pw_C, np.float64) @ C
    b_var = mode == "tiled" or (mode == "flat" and B.shape[1] == E)
    c_var = mode == "tiled" or (mode == "flat" and C.shape[1] == E)
    cs = ref_chunk_size(max_seqlen)
    u_pad = P.pad(u)
    k_pad = P.pad(k, fill=1.0)
    dti = np.asarray(dt_idle, np.float64)[P.d][:, None]
    dta = np.asarray(dt_active, np.float64)[P.d][:, None]
    delta = dti * (k_pad - 1.0) + dta
    delta[~P.mask] = 0.0
    Ad = A[P.d]  # (NC, N)
    if fp32_decay:
        # The decays exactly as the reference kernel forms them in fp32
        # (selective_scan_fwd_kernel.cuh:545, :559, :650-651): delta by one fused
        # multiply-add, A*log2e rounded to fp32, their product rounded, clamped,
        # exp2 rounded to fp32.  With near-uniform gaps and long memory (a ~ 1)
        # every event reuses the same rounded decay, so its rounding compounds
        # over ~1/(1-a) events; this mode reproduces that arithmetic.
        delta = delta.astype(np.float32).astype(np.float64)
        A2 = (Ad * LOG2E).astype(np.float32).astype(np.float64)
        x = (delta[:, :, None] * A2[:, None, :]).astype(np.float32).astype(np.float64)
        a = np.exp2(np.clip(x, -126.0, 126.0)).astype(np.float32).astype(np.float64)
    else:
        a = np.exp2(np.clip(delta[:, :, None] * Ad[:, None, :] * LOG2E, -126.0, 126.0))
    a[~P.mask] = 1.0
    Bp = _bc_pad(P, B, mode, b_var, u_pad, tile_offsets, cs, N)
    Cp = _bc_pad(P, C, mode, c_var, u_pad, tile_offsets, cs, N)
    return dict(P=P, mode=mode, B=B, C=C, b_var=b_var, c_var=c_var, cs=cs, u=u_pad, k=k_pad,
                delta=delta, a=a, Bp=Bp, Cp=Cp, Ad=Ad, N=N, dim=dim, E=E)


def _forward(S):
    P, a = S["P"], S["a"]
    b = S["delta"][:, :, None] * S["u"][:, :, None] * S["Bp"]
    h = np.zeros((P.NC, S["N"]))
    hs = np.zeros((P.NC, P.Lmax, S["N"]))
    for j in range(P.Lmax):
        h = a[:, j] * h + b[:, j]
        hs[:, j] = h
    return hs


def scan_fwd(u, k, cu, max_seqlen, dt_idle, dt_active, A, B, C, D=None, z=None,
             tile_offsets=None, is_depthwise_bc=False, pw_B=None, pw_C=None, fp32_decay=False):
    """Returns (out[E], x[NC, n_chunks, 2N], out_z or None), float64."""
    S = _prepare(u, k, cu, max_seqlen, dt_idle, dt_active, A, B, C, tile_offsets,
                 is_depthwise_bc, pw_B, pw_C, fp32_decay)
    P, N = S["P"], S["N"]
    hs = _forward(S)
    y = (hs * S["Cp"]).sum(-1)
    if D is not None:
        y = y + np.asarray(D, np.float64)[P.d][:, None] * S["u"]
    out = np.zeros(S["E"])
    out[P.idx[P.mask]] = y[P.mask]
    nck = n_chunks_for(max_seqlen)
    x = np.zeros((P.NC, nck, 2 * N))
    cum = np.cumprod(S["a"], axis=1)
    for c in range(P.NC):
        n = int(P.n[c])
        for j in range(n):
            if (j + 1) % CHUNK_X == 0 or j == n - 1:
                ck = j // CHUNK_X
                if ck < nck:
                    x[c, ck, 0::2] = cum[c, j]
                    x[c, ck, 1::2] = hs[c, j]
    out_z = None
    if z is not None:
        out_z = out * _silu(np.asarray(z, np.float64))
    return out, x, out_z


def scan_bwd(u, k, cu, max_seqlen, dt_idle, dt_active, A, B, C, dout, D=None, z=None, out=None,
             tile_offsets=None, is_depthwise_bc=False, pw_B=None, pw_C=None, fp32_decay=False):
    """Gradients in the reference's return order:
    [du, dA, dB (or dW_B), dC (or dW_C), ddt_idle, ddt_active, (dD), (dz), (dpw_B, dpw_C)]."""
    S = _prepare(u, k, cu, max_seqlen, dt_idle, dt_active, A, B, C, tile_offsets,
                 is_depthwise_bc, pw_B, pw_C, fp32_decay)
    P, N, dim, E = S["P"], S["N"], S["dim"], S["E"]
    mode = S["mode"]
    hs = _forward(S)
    dout = np.asarray(dout, np.float64)
    dz = None
    if z is not None:
        zz = np.asarray(z, np.float64)
        sg = 1.0 / (1.0 + np.exp(-zz))
        dz = dout * np.asarray(out, np.float64) * sg * (1.0 + zz * (1.0 - sg))
        dout = dout * zz * sg
    dpad = P.pad(dout)
    a, delta, uu, Bp, Cp, Ad = S["a"], S["delta"], S["u"], S["Bp"], S["Cp"], S["Ad"]
    g = np.zeros((P.NC, N))
    a_next = np.ones((P.NC, N))
    dB_ev = np.zeros_like(Bp)
    dC_ev = np.zeros_like(Cp)
    du = np.zeros((P.NC, P.Lmax))
    ddel = np.zeros((P.NC, P.Lmax))
    dA_c = np.zeros((P.NC, N))
    for j in range(P.Lmax - 1, -1, -1):
        m = P.mask[:, j][:, None]
        g = np.where(m, dpad[:, j, None] * Cp[:, j] + a_next * g, 0.0)
        a_next = np.where(m, a[:, j], 1.0)
        hprev = hs[:, j - 1] if j > 0 else np.zeros((P.NC, N))
        ah = a[:, j] * hprev
        dB_ev[:, j] = g * delta[:, j, None] * uu[:, j, None]
        dC_ev[:, j] = dpad[:, j, None] * hs[:, j]
        du[:, j] = (g * Bp[:, j]).sum(-1) * delta[:, j]
        ddel[:, j] = (g * (uu[:, j, None] * Bp[:, j] + Ad * ah)).sum(-1)
        dA_c += g * delta[:, j, None] * ah
    Dv = np.zeros(dim) if D is None else np.asarray(D, np.float64)
    du = du + Dv[P.d][:, None] * dpad
    grads_B = grads_C = None
    dpw_B = dpw_C = None
    if mode == "depthwise":
        We_B, We_C = S["B"], S["C"]  # effective (mixed) weights
        du = du + (dB_ev * We_B[P.d][:, None, :]).sum(-1) + (dC_ev * We_C[P.d][:, None, :]).sum(-1)
        dWe_B = np.zeros((dim, N))
        dWe_C = np.zeros((dim, N))
        np.add.at(dWe_B, P.d, (dB_ev * uu[:, :, None]).sum(1))
        np.add.at(dWe_C, P.d, (dC_ev * uu[:, :, None]).sum(1))
        if pw_B is not None:
            pB = np.asarray(pw_B, np.float64)
            pC = np.asarray(pw_C, np.float64)
            W_B0 = np.asarray(B, np.float64)
            W_C0 = np.asarray(C, np.float64)
            grads_B = pB.T @ dWe_B
            grads_C = pC.T @ dWe_C
            dpw_B = dWe_B @ W_B0.T
            dpw_C = dWe_C @ W_C0.T
        else:
            grads_B, grads_C = dWe_B, dWe_C
    else:
        def scatter(ev, W, var):
            W = np.asarray(W, np.float64)
            res = np.zeros_like(W)
            if mode == "tiled":
                j = np.arange(P.Lmax)
                tile = np.asarray(tile_offsets, np.int64)[:, None] + j[None, :] // S["cs"]
                pos = np.broadcast_to(j % S["cs"], tile.shape)
                for s in range(N):
                    np.add.at(res, (tile[P.mask], s, pos[P.mask]), ev[:, :, s][P.mask])
            elif var:
                for s in range(N):
                    res[s, P.idx[P.mask]] = ev[:, :, s][P.mask]
            else:
                for s in range(N):
                    np.add.at(res[s], P.d, ev[:, :, s].sum(1))
            return res
        grads_B = scatter(dB_ev, B, S["b_var"])
        grads_C = scatter(dC_ev, C, S["c_var"])
    dA = np.zeros((dim, N))
    np.add.at(dA, P.d, dA_c)
    ddt_idle = np.zeros(dim)
    ddt_active = np.zeros(dim)
    np.add.at(ddt_idle, P.d, (ddel * (S["k"] - 1.0) * P.mask).sum(1))
    np.add.at(ddt_active, P.d, (ddel * P.mask).sum(1))
    du_flat = np.zeros(E)
    du_flat[P.idx[P.mask]] = du[P.mask]
    res = [du_flat, dA, grads_B, grads_C, ddt_idle, ddt_active]
    if D is not None:
        dD = np.zeros(dim)
        np.add.at(dD, P.d, (dpad * uu).sum(1))
        res.append(dD)
    if z is not None:
        res.append(dz)
    if dpw_B is not None:
        res += [dpw_B, dpw_C]
    return res
