"""Event extraction / expansion / gather restated in numpy (test oracle).

Follows csrc/extract/extract_events_cuda.cu of the reference:
  * extract_base_events  — count_base_kernel :192-208 (strict float(x) > thr),
    fill_base_kernel :226-312 (ascending t, k = t - t_prev, first k = t + 1),
    host entry :324-418 (E == 0 shapes :381-385, max = counts.max()).
  * expand_base_events   — build_logical_cu_kernel :449-467,
    expand_events_direct_kernel :482-509, slice-diff max :596-600, E == 0 :551-556.
  * gather_events_fwd/bwd — :629-662, :670-754.
  * extract_events (legacy bool mask) — :38-179.
"""
from __future__ import annotations

import numpy as np

I32 = np.int32


def _k_flat(ch: np.ndarray, t: np.ndarray) -> np.ndarray:
    k = np.empty_like(t)
    if t.size == 0:
        return k
    start = np.ones(t.size, dtype=bool)
    start[1:] = ch[1:] != ch[:-1]
    k[start] = t[start] + 1
    k[~start] = t[~start] - t[np.flatnonzero(~start) - 1]
    return k


def extract_base_events(base_input: np.ndarray, threshold):
    """base_input (B, d_model, L) -> (ch, t, k, cu[NCb+1], counts[NCb], max).
    `threshold`: a scalar (the reference's API), or d_model values, one per
    feature (the per-feature form of bcm_extract_expanded_ft)."""
    B, dm, L = base_input.shape
    x = np.asarray(base_input, dtype=np.float32).reshape(B * dm, L)
    thr = np.asarray(threshold, dtype=np.float32)
    mask = x > (thr if thr.ndim == 0 else np.tile(thr.reshape(dm), B)[:, None])
    counts = mask.sum(axis=1).astype(I32)
    cu = np.zeros(B * dm + 1, dtype=I32)
    np.cumsum(counts, out=cu[1:])
    ch, t = np.nonzero(mask)
    ch = ch.astype(I32)
    t = t.astype(I32)
    if ch.size == 0:
        e = np.zeros(0, I32)
        return e, e, e, cu, counts, np.zeros(1, I32)
    return ch, t, _k_flat(ch, t), cu, counts, np.array(counts.max(), dtype=I32)


def expand_base_events(bch, bt, bk, bcu, B: int, d_model: int, expand: int):
    """Replicate each base channel c into logical channels c*expand + r."""
    ncb = B * d_model
    nci = ncb * expand
    eb = bch.size
    if eb == 0:
        e = np.zeros(0, I32)
        return e, e, e, np.zeros(nci + 1, I32), np.zeros(1, I32)
    bcu = np.asarray(bcu, dtype=np.int64)
    cnt = bcu[1:ncb + 1] - bcu[:ncb]
    cu = np.empty(nci + 1, dtype=I32)
    for r in range(expand):
        cu[np.arange(ncb) * expand + r] = bcu[:ncb] * expand + r * cnt
    cu[nci] = bcu[ncb] * expand
    c = np.asarray(bch, dtype=np.int64)
    s = bcu[c]
    local = np.arange(eb) - s
    e = eb * expand
    ch = np.empty(e, I32)
    t = np.empty(e, I32)
    k = np.empty(e, I32)
    for r in range(expand):
        pos = s * expand + r * cnt[c] + local
        ch[pos] = c * expand + r
        t[pos] = bt
        k[pos] = bk
    return ch, t, k, cu, np.array(cnt.max(), dtype=I32)


def gather_events_fwd(x: np.ndarray, ch: np.ndarray, t: np.ndarray) -> np.ndarray:
    B, D, L = x.shape
    return x.reshape(B * D, L)[ch.astype(np.int64), t.astype(np.int64)]


def gather_events_bwd(g: np.ndarray, ch: np.ndarray, t: np.ndarray, NC: int, L: int) -> np.ndarray:
    dx = np.zeros((NC, L), dtype=g.dtype)
    dx[ch.astype(np.int64), t.astype(np.int64)] = g
    return dx


def extract_events(mask: np.ndarray):
    """Legacy bool mask (B, D, L) -> (ch, t, k, cu, max, head_flags)."""
    ch, t, k, cu, counts, mx = extract_base_events(mask.astype(np.float32), 0.5)
    if ch.size == 0:
        e = np.zeros(0, I32)
        return e, e, e, cu, np.zeros(1, I32), e
    hf = np.zeros(ch.size, I32)
    hf[cu[:-1][counts > 0]] = 1
    return ch, t, k, cu, mx, hf
