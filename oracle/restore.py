"""Zero-order-hold restore restated in numpy (test oracle).

Follows csrc/r_nodecay of the reference:
  * forward  restore_dense_fwd_kernel.cuh:86-111 — upper_bound(ts, t) - 1 with
    the 12-step search (s = 2048 ... 1), which can reach lo = 4095 at most, so
    e* = min(#events <= t, 4095) - 1; positions before the first event stay 0;
    output layout (B, L, D); host entry restore_dense.cpp:41-123.
  * backward restore_dense_bwd_kernel.cuh:94-111 — dy[e*(t)] += dout[b, t, d],
    fp32 result (restore_dense.cpp:175-176).
"""
from __future__ import annotations

import numpy as np

SEARCH_CAP = 4095


def hold_index(ts_c: np.ndarray, L: int) -> np.ndarray:
    """Local event index held at each t in [0, L) (-1 before the first)."""
    cnt = np.searchsorted(ts_c, np.arange(L), side="right")
    return np.minimum(cnt, SEARCH_CAP) - 1


def restore_dense_fwd(y, ts, cu, dim: int, seqlen: int, out_dtype=None):
    NC = cu.size - 1
    B = NC // dim
    out = np.zeros((B, seqlen, dim), dtype=np.float64)
    y64 = np.asarray(y, dtype=np.float64)
    for ch in range(NC):
        s, e = int(cu[ch]), int(cu[ch + 1])
        if e == s:
            continue
        idx = hold_index(ts[s:e], seqlen)
        ok = idx >= 0
        b, d = divmod(ch, dim)
        out[b, ok, d] = y64[s + idx[ok]]
    return out if out_dtype is None else out.astype(out_dtype)


def restore_dense_bwd(dout, ts, cu, dim: int, seqlen: int):
    NC = cu.size - 1
    E = ts.size
    dy = np.zeros(E, dtype=np.float64)
    d64 = np.asarray(dout, dtype=np.float64)
    for ch in range(NC):
        s, e = int(cu[ch]), int(cu[ch + 1])
        if e == s:
            continue
        idx = hold_index(ts[s:e], seqlen)
        ok = idx >= 0
        b, d = divmod(ch, dim)
        np.add.at(dy, s + idx[ok], d64[b, ok, d])
    return dy


def event_bitmap(ts, cu, dim: int, seqlen: int) -> np.ndarray:
    """uint32 [B, ceil(L/32), dim]: bit t%32 of word [b, t//32, d] is set where
    channel b*dim+d has an addressable event (one of its first SEARCH_CAP) at
    t in [0, L).  The product's restore forward writes this for its backward;
    the reference has no such array (it searches the times again)."""
    NC = cu.size - 1
    B = NC // dim
    nw = (seqlen + 31) // 32
    bm = np.zeros((B, nw, dim), dtype=np.uint64)
    for ch in range(NC):
        s, e = int(cu[ch]), int(cu[ch + 1])
        t = np.asarray(ts[s:min(e, s + SEARCH_CAP)], dtype=np.int64)
        t = t[(t >= 0) & (t < seqlen)]
        b, d = divmod(ch, dim)
        np.bitwise_or.at(bm[b, :, d], t >> 5, np.left_shift(np.uint64(1), (t & 31).astype(np.uint64)))
    return bm.astype(np.uint32)
