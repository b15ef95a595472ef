"""Shared comparison helpers for the parity tests.

Tolerance convention (fp32 paths): elementwise
    |x - ref| <= tol * |ref| + tol * max|ref|
with tol = 1e-5 for fp32 and 2e-2 for bf16/fp16 event values, ref the float64
oracle.  Integer streams and index maps are compared bit-exactly.
"""
from __future__ import annotations

import numpy as np
import torch

TOL_F32 = 1e-5
TOL_16 = 2e-2


def to_np(x):
    if isinstance(x, torch.Tensor):
        x = x.detach()
        if x.dtype in (torch.bfloat16, torch.float16):
            x = x.float()
        return x.cpu().numpy()
    return np.asarray(x)


def assert_exact(a, b, what=""):
    a, b = to_np(a), to_np(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if a.size:
        bad = np.flatnonzero(a.reshape(-1) != b.reshape(-1))
        assert bad.size == 0, f"{what}: {bad.size} mismatches, first at {bad[:5]}: {a.reshape(-1)[bad[:5]]} vs {b.reshape(-1)[bad[:5]]}"


def assert_close(a, b, tol=TOL_F32, what=""):
    a = to_np(a).astype(np.float64)
    b = to_np(b).astype(np.float64)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if a.size == 0:
        return
    scale = np.max(np.abs(b))
    err = np.abs(a - b)
    lim = tol * np.abs(b) + tol * scale
    worst = np.argmax(err - lim)
    assert np.all(err <= lim), (
        f"{what}: max err {err.reshape(-1)[worst]:.3e} at {worst} (ref {b.reshape(-1)[worst]:.4e}, "
        f"got {a.reshape(-1)[worst]:.4e}, scale {scale:.3e}, tol {tol})")
