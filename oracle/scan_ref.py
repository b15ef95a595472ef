"""The reference's pure-PyTorch scan path, restated — CPU baseline and a second
scan oracle (TEST INFRASTRUCTURE ONLY).

``selective_scan_ref`` restates spike_mamba/selective_scan_interface.py:708-774
(the dense sequential Mamba reference: deltaA = exp(delta*A), deltaB_u =
delta*B*u, x = deltaA*x + deltaB_u, y = <x, C>, + D*u, * silu(z)) for the
real-A case.  ``compact`` builds the event-compacted, zero-padded tensors on
which that dense scan reproduces the flat per-channel event scan: channel
(b, d) packs its events into slots j < Lmax with delta = dt_idle*(k-1) +
dt_active and, in depthwise mode, B = u*W_B[d], C = u*W_C[d] as 4-D
(B, G=D, N, Lmax) tensors; padding slots carry u = 0 and delta = 0, i.e. a
decay of exp(0) = 1 and zero input, so the state is frozen.  The only
difference from the CUDA scan is exp versus exp2(clamp(., +-126)), below 1e-30.
"""
from __future__ import annotations

import numpy as np
import torch


def selective_scan_ref(u, delta, A, B, C, D=None, z=None):
    """u, delta (b, d, l); A (d, n); B, C (d, n) | (b, n, l) | (b, g, n, l)."""
    dtype_in = u.dtype
    u = u.float()
    delta = delta.float()
    bsz, dim, L = u.shape
    n = A.shape[1]
    var_b, var_c = B.dim() >= 3, C.dim() >= 3
    B = B.float()
    C = C.float()
    if var_b and B.dim() == 4:
        B = B.repeat_interleave(dim // B.shape[1], dim=1)
    if var_c and C.dim() == 4:
        C = C.repeat_interleave(dim // C.shape[1], dim=1)
    dA = torch.exp(delta.unsqueeze(-1) * A.unsqueeze(1))             # (b, d, l, n)
    if not var_b:
        dBu = (delta * u).unsqueeze(-1) * B.unsqueeze(1)             # B (d, n)
    elif B.dim() == 3:
        dBu = (delta * u).unsqueeze(-1) * B.transpose(1, 2).unsqueeze(1)
    else:
        dBu = (delta * u).unsqueeze(-1) * B.permute(0, 1, 3, 2)
    x = u.new_zeros(bsz, dim, n)
    ys = []
    for i in range(L):
        x = dA[:, :, i] * x + dBu[:, :, i]
        if not var_c:
            ys.append((x * C).sum(-1))
        elif C.dim() == 3:
            ys.append((x * C[:, :, i].unsqueeze(1)).sum(-1))
        else:
            ys.append((x * C[:, :, :, i]).sum(-1))
    y = torch.stack(ys, dim=2)
    out = y if D is None else y + u * D.unsqueeze(-1)
    if z is not None:
        out = out * torch.nn.functional.silu(z)
    return out.to(dtype_in)


def compact(u_flat, k_flat, cu, batch: int, dim: int):
    """Event-compact (E,) streams into (batch, dim, Lmax) slots.

    Returns (u_c, kminus1_c, mask, idx) with idx[b, d, j] the flat event index.
    """
    cu = np.asarray(cu, np.int64)
    n = cu[1:] - cu[:-1]
    Lmax = max(int(n.max()) if n.size else 0, 1)
    j = np.arange(Lmax)
    mask = j[None, :] < n[:, None]
    idx = np.where(mask, cu[:-1, None] + j[None, :], 0)
    u_c = torch.as_tensor(np.asarray(u_flat)[idx], dtype=torch.float32) * torch.as_tensor(mask)
    km1 = torch.as_tensor((np.asarray(k_flat)[idx] - 1) * mask, dtype=torch.float32)
    shape = (batch, dim, Lmax)
    return (u_c.reshape(shape), km1.reshape(shape), torch.as_tensor(mask).reshape(shape),
            idx.reshape(shape))


def depthwise_event_scan(u_c, km1, mask, dt_idle, dt_active, A, W_B, W_C, D):
    """Flat depthwise event scan via selective_scan_ref on compacted tensors."""
    delta = (dt_idle[None, :, None] * km1 + dt_active[None, :, None]) * mask
    Bc = (u_c.unsqueeze(2) * W_B[None, :, :, None])   # (b, d, n, l) = (B, G=D, N, L)
    Cc = (u_c.unsqueeze(2) * W_C[None, :, :, None])
    return selective_scan_ref(u_c, delta, A, Bc, Cc, D=D)
