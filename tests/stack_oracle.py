"""CPU float64 event path of one stack block built from the oracle (TEST
INFRASTRUCTURE ONLY): the same computation as ``bc_mamba_b200.stack.event_path``
(extraction of the membrane -> expansion -> gather of x_conv -> depthwise
scan -> ZOH restore) as a torch autograd Function whose backward is the
oracle's restore / scan / gather backward, so ``EventStack`` runs on CPU ranks
with this path in place of the CUDA one."""
from __future__ import annotations

import numpy as np
import torch

from oracle import events as ev
from oracle import restore as rs
from oracle import scan as sc


class OracleEventPath(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_conv, dt_idle, dt_active, A, W_B, W_C, D, v, threshold, expand, info):
        B, L, dm = v.shape
        dim = x_conv.shape[1]
        base = v.detach().transpose(1, 2).contiguous().numpy()           # (B, d_model, L)
        thr = threshold.detach().cpu().numpy() if isinstance(threshold, torch.Tensor) else threshold
        bch, bt, bk, bcu, _, _ = ev.extract_base_events(base, thr)
        ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, B, dm, expand)
        uf = ev.gather_events_fwd(x_conv.detach().numpy(), ch, t)
        p = [x.detach().double().numpy() for x in (dt_idle, dt_active, A, W_B, W_C, D)]
        out, _x, _ = sc.scan_fwd(uf, k, cu, int(mx), p[0], p[1], p[2], p[3], p[4], D=p[5], is_depthwise_bc=True)
        y = rs.restore_dense_fwd(out, t, cu, dim, L)
        ctx.stream = (ch, t, k, cu, int(mx), uf, p, B, dim, L)
        info.append((int(ch.size), int(mx)))
        return torch.as_tensor(np.asarray(y, np.float64))

    @staticmethod
    def backward(ctx, g):
        ch, t, k, cu, mx, uf, p, B, dim, L = ctx.stream
        dy = rs.restore_dense_bwd(g.detach().double().numpy(), t, cu, dim, L)
        r = sc.scan_bwd(uf, k, cu, mx, p[0], p[1], p[2], p[3], p[4], dy, D=p[5], is_depthwise_bc=True)
        du, dA, dWB, dWC, ddi, dda, dD = r[:7]
        dx = ev.gather_events_bwd(du, ch, t, B * dim, L).reshape(B, dim, L)
        as_t = lambda a: torch.as_tensor(np.asarray(a, np.float64))
        return (as_t(dx), as_t(ddi), as_t(dda), as_t(dA), as_t(dWB), as_t(dWC), as_t(dD),
                None, None, None, None)


def oracle_path(v, x_conv, threshold, expand, dt_idle, dt_active, A, W_B, W_C, D):
    info = []
    y = OracleEventPath.apply(x_conv, dt_idle, dt_active, A, W_B, W_C, D, v, threshold, expand, info)
    return y, info[0]
