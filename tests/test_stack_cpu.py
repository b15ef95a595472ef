"""The block stack's scaled membrane (z_l = leak^(n-l) * v_l, one in-place
GEMM per block, per-feature thresholds on z's scale) against the unscaled
recurrence v_{l+1} = leak * v_l + y_l W_out^T with spikes where v_l > theta_l,
both on the float64 oracle event path (CPU).  With thresholds off the sample
values (no membrane value equals its threshold) both fire the same events and
give the same final membrane and parameter gradients to float64 rounding."""
import torch
import torch.nn.functional as F

from stack_oracle import oracle_path
from bc_mamba_b200 import stack as stk
from bc_mamba_b200.workloads import CONFIGS


def test_scaled_membrane_equals_unscaled_recurrence():
    f64 = torch.float64
    cfg = CONFIGS["c4"].with_(B=2, D=32, N=16, L=300, rho=0.2, blocks=3, seed=5)
    inp = stk.stack_inputs(cfg, range(cfg.B), "cpu")
    m = stk.EventStack(cfg, "cpu", seed=cfg.seed, path=oracle_path, dtype=f64)
    v0 = inp["v0"].double()
    xs = [x.double().requires_grad_(True) for x in inp["x_conv"]]
    thr = [t + 1e-3 for t in stk.calibrate_thresholds(m, v0, xs, gather=False)]
    z, ev = m.forward(v0, xs, thr)
    z.backward(inp["dout"].double())
    g_scaled = [p.grad.clone() for p in m.all_params()]
    dx_scaled = [x.grad.clone() for x in xs]
    for p in m.all_params():
        p.grad = None
    for x in xs:
        x.grad = None

    v = v0
    ev_ref = []
    N = cfg.N
    for l in range(cfg.blocks):
        p = m.params[l]
        y, e = oracle_path(v, xs[l], thr[l], cfg.expand, F.softplus(p.a0) + 1e-6, F.softplus(p.a1) + 1e-6,
                           -torch.exp(p.A_log), p.W_BC[:, :N], p.W_BC[:, N:], p.D)
        v = m.leak * v + y @ p.W_out.t()
        ev_ref.append(e)
    v.backward(inp["dout"].double())

    assert ev == ev_ref
    scale = v.abs().max().item()
    assert (z - v).abs().max().item() <= 1e-12 * scale
    for a, p in zip(g_scaled, m.all_params()):
        assert (a - p.grad).abs().max().item() <= 1e-12 * max(1.0, p.grad.abs().max().item())
    for a, x in zip(dx_scaled, xs):
        assert (a - x.grad).abs().max().item() <= 1e-12 * max(1.0, x.grad.abs().max().item())
