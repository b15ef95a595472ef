"""GPU parity of the fused event-block parameter transforms
(bcm_event_params_fwd / _bwd through interface.event_params) against the
PyTorch ops they replace (spike_mamba/e_model.py:463 A = -exp(A_log);
:475-476 the W_BC halves; :210-230 softplus(a0 / a1) + eps), forward values
and gradients.  The slices and dA_log = dA * A are exact; the softplus
values and derivatives within 1e-6 of PyTorch's (the same fp32 formulas)."""
import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close, assert_exact
from bc_mamba_b200 import interface as itf

pytestmark = pytest.mark.gpu
dev = "cuda"


def _leaves(dim, N, seed, spread=1.0):
    g = torch.Generator().manual_seed(seed)
    t = dict(A_log=torch.randn(dim, N, generator=g), W_BC=torch.randn(dim, 2 * N, generator=g),
             a0=spread * torch.randn(dim, generator=g), a1=spread * torch.randn(dim, generator=g))
    return {k: v.to(dev).requires_grad_(True) for k, v in t.items()}


def _torch_ops(p, N, eps):
    return (-torch.exp(p["A_log"]), p["W_BC"][:, :N].contiguous(), p["W_BC"][:, N:].contiguous(),
            F.softplus(p["a0"]) + eps, F.softplus(p["a1"]) + eps)


@pytest.mark.parametrize("dim,N", [(256, 16), (5, 3), (1, 1), (130, 64), (4096, 16)])
def test_event_params_match_torch(dim, N):
    eps = 1e-6
    p, q = _leaves(dim, N, seed=dim + N), _leaves(dim, N, seed=dim + N)
    mine = itf.event_params(p["A_log"], p["W_BC"], p["a0"], p["a1"], eps)
    ref = _torch_ops(q, N, eps)
    names = ["A", "W_B", "W_C", "dt_idle", "dt_active"]
    for a, b, n in zip(mine, ref, names):
        if n in ("W_B", "W_C"):
            assert_exact(a, b, n)
        else:
            assert_close(a, b, 1e-6, n)
    g = torch.Generator().manual_seed(7)
    ups = [torch.randn(t.shape, generator=g).to(dev) for t in ref]
    sum(((a * u).sum() for a, u in zip(mine, ups))).backward()
    sum(((b * u).sum() for b, u in zip(ref, ups))).backward()
    for k in p:
        if k in ("A_log", "W_BC"):
            assert_exact(p[k].grad, q[k].grad, "d" + k)
        else:
            assert_close(p[k].grad, q[k].grad, 1e-6, "d" + k)


def test_event_params_softplus_threshold():
    """Inputs around the pass-through threshold (20) and far below it."""
    dim, N = 64, 4
    p = _leaves(dim, N, seed=3)
    vals = torch.linspace(-40.0, 40.0, dim, device=dev)
    vals[dim // 2] = 20.0
    with torch.no_grad():
        p["a0"].copy_(vals)
        p["a1"].copy_(vals.flip(0) + 0.5)
    q = {k: v.detach().clone().requires_grad_(True) for k, v in p.items()}
    mine = itf.event_params(p["A_log"], p["W_BC"], p["a0"], p["a1"], 1e-6)
    ref = _torch_ops(q, N, 1e-6)
    for a, b, n in zip(mine[3:], ref[3:], ["dt_idle", "dt_active"]):
        assert_close(a, b, 1e-6, n)
    (mine[3].sum() + 2 * mine[4].sum()).backward()
    (ref[3].sum() + 2 * ref[4].sum()).backward()
    assert_close(p["a0"].grad, q["a0"].grad, 1e-6, "da0")
    assert_close(p["a1"].grad, q["a1"].grad, 1e-6, "da1")
    # only dt_* carried a gradient: the others are exact zeros
    assert torch.count_nonzero(p["A_log"].grad) == 0 and torch.count_nonzero(p["W_BC"].grad) == 0


def test_event_params_partial_gradients():
    """Outputs without a gradient (None in the backward) give zeros."""
    dim, N = 32, 8
    p = _leaves(dim, N, seed=9)
    A, W_B, W_C, dt_i, dt_a = itf.event_params(p["A_log"], p["W_BC"], p["a0"], p["a1"], 1e-6)
    W_C.sum().backward()
    assert torch.count_nonzero(p["A_log"].grad) == 0
    assert torch.count_nonzero(p["a0"].grad) == 0 and torch.count_nonzero(p["a1"].grad) == 0
    assert torch.all(p["W_BC"].grad[:, :N] == 0) and torch.all(p["W_BC"].grad[:, N:] == 1)


def test_event_params_errors():
    ops = itf.load_ops()
    A_log = torch.randn(4, 8, device=dev)
    a = torch.randn(4, device=dev)
    with pytest.raises(RuntimeError, match="W_BC must have shape"):
        ops.event_params_fwd(A_log, torch.randn(4, 8, device=dev), a, a, 1e-6)
    with pytest.raises(RuntimeError, match="contiguous float32"):
        ops.event_params_fwd(A_log.double(), torch.randn(4, 16, device=dev), a, a, 1e-6)
    with pytest.raises(RuntimeError, match="a1 must have shape"):
        ops.event_params_fwd(A_log, torch.randn(4, 16, device=dev), a, torch.randn(5, device=dev), 1e-6)
