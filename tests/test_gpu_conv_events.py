"""GPU parity of the conv-at-events op (causal depthwise conv1d + SiLU
evaluated only at the events, replacing the dense conv + gather of
Mamba.forward): forward values and the dense input, weight and bias gradients
against the float64 oracle (itself pinned to torch's nn.Conv1d path on CPU)
and, through autograd, against torch's dense conv1d + silu + gather on the
GPU.  Tolerance |x - ref| <= tol*|ref| + tol*max|ref|: 1e-5 fp32, 2e-2
bf16/fp16."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_16, TOL_F32, assert_close
from oracle import conv as cv
from oracle import events as ev
from bc_mamba_b200 import interface as itf
from bc_mamba_b200 import load_ops

pytestmark = pytest.mark.gpu
dev = "cuda"


def _stream(B, D, L, rho, seed):
    g = torch.Generator().manual_seed(seed)
    mask = (torch.rand(B, D, L, generator=g) < rho).float()
    ch, t, _, cu, _, _ = ev.extract_base_events(mask.numpy(), 0.5)
    return ch, t, cu


def _case(B, D, L, K, rho, seed, dtype=torch.float32, bias=True, tol=TOL_F32):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, D, L, generator=g).to(dtype)
    w = torch.randn(D, K, generator=g) * 0.5
    b = torch.randn(D, generator=g) if bias else None
    ch, t, cu = _stream(B, D, L, rho, seed + 1)
    gu = torch.randn(ch.size, generator=g).to(dtype)
    ops = load_ops()
    T = lambda a: torch.as_tensor(a).to(dev)
    u = ops.conv_events_fwd(x.to(dev), w.to(dev), None if b is None else b.to(dev), T(ch), T(t))[0]
    xr = x.float().numpy()
    assert u.dtype == dtype
    assert_close(u.float(), cv.conv_events_fwd(xr, w.numpy(), None if b is None else b.numpy(), ch, t), tol, "u")
    dx, dw, db = ops.conv_events_bwd(x.to(dev), w.to(dev), None if b is None else b.to(dev), T(t), T(cu),
                                     gu.to(dev))
    rdx, rdw, rdb = cv.conv_events_bwd(xr, w.numpy(), None if b is None else b.numpy(), ch, t,
                                       gu.float().numpy())
    assert dx.dtype == dtype and dx.shape == (B, D, L)
    assert_close(dx.float(), rdx, tol, "dx")
    assert_close(dw, rdw, tol, "dw")
    assert_close(db, rdb, tol, "db")


@pytest.mark.parametrize("K", [1, 3, 4, 8])
def test_conv_events_vs_oracle(K):
    _case(2, 64, 256, K, 0.25, 10 + K)


def test_conv_events_long_rows_chunk_edges():
    """Dense events across many 256-position chunks (boundary-straddling windows)."""
    _case(2, 8, 1300, 4, 0.9, 21)


def test_conv_events_sparse_and_no_bias():
    _case(3, 24, 700, 4, 0.03, 22, bias=False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_conv_events_16bit(dtype):
    _case(2, 32, 300, 4, 0.3, 23, dtype=dtype, tol=TOL_16)


def test_conv_events_no_events():
    ops = load_ops()
    x = torch.randn(2, 4, 50, device=dev)
    w = torch.randn(4, 4, device=dev)
    b = torch.randn(4, device=dev)
    e = torch.zeros(0, dtype=torch.int32, device=dev)
    cu = torch.zeros(9, dtype=torch.int32, device=dev)
    assert ops.conv_events_fwd(x, w, b, e, e)[0].numel() == 0
    dx, dw, db = ops.conv_events_bwd(x, w, b, e, cu, torch.zeros(0, device=dev))
    assert float(dx.abs().sum()) == 0.0 and float(dw.abs().sum()) == 0.0 and float(db.abs().sum()) == 0.0


def test_autograd_matches_dense_torch_path():
    """ConvEventsFn gradients equal those of torch's dense conv1d + silu +
    gather (the computation it replaces) for x, weight and bias."""
    g = torch.Generator().manual_seed(5)
    B, D, L, K = 2, 32, 400, 4
    x0 = torch.randn(B, D, L, generator=g).to(dev)
    w0 = (torch.randn(D, 1, K, generator=g) * 0.5).to(dev)
    b0 = torch.randn(D, generator=g).to(dev)
    ch, t, cu = _stream(B, D, L, 0.2, 6)
    T = lambda a: torch.as_tensor(a).to(dev)
    gu = torch.randn(ch.size, generator=g).to(dev)

    x1, w1, b1 = (v.clone().requires_grad_(True) for v in (x0, w0, b0))
    u1 = itf.conv_events(x1, w1, b1, T(ch), T(t), T(cu))
    u1.backward(gu)

    x2, w2, b2 = (v.clone().requires_grad_(True) for v in (x0, w0, b0))
    xc = F.silu(F.conv1d(x2, w2, b2, padding=K - 1, groups=D)[..., :L])
    u2 = xc.reshape(B * D, L)[T(ch).long(), T(t).long()]
    u2.backward(gu)

    assert_close(u1.detach(), u2.detach().cpu().numpy(), TOL_F32, "u")
    assert_close(x1.grad, x2.grad.cpu().numpy(), TOL_F32, "dx")
    assert_close(w1.grad, w2.grad.cpu().numpy(), TOL_F32, "dw")
    assert_close(b1.grad, b2.grad.cpu().numpy(), TOL_F32, "db")
