"""GPU parity of the event decode step (``event_decode_step`` through
``interface.EventDecoder``): decoding a sequence token by token equals the
forward path on the same inputs (fused extraction -> depthwise scan ->
restore) and the decode oracle within the fp32 tolerance (the forward
composes lane aggregates with the scan operator, so its rounding differs from
one event at a time); with the conv state it equals conv-at-events -> scan ->
restore; 16-bit inputs within the 16-bit tolerance."""
import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32, assert_close
from oracle import decode as dc
from bc_mamba_b200 import interface as itf
from bc_mamba_b200 import load_ops

pytestmark = pytest.mark.gpu
dev = "cuda"


def _params(D, N, seed):
    g = torch.Generator().manual_seed(seed)
    sp = torch.nn.functional.softplus
    return dict(dt_idle=sp(torch.randn(D, generator=g) - 2), dt_active=sp(torch.randn(D, generator=g) - 1),
                A=-torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1) * 0.3,
                W_B=torch.randn(D, N, generator=g), W_C=torch.randn(D, N, generator=g),
                D=torch.randn(D, generator=g))


def _inputs(B, d_model, expand, L, rho, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    D = d_model * expand
    xs = torch.randn(B, D, L, generator=g).to(dtype)
    spikes = (torch.rand(B, d_model, L, generator=g) < rho).to(dtype)
    return xs, spikes


def _decode(xs, spikes, p, conv=None):
    B, D, L = xs.shape
    N = p["A"].shape[1]
    dec = itf.EventDecoder(B, D, N, dev, xs.dtype, kernel_size=0 if conv is None else conv[0].shape[1])
    pd = {k: v.to(dev) for k, v in p.items()}
    ys = []
    for t in range(L):
        ys.append(dec.step(xs[:, :, t].to(dev), spikes[:, :, t].to(dev), 0.5, pd["dt_idle"], pd["dt_active"],
                           pd["A"], pd["W_B"], pd["W_C"], pd["D"],
                           None if conv is None else conv[0].to(dev), None if conv is None else conv[1].to(dev)))
    return torch.stack(ys, dim=1)   # (B, L, D)


def _forward(xs, spikes, p, conv=None):
    ops = load_ops()
    B, D, L = xs.shape
    d_model = spikes.shape[1]
    pd = {k: v.to(dev) for k, v in p.items()}
    (ch, ts, kf, cu, _mx, u), mx = ops.extract_expanded_events(spikes.to(dev), 0.5, D // d_model, x_conv=xs.to(dev))
    if conv is not None:
        u = ops.conv_events_fwd(xs.to(dev), conv[0].to(dev), conv[1].to(dev), ch, ts)[0]
    out = ops.fwd_flat_ch(u, kf, cu, mx, pd["dt_idle"], pd["dt_active"], pd["A"], pd["W_B"], pd["W_C"], pd["D"],
                          None, None, 0, True)[0]
    return ops.restore_dense_fwd(out, ts, cu, D, L)


@pytest.mark.parametrize("B,d_model,expand,N,L,rho", [(8, 8, 2, 16, 300, 0.2), (16, 4, 2, 8, 200, 0.5),
                                                       (8, 16, 1, 32, 150, 0.05)])
def test_decode_equals_forward(B, d_model, expand, N, L, rho):
    xs, spikes = _inputs(B, d_model, expand, L, rho, seed=B + N + L)
    p = _params(d_model * expand, N, seed=L)
    got = _decode(xs, spikes, p)
    ref = _forward(xs, spikes, p)
    assert got.shape == ref.shape
    assert_close(got, ref.cpu().numpy(), TOL_F32, "decode vs forward")
    oracle = dc.decode_sequence(xs.numpy(), spikes.numpy(), 0.5, **{k: v.numpy() for k, v in p.items()})
    assert_close(got, oracle, TOL_F32, "decode vs oracle")


def test_decode_with_conv_state():
    B, d_model, expand, N, L, K = 8, 8, 2, 16, 120, 4
    xs, spikes = _inputs(B, d_model, expand, L, 0.3, seed=3)
    p = _params(d_model * expand, N, seed=4)
    g = torch.Generator().manual_seed(5)
    conv = (torch.randn(d_model * expand, K, generator=g), torch.randn(d_model * expand, generator=g))
    got = _decode(xs, spikes, p, conv)
    assert_close(got, _forward(xs, spikes, p, conv), TOL_F32, "decode+conv vs conv-at-events forward")
    oracle = dc.decode_sequence(xs.numpy(), spikes.numpy(), 0.5, **{k: v.numpy() for k, v in p.items()},
                                conv_weight=conv[0].numpy(), conv_bias=conv[1].numpy())
    assert_close(got, oracle, TOL_F32, "decode+conv vs oracle")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_16bit(dtype):
    B, d_model, expand, N, L = 8, 8, 2, 16, 100
    xs, spikes = _inputs(B, d_model, expand, L, 0.3, seed=9, dtype=dtype)
    p = _params(d_model * expand, N, seed=10)
    got = _decode(xs, spikes, p)
    assert got.dtype == dtype
    oracle = dc.decode_sequence(xs.float().numpy(), spikes.float().numpy(), 0.5,
                                **{k: v.numpy() for k, v in p.items()})
    assert_close(got.float(), oracle, TOL_16, "decode 16-bit vs oracle")
