"""CPU tests: the conv-at-events oracle against PyTorch's own dense
nn.Conv1d + SiLU + gather (the reference's fallback path when causal_conv1d is
not installed, spike_mamba/e_model.py:442-443), forward and backward, in
float64."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import conv as cv
from oracle import events as ev


def _dense(x, w, bias, ch, t):
    B, D, L = x.shape
    K = w.shape[1]
    xc = F.silu(F.conv1d(x, w.unsqueeze(1), bias, padding=K - 1, groups=D)[..., :L])
    return xc.reshape(B * D, L)[torch.as_tensor(ch, dtype=torch.long), torch.as_tensor(t, dtype=torch.long)]


@pytest.mark.parametrize("K", [1, 3, 4])
@pytest.mark.parametrize("with_bias", [True, False])
def test_oracle_matches_torch_conv1d(K, with_bias):
    g = torch.Generator().manual_seed(K * 10 + with_bias)
    B, D, L = 2, 6, 40
    x = torch.randn(B, D, L, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(D, K, generator=g, dtype=torch.float64, requires_grad=True)
    bias = torch.randn(D, generator=g, dtype=torch.float64, requires_grad=True) if with_bias else None
    mask = torch.rand(B * D, L, generator=g) < 0.3
    mask[0, 0] = mask[1, 1] = True          # events inside the zero-padded head
    ch, t, _, _, _, _ = ev.extract_base_events(mask.reshape(B, D, L).float().numpy(), 0.5)
    u = _dense(x, w, bias, ch, t)
    gu = torch.randn(u.shape, generator=g, dtype=torch.float64)
    u.backward(gu)
    np.testing.assert_allclose(cv.conv_events_fwd(x.detach().numpy(), w.detach().numpy(),
                                                  None if bias is None else bias.detach().numpy(), ch, t),
                               u.detach().numpy(), rtol=1e-12, atol=1e-12)
    dx, dw, db = cv.conv_events_bwd(x.detach().numpy(), w.detach().numpy(),
                                    None if bias is None else bias.detach().numpy(), ch, t, gu.numpy())
    np.testing.assert_allclose(dx, x.grad.numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dw, w.grad.numpy(), rtol=1e-12, atol=1e-12)
    if with_bias:
        np.testing.assert_allclose(db, bias.grad.numpy(), rtol=1e-12, atol=1e-12)
