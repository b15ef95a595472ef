"""GPU parity of the gather backward that takes the stream's cu_seqlens
(``gather_events_bwd_rows``, used by the interface's gather autograd function):
equal, bit for bit, to ``gather_events_bwd`` and to the oracle scatter for
extraction-order streams of the configs, every dtype, ragged L (vector and
scalar row stores), rows too long for shared memory, and empty streams; and,
through the device fallback, for streams whose times are shuffled inside each
channel."""
import numpy as np
import pytest
import torch

from helpers import assert_exact
from oracle import events as ev
from bc_mamba_b200 import load_ops
from bc_mamba_b200.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"


def _stream(c):
    inp = make_inputs(c)
    r = ev.extract_base_events(inp["v"].float().numpy(), inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(*r[:4], c.B, c.d_model, c.expand)
    return ch, t, cu


def _check(ch, t, cu, NC, L, dtype, seed=0):
    ops = load_ops()
    g = torch.randn(ch.size, generator=torch.Generator().manual_seed(seed)).to(dtype)
    ref = ev.gather_events_bwd(g.double().numpy(), ch, t, NC, L)
    dx = ops.gather_events_bwd_rows(g.to(dev), torch.as_tensor(t).to(dev), torch.as_tensor(cu).to(dev), NC, L)
    assert dx.dtype == dtype and dx.shape == (NC, L)
    assert_exact(dx.double(), ref, "dx rows")
    via_ids = ops.gather_events_bwd(g.to(dev), torch.as_tensor(ch).to(dev), torch.as_tensor(t).to(dev), NC, L)[0]
    assert torch.equal(dx, via_ids)


@pytest.mark.parametrize("cfg", ["c0", "c1", "c3"])
def test_configs(cfg):
    c = CONFIGS[cfg]
    ch, t, cu = _stream(c)
    _check(ch, t, cu, c.B * c.D, c.L, torch.float32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("L", [250, 256, 257])
def test_dtypes_and_ragged_rows(dtype, L):
    c = CONFIGS["c0"].with_(L=L)
    ch, t, cu = _stream(c)
    _check(ch, t, cu, c.B * c.D, L, dtype)


def test_rows_longer_than_shared_memory():
    # 13,000 fp32 positions = 52 KB a row: the chunked row writer
    c = CONFIGS["c0"].with_(B=1, D=8, L=13000, rho=0.3)
    ch, t, cu = _stream(c)
    _check(ch, t, cu, c.B * c.D, c.L, torch.float32)
    _check(ch, t, cu, c.B * c.D, c.L, torch.float64)


def test_shuffled_within_channels_takes_fallback():
    c = CONFIGS["c0"].with_(L=300)
    ch, t, cu = _stream(c)
    rng = np.random.default_rng(3)
    ts = t.copy()
    for r in range(cu.size - 1):
        s, e = cu[r], cu[r + 1]
        ts[s:e] = ts[s:e][rng.permutation(e - s)]
    assert not np.array_equal(ts, t)
    ops = load_ops()
    NC = c.B * c.D
    g = torch.randn(ch.size, generator=torch.Generator().manual_seed(4))
    ref = ev.gather_events_bwd(g.double().numpy(), ch, ts, NC, c.L)
    dx = ops.gather_events_bwd_rows(g.to(dev), torch.as_tensor(ts).to(dev), torch.as_tensor(cu).to(dev), NC, c.L)
    assert_exact(dx.double(), ref, "dx fallback")


def test_empty_stream():
    ops = load_ops()
    NC, L = 6, 40
    dx = ops.gather_events_bwd_rows(torch.zeros(0, device=dev), torch.zeros(0, dtype=torch.int32, device=dev),
                                    torch.zeros(NC + 1, dtype=torch.int32, device=dev), NC, L)
    assert dx.shape == (NC, L) and not dx.any()
