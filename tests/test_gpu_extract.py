"""GPU parity: extraction, expansion and gather through the drop-in
``extract_events_cuda`` entry points, bit-exact against the oracle
(reference csrc/extract/extract_events_cuda.cu semantics)."""
import numpy as np
import pytest
import torch

from helpers import assert_exact
from oracle import events as ev
from bc_mamba_b200 import load_ops
from bc_mamba_b200.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"


def _check_extract(x: torch.Tensor, thr: float):
    ops = load_ops()
    got = ops.extract_base_events(x.to(dev), thr)
    ref = ev.extract_base_events(x.float().cpu().numpy(), thr)
    for g, r, name in zip(got, ref, ["ch", "t", "k", "cu", "counts", "max"]):
        assert g.dtype == torch.int32, name
        assert_exact(g, r, name)
    return got


@pytest.mark.parametrize("cfg", ["c0", "c1", "c3"])
def test_extract_expand_configs(cfg):
    c = CONFIGS[cfg]
    inp = make_inputs(c)
    got = _check_extract(inp["v"], inp["threshold"])
    ops = load_ops()
    ex = ops.expand_base_events(got[0], got[1], got[2], got[3], c.B, c.d_model, c.expand)
    ref = ev.expand_base_events(*(to.cpu().numpy() for to in got[:4]), c.B, c.d_model, c.expand)
    for g, r, name in zip(ex, ref, ["ch", "t", "k", "cu", "max"]):
        assert_exact(g, r, "expand " + name)
    # gather fwd / bwd are exact copies
    u = inp["u"].to(dev)
    uf = ops.gather_events_fwd(u, ex[0], ex[1])[0]
    assert_exact(uf, ev.gather_events_fwd(inp["u"].float().numpy(), ref[0], ref[1]), "gather")
    g = torch.randn(uf.shape, device=dev)
    dx = ops.gather_events_bwd(g, ex[0], ex[1], c.B * c.D, c.L)[0]
    assert_exact(dx, ev.gather_events_bwd(g.cpu().numpy(), ref[0], ref[1], c.B * c.D, c.L), "scatter")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_gather_bwd_any_order(dtype):
    """Rows in extraction order take the one-pass row writer; a shuffled
    stream (same unique (ch, t) pairs) falls back to zero-fill + scatter on
    the device and gives the same dx."""
    c = CONFIGS["c0"].with_(L=250)   # L not a multiple of the vector width
    inp = make_inputs(c)
    r = ev.extract_base_events(inp["v"].numpy(), inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(*r[:4], c.B, c.d_model, c.expand)
    NC = c.B * c.D
    g = torch.randn(ch.size, generator=torch.Generator().manual_seed(1)).to(dtype)
    ref = ev.gather_events_bwd(g.double().numpy(), ch, t, NC, c.L)
    ops = load_ops()
    for perm in [np.arange(ch.size), np.random.default_rng(2).permutation(ch.size)]:
        dx = ops.gather_events_bwd(g[perm].to(dev), torch.as_tensor(ch[perm]).to(dev),
                                   torch.as_tensor(t[perm]).to(dev), NC, c.L)[0]
        assert dx.dtype == dtype
        assert_exact(dx.double(), ref, "dx")


def test_known_answer():
    # x = [0.1, 0.9, 0.6, 0.2, 0.7], thr 0.5 -> t = [1, 2, 4], k = [2, 1, 2]
    x = torch.tensor([[[0.1, 0.9, 0.6, 0.2, 0.7]]])
    ch, t, k, cu, counts, mx = load_ops().extract_base_events(x.to(dev), 0.5)
    assert t.tolist() == [1, 2, 4] and k.tolist() == [2, 1, 2] and ch.tolist() == [0, 0, 0]
    assert cu.tolist() == [0, 3] and counts.tolist() == [3] and int(mx) == 3 and mx.dim() == 0


@pytest.mark.parametrize("L", [1, 31, 32, 33, 100, 1023, 1024, 1025, 5000])
def test_ragged_lengths(L):
    g = torch.Generator().manual_seed(L)
    x = torch.randn(3, 5, L, generator=g)
    _check_extract(x, 0.3)


def test_ties_exactly_at_threshold_and_edges():
    x = torch.full((2, 3, 64), 0.5)
    x[0, 0, 0] = 0.75      # event at t = 0
    x[1, 2, 63] = 0.5001   # event at t = L - 1
    x[0, 1, 10] = 0.5      # tie: not an event (strict >)
    got = _check_extract(x, 0.5)
    assert got[1].tolist() == [0, 63] and got[2].tolist() == [1, 64]


def test_no_events_and_all_events():
    ops = load_ops()
    x = torch.randn(2, 4, 77)
    ch, t, k, cu, counts, mx = ops.extract_base_events(x.to(dev), 1e9)
    assert ch.numel() == 0 and mx.shape == (1,) and int(mx) == 0
    assert cu.tolist() == [0] * 9 and counts.sum() == 0
    e = ops.expand_base_events(ch, t, k, cu, 2, 4, 2)
    assert e[0].numel() == 0 and e[3].tolist() == [0] * 17 and e[4].shape == (1,)
    _check_extract(x, -1e9)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_input_dtypes(dtype):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 8, 300, generator=g).to(dtype)
    _check_extract(x, 0.25)


def test_legacy_bool_mask():
    g = torch.Generator().manual_seed(9)
    m = torch.rand(2, 6, 200, generator=g) < 0.3
    got = load_ops().extract_events(m.to(dev))
    ref = ev.extract_events(m.numpy())
    for a, b, name in zip(got, ref, ["ch", "t", "k", "cu", "max", "head"]):
        assert_exact(a, b, name)


def test_argument_errors():
    ops = load_ops()
    with pytest.raises(RuntimeError, match="base_input must be 3-D"):
        ops.extract_base_events(torch.zeros(4, 4, device=dev), 0.5)
    with pytest.raises(RuntimeError, match="must be contiguous"):
        ops.extract_base_events(torch.zeros(2, 4, 8, device=dev).transpose(1, 2), 0.5)
    with pytest.raises(RuntimeError, match="channel_ids must be int32"):
        ops.gather_events_fwd(torch.zeros(1, 2, 3, device=dev), torch.zeros(2, device=dev, dtype=torch.int64),
                              torch.zeros(2, device=dev, dtype=torch.int32))
