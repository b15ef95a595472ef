"""GPU parity of the extraction from the (B, L, d_model) layout
(``extract_base_events_bld``, no transposed copy): the six outputs equal those
of ``extract_base_events`` on the transposed (B, d_model, L) copy and the
oracle, bit for bit, for ragged shapes, every input dtype and the empty and
all-events edge cases; ``extract_events_1d`` built on it gives the same
streams and gathered values as the transposed route."""
import pytest
import torch

from helpers import assert_exact
from oracle import events as ev
from bc_mamba_b200 import load_ops
from bc_mamba_b200 import interface as itf

pytestmark = pytest.mark.gpu
dev = "cuda"
NAMES = ["ch", "t", "k", "cu", "counts", "max"]


def _check(x_bld, thr):
    ops = load_ops()
    got = ops.extract_base_events_bld(x_bld.to(dev), thr)
    via_t = ops.extract_base_events(x_bld.transpose(1, 2).contiguous().to(dev), thr)
    ref = ev.extract_base_events(x_bld.transpose(1, 2).float().numpy(), thr)
    for g, v, r, n in zip(got, via_t, ref, NAMES):
        assert g.dtype == torch.int32, n
        assert g.shape == v.shape, n
        assert torch.equal(g, v), n
        assert_exact(g, r, n)
    return got


@pytest.mark.parametrize("B,L,dm", [(1, 1, 1), (2, 31, 5), (2, 33, 32), (3, 300, 33), (2, 257, 64),
                                    (4, 1000, 96), (1, 2048, 128)])
def test_shapes(B, L, dm):
    g = torch.Generator().manual_seed(B * 1000 + L + dm)
    _check(torch.randn(B, L, dm, generator=g), 0.4)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_dtypes(dtype):
    g = torch.Generator().manual_seed(7)
    _check(torch.randn(2, 300, 40, generator=g).to(dtype), 0.25)


def test_ties_nan_and_edges():
    x = torch.full((2, 70, 33), 0.5)
    x[0, 0, 0] = 0.75          # event at t = 0
    x[1, 69, 32] = 0.6         # event at t = L - 1 in the last (partial) feature block
    x[0, 10, 1] = float("nan")  # NaN > thr is false
    _check(x, 0.5)


def test_no_events_and_all_events():
    x = torch.randn(2, 77, 9)
    got = _check(x, 1e9)
    assert got[0].numel() == 0 and got[5].shape == (1,)
    _check(x, -1e9)


def test_extract_events_1d_matches_transposed_route():
    ops = load_ops()
    g = torch.Generator().manual_seed(3)
    B, L, dm, expand = 4, 500, 48, 2
    hs = torch.randn(B, L, dm, generator=g).to(dev)
    xc = torch.randn(B, dm * expand, L, generator=g).to(dev)
    ch, ts, kf, cu, mx, uf = itf.extract_events_1d(hs, xc, 0.3, expand)
    b = ops.extract_base_events(hs.transpose(1, 2).contiguous(), 0.3)
    e = ops.expand_base_events(*b[:4], B, dm, expand)
    for a, r, n in zip((ch, ts, kf, cu), e[:4], ["ch", "t", "k", "cu"]):
        assert torch.equal(a, r), n
    assert mx == int(e[4])
    assert torch.equal(uf, ops.gather_events_fwd(xc, e[0], e[1])[0])


@pytest.mark.parametrize("bld", [False, True])
def test_host_max_matches_device_outputs(bld):
    """extract_base_events_host_max: the same six outputs, and the maximum
    count as a host integer equal to the device max (also for no events)."""
    ops = load_ops()
    g = torch.Generator().manual_seed(11)
    for thr in (0.3, 1e9):
        x = torch.randn(3, 200, 40, generator=g).to(dev)        # (B, L, d_model)
        xin = x if bld else x.transpose(1, 2).contiguous()
        outs, mh = ops.extract_base_events_host_max(xin, thr, bld=bld)
        ref = ops.extract_base_events_bld(x, thr) if bld else ops.extract_base_events(xin, thr)
        for a, r, n in zip(outs, ref, NAMES):
            assert torch.equal(a, r), n
        assert isinstance(mh, int) and mh == int(ref[5].max())
