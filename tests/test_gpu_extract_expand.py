"""GPU parity of the fused extraction + expansion (``extract_expanded_events``,
the fill pass writing the expanded stream directly): its outputs equal
``expand_base_events`` applied to ``extract_base_events`` bit for bit, and the
oracle's expansion, for both input layouts, expand 1..3, ragged shapes, 16-bit
and float64 inputs, and the empty and all-events edge cases; the host-side
maximum equals the device maximum; with x_conv the fused gather equals
``gather_events_fwd`` at the same stream, and the autograd function built on
it gives the gather's gradient."""
import numpy as np
import pytest
import torch

from helpers import assert_exact
from oracle import events as ev
from bc_mamba_b200 import load_ops

pytestmark = pytest.mark.gpu
dev = "cuda"
NAMES = ["ch", "t", "k", "cu", "max"]


def _check(x_bdl, thr, expand):
    """x_bdl: (B, d_model, L) on the host."""
    ops = load_ops()
    B, dm, L = x_bdl.shape
    base = ops.extract_base_events(x_bdl.contiguous().to(dev), thr)
    two_pass = ops.expand_base_events(*base[:4], B, dm, expand)
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(x_bdl.float().numpy(), thr)
    ref = ev.expand_base_events(bch, bt, bk, bcu, B, dm, expand)
    for bld, x_in in ((False, x_bdl.contiguous()), (True, x_bdl.transpose(1, 2).contiguous())):
        got, mx_host = ops.extract_expanded_events(x_in.to(dev), thr, expand, bld=bld)
        assert len(got) == 5
        for g, v, n in zip(got, two_pass, NAMES):
            assert g.dtype == torch.int32, n
            assert g.numel() == v.numel(), n
            assert torch.equal(g.reshape(-1), v.reshape(-1)), (n, bld)
        for g, r, n in zip(got[:4], ref[:4], NAMES):
            assert_exact(g, r, n)
        assert mx_host == int(np.asarray(ref[4]).reshape(-1)[0]) == int(got[4].reshape(-1)[0].item())
        # with x_conv: the same stream and the gather of x_conv at it
        xc = torch.randn(B, dm * expand, L, generator=torch.Generator().manual_seed(L + dm)).to(
            x_bdl.dtype if x_bdl.dtype in (torch.float16, torch.bfloat16, torch.float64) else torch.float32).to(dev)
        got_x, mx2 = ops.extract_expanded_events(x_in.to(dev), thr, expand, bld=bld, x_conv=xc)
        assert len(got_x) == 6 and mx2 == mx_host
        for g, v in zip(got_x[:5], got):
            assert torch.equal(g.reshape(-1), v.reshape(-1))
        assert got_x[5].dtype == xc.dtype and got_x[5].numel() == got[0].numel()
        if got[0].numel():
            assert torch.equal(got_x[5], ops.gather_events_fwd(xc, got[0], got[1])[0])
    return got


@pytest.mark.parametrize("B,dm,L", [(1, 1, 1), (2, 5, 31), (2, 32, 33), (3, 33, 300), (2, 64, 257),
                                    (4, 96, 1000), (1, 128, 2048)])
@pytest.mark.parametrize("expand", [1, 2, 3])
def test_shapes(B, dm, L, expand):
    g = torch.Generator().manual_seed(B * 1000 + L + dm + expand)
    _check(torch.randn(B, dm, L, generator=g), 0.4, expand)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_dtypes(dtype):
    g = torch.Generator().manual_seed(9)
    _check(torch.randn(2, 40, 300, generator=g).to(dtype), 0.25, 2)


def test_dense_channels_over_one_fill_block():
    # > 1024 events in a channel: the fill's 1024-slot list wraps several times
    x = torch.randn(2, 3, 3000)
    x[0, 1, :] = 1.0
    _check(x, 0.5, 2)


def test_no_events_and_all_events():
    x = torch.randn(2, 9, 77)
    got = _check(x, 1e9, 2)
    assert got[0].numel() == 0 and got[3].numel() == 2 * 9 * 2 + 1
    assert not got[3].any()
    _check(x, -1e9, 2)


def test_extract_gather_autograd():
    """interface.extract_events_base / extract_events_1d (fused fill + gather)
    against the unfused ops: same stream, same x_flat, same d x_conv."""
    from bc_mamba_b200 import interface as itf
    ops = load_ops()
    g = torch.Generator().manual_seed(11)
    B, dm, L, expand = 3, 40, 300, 2
    v = torch.randn(B, dm, L, generator=g).to(dev)
    xc = torch.randn(B, dm * expand, L, generator=g).to(dev)
    for fn, spikes in ((itf.extract_events_base, v), (itf.extract_events_1d, v.transpose(1, 2).contiguous())):
        x_leaf = xc.clone().requires_grad_(True)
        ch, ts, kf, cu, mx, x_flat = fn(spikes, x_leaf, 0.3, expand)
        base = ops.extract_base_events(v, 0.3)
        ref = ops.expand_base_events(*base[:4], B, dm, expand)
        for a, b in zip((ch, ts, kf, cu), ref[:4]):
            assert torch.equal(a, b)
        assert mx == int(ref[4].reshape(-1)[0].item())
        assert torch.equal(x_flat.detach(), ops.gather_events_fwd(xc, ch, ts)[0])
        w = torch.randn(x_flat.shape, generator=g).to(dev)
        (x_flat * w).sum().backward()
        assert torch.equal(x_leaf.grad, ops.gather_events_bwd(w, ch, ts, B * dm * expand, L)[0].view(B, -1, L))


@pytest.mark.parametrize("cap_bytes", ["0", "16000", "1000000000"])
def test_capacity_paths(cap_bytes, monkeypatch):
    """The fill runs before the host waits for the event total, into buffers
    of a capacity (BCM_ASYNC_FILL_BYTES / 16 bytes per event here); events
    past it are skipped there and the whole stream is filled again after:
    every capacity gives the same outputs."""
    ops = load_ops()
    g = torch.Generator().manual_seed(12)
    B, dm, L, expand = 2, 24, 500, 2
    v = torch.randn(B, dm, L, generator=g).to(dev)
    xc = torch.randn(B, dm * expand, L, generator=g).to(dev)
    base = ops.extract_base_events(v, 0.2)
    ref = ops.expand_base_events(*base[:4], B, dm, expand)
    assert ref[0].numel() * 16 > 16000            # the middle capacity is partial
    monkeypatch.setenv("BCM_ASYNC_FILL_BYTES", cap_bytes)
    got, mx = ops.extract_expanded_events(v, 0.2, expand, x_conv=xc)
    for a, b in zip(got[:4], ref[:4]):
        assert torch.equal(a, b)
    assert mx == int(ref[4].reshape(-1)[0].item())
    assert torch.equal(got[5], ops.gather_events_fwd(xc, ref[0], ref[1])[0])


def test_capacity_pins_little_more_than_the_stream():
    """The outputs are views of the fill's capacity buffers.  The capacity
    follows the largest of the last totals of the same input shape (x 1.25,
    + 4096 events), so no call's outputs keep much more storage alive than
    they hold (the first call of a shape fills exact-size outputs)."""
    ops = load_ops()
    g = torch.Generator().manual_seed(77)
    B, dm, L, expand = 3, 40, 777, 2              # a shape no other test uses
    xc = torch.randn(B, dm * expand, L, generator=g).to(dev)
    for _ in range(4):
        v = torch.randn(B, L, dm, generator=g).to(dev)
        got, _mx = ops.extract_expanded_events(v, 0.5, expand, bld=True, x_conv=xc)
        n = got[0].numel()
        limit = int(1.25 * 1.05 * n) + 4096       # draws at one density differ by well under 5 %
        for t in (got[0], got[1], got[2], got[5]):
            assert t.untyped_storage().nbytes() <= 4 * limit, (t.untyped_storage().nbytes(), n)


@pytest.mark.parametrize("B,dm,L", [(1, 1, 1), (2, 5, 31), (3, 33, 300), (4, 96, 1000), (2, 128, 4000)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_feature_thresholds(B, dm, L, dtype):
    """The per-feature form (bcm_extract_expanded_ft): feature j fires above
    thr[j]; bit-exact against the oracle's per-feature extraction, with the
    fused gather of x_conv; one value in every threshold repeats an input
    value exactly (strict compare)."""
    ops = load_ops()
    g = torch.Generator().manual_seed(B * 7 + dm + L)
    x = torch.randn(B, L, dm, generator=g).to(dtype)
    thr = (0.8 * torch.randn(dm, generator=g)).float()
    thr[0] = x[0, 0, 0].float()
    x_bdl = x.transpose(1, 2).contiguous()
    for expand in (1, 2):
        xc = torch.randn(B, dm * expand, L, generator=g).to(dev)
        got, mx = ops.extract_expanded_events(x.to(dev), 0.0, expand, bld=True, x_conv=xc,
                                              feature_thresholds=thr.to(dev))
        bch, bt, bk, bcu, _, _ = ev.extract_base_events(x_bdl.float().numpy(), thr.numpy())
        ref = ev.expand_base_events(bch, bt, bk, bcu, B, dm, expand)
        for a, r, n in zip(got[:4], ref[:4], NAMES):
            assert_exact(a, r, n)
        assert mx == int(np.asarray(ref[4]).reshape(-1)[0])
        if got[0].numel():
            assert torch.equal(got[5], ops.gather_events_fwd(xc, got[0], got[1])[0])
    # a threshold per feature equal to one scalar gives the scalar extraction
    same, _ = ops.extract_expanded_events(x.to(dev), 0.3, 2, bld=True,
                                          feature_thresholds=torch.full((dm,), 0.3, device=dev))
    scal, _ = ops.extract_expanded_events(x.to(dev), 0.3, 2, bld=True)
    for a, b in zip(same, scal):
        assert torch.equal(a.reshape(-1), b.reshape(-1))


def test_feature_thresholds_errors():
    ops = load_ops()
    x = torch.randn(2, 10, 4, device=dev)
    with pytest.raises(RuntimeError, match="need the"):
        ops.extract_expanded_events(x, 0.0, 1, bld=False, feature_thresholds=torch.zeros(4, device=dev))
    with pytest.raises(RuntimeError, match="feature_thresholds must be"):
        ops.extract_expanded_events(x, 0.0, 1, bld=True, feature_thresholds=torch.zeros(5, device=dev))
