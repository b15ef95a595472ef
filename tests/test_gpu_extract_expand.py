"""GPU parity of the fused extraction + expansion (``extract_expanded_events``,
the fill pass writing the expanded stream directly): its outputs equal
``expand_base_events`` applied to ``extract_base_events`` bit for bit, and the
oracle's expansion, for both input layouts, expand 1..3, ragged shapes, 16-bit
and float64 inputs, and the empty and all-events edge cases; the host-side
maximum equals the device maximum."""
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
