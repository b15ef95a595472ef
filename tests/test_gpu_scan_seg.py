"""GPU parity of the event-parallel depthwise scan kernels (scan_seg.cu)
against the float64 oracle: warp groups of 1..16 batch rows (BCM_SEG_CPW pins
the group size, which at these sizes would otherwise be 1), ragged, empty and
one-event channels, channels spanning many 256-event tiles and several
2048-event chunks, gaps past the 256-row decay table, every dstate up to 64,
16-bit inputs, and the backward with and without the forward's tile carries
(bit-identical to each other).  BCM_SCAN_SEG=2 selects these kernels
wherever they apply.  Tolerance as test_gpu_scan.py."""
import os

import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32
from test_gpu_scan import _events, _params, _run_and_check
from bc_mamba_b200.workloads import CONFIGS

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def seg_everywhere():
    """Run the event-parallel kernels wherever they apply (by default they
    serve the shapes the staged kernels do not)."""
    old = os.environ.get("BCM_SCAN_SEG")
    os.environ["BCM_SCAN_SEG"] = "2"
    yield
    if old is None:
        os.environ.pop("BCM_SCAN_SEG", None)
    else:
        os.environ["BCM_SCAN_SEG"] = old


@pytest.fixture
def cpw(request):
    old = os.environ.get("BCM_SEG_CPW")
    os.environ["BCM_SEG_CPW"] = str(request.param)
    yield request.param
    if old is None:
        os.environ.pop("BCM_SEG_CPW", None)
    else:
        os.environ["BCM_SEG_CPW"] = old


def _ragged(B, D, N, seed, lo=0, hi=90, kmax=9, big_gap_every=0):
    rng = np.random.default_rng(seed)
    NC = B * D
    n = rng.integers(lo, hi, NC)
    n[::5] = 0
    n[1::7] = 1
    cu = np.zeros(NC + 1, np.int32)
    cu[1:] = np.cumsum(n)
    E = int(cu[-1])
    k = rng.integers(1, kmax, E).astype(np.int32)
    if big_gap_every:
        k[::big_gap_every] = rng.integers(257, 900, k[::big_gap_every].size)
    u = rng.standard_normal(E).astype(np.float32)
    return u, k, cu, int(n.max())


@pytest.mark.parametrize("cpw", [1, 3, 16], indirect=True)
def test_seg_ragged_groups(cpw):
    B, D, N = 16, 4, 16
    u, k, cu, mx = _ragged(B, D, N, seed=3)
    dti, dta, A, WB, WC, Dv = _params(D, N, 3)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("cpw", [2, 8], indirect=True)
def test_seg_tiny_channels_many_per_lane(cpw):
    """Channels of 0..5 events: a lane's 8 events cross several channels."""
    B, D, N = 32, 2, 16
    u, k, cu, mx = _ragged(B, D, N, seed=4, lo=0, hi=6)
    dti, dta, A, WB, WC, Dv = _params(D, N, 4)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("cpw", [1, 4], indirect=True)
def test_seg_gaps_past_table(cpw):
    B, D, N = 8, 4, 16
    u, k, cu, mx = _ragged(B, D, N, seed=5, lo=20, hi=400, big_gap_every=7)
    dti, dta, A, WB, WC, Dv = _params(D, N, 5)
    _run_and_check(u, k, cu, mx, 0.01 * dti, 0.01 * dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("cpw", [1, 2], indirect=True)
def test_seg_multi_chunk_channels(cpw):
    """Channels of up to ~4800 events: many tiles and three x chunks."""
    c = CONFIGS["c0"].with_(B=4, D=4, N=16, L=6000, rho=0.8, seed=23)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 4096
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 23)
    res, _ = _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)
    assert res[1].shape[1] == (mx + 2047) // 2048


@pytest.mark.parametrize("cpw", [1, 2], indirect=True)
def test_seg_multi_chunk_long_memory(cpw):
    """Small dt: the chunk products of x stay far from 0, so each must be the
    product since the channel's first event (carried across chunks)."""
    c = CONFIGS["c0"].with_(B=2, D=4, N=16, L=6000, rho=0.9, seed=24)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 4096
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 24)
    res, _ = _run_and_check(u, k, cu, mx, 0.01 * dti, 0.01 * dta, A, 0.3 * WB, 0.3 * WC, D=Dv,
                            fp32_decay=True)
    assert float(res[1][:, 1:, 0::2].max()) > 1e-3


@pytest.mark.parametrize("N", [1, 3, 8, 16, 33, 64])
def test_seg_dstates(N):
    c = CONFIGS["c0"].with_(B=4, D=8, N=N, L=700, rho=0.3, seed=60 + N)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, N, N)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_seg_16bit(dtype):
    c = CONFIGS["c0"].with_(B=4, D=8, N=16, L=900, rho=0.3, seed=61)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 61)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv, dtype=dtype, tol=TOL_16)


def test_seg_no_skip_and_pw_mixing():
    c = CONFIGS["c0"].with_(B=4, D=8, N=16, L=600, rho=0.3, seed=62)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, _ = _params(c.D, c.N, 62)
    rng = np.random.default_rng(62)
    pw = (rng.standard_normal((c.D, c.D)).astype(np.float32) * 0.3,
          rng.standard_normal((c.D, c.D)).astype(np.float32) * 0.3)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=None, pw=pw)


def test_seg_bench_shape_rows():
    """The c4 row layout (128 rows per feature, density 10 %) on a short
    sequence, with the group size the kernels pick themselves."""
    c = CONFIGS["c4"].with_(D=4, L=600)
    inp, ch, t, k, cu, mx, u = _events(c)
    p = lambda n: inp[n].numpy()
    _run_and_check(u, k, cu, mx, p("dt_idle"), p("dt_active"), p("A"), p("W_B"), p("W_C"), D=p("D"))


def test_seg_and_staged_agree_on_bursty_rows():
    """Both kernel families on the c4 row layout with 50 % Markov spikes
    (channels of very different lengths, some over 2048 events): every output
    and gradient within the fp32 tolerance of each other."""
    import bc_mamba_b200 as bcm
    from helpers import assert_close

    ops = bcm.load_ops()
    c = CONFIGS["c4"].with_(B=32, D=64, L=4000, rho=0.5, spikes="markov", seed=25)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 2048
    dev = "cuda"
    T_ = lambda x: torch.as_tensor(np.asarray(x)).to(dev).contiguous()
    ps = [T_(inp[n].numpy()) for n in ["dt_idle", "dt_active", "A", "W_B", "W_C"]]
    args = (T_(u), T_(k), T_(cu), mx, *ps)
    dout = torch.randn(u.size, generator=torch.Generator().manual_seed(3)).to(dev)
    res = {}
    for mode in ("0", "2"):
        os.environ["BCM_SCAN_SEG"] = mode
        out, x, ck = ops.fwd_flat_ch_ckpt(*args, T_(inp["D"].numpy()), None, None, 0, True, None, None)
        g = ops.bwd_flat_ch(*args, dout, x, T_(inp["D"].numpy()), None, None, None, 0, True, None, None, ck)
        res[mode] = [out, x] + list(g)
    names = ["out", "x", "du", "dA", "dW_B", "dW_C", "ddt_idle", "ddt_active", "dD"]
    for n, a, b in zip(names, res["0"], res["2"]):
        assert_close(a, b.cpu().numpy(), TOL_F32, n)
