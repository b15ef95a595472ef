"""GPU parity of the staged depthwise scan kernels (dstate <= 64 with the
channels of each feature filling whole warps: batch a multiple of 16), forward
and backward against the float64 oracle, tolerance as test_gpu_scan.py.
Covers every dstate the layouts pad (1..64), ragged and empty channels,
channels over one 2048-event chunk, gaps past the decay table (sparse
spikes), 16-bit inputs, the silu gate and growing (A > 0) states."""
import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32
from test_gpu_scan import _events, _params, _run_and_check
from bc_mamba_b200.workloads import CONFIGS

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def staged_only():
    """The staged kernels at every size (by default small batches take the
    event-parallel ones)."""
    import os
    old = os.environ.get("BCM_SCAN_SEG")
    os.environ["BCM_SCAN_SEG"] = "0"
    yield
    if old is None:
        os.environ.pop("BCM_SCAN_SEG", None)
    else:
        os.environ["BCM_SCAN_SEG"] = old


@pytest.mark.parametrize("N", [1, 4, 7, 8, 9, 12, 16, 17, 24, 32, 33, 48, 64])
def test_staged_dstates(N):
    c = CONFIGS["c0"].with_(B=16, D=8, N=N, L=300, rho=0.25, seed=40 + N)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, N, N)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


def test_staged_c1_shape_rows():
    """The bench layout (B = 32 rows per feature, N = 16) on a short sequence."""
    c = CONFIGS["c1"].with_(D=8, L=400)
    inp, ch, t, k, cu, mx, u = _events(c)
    p = lambda n: inp[n].numpy()
    _run_and_check(u, k, cu, mx, p("dt_idle"), p("dt_active"), p("A"), p("W_B"), p("W_C"), D=p("D"))


def test_staged_ragged_and_empty_channels():
    rng = np.random.default_rng(7)
    B, D, N = 16, 4, 16
    NC = B * D
    n = rng.integers(0, 90, NC)
    n[::5] = 0
    n[3] = 97
    cu = np.zeros(NC + 1, np.int32)
    cu[1:] = np.cumsum(n)
    E = int(cu[-1])
    k = rng.integers(1, 9, E).astype(np.int32)
    u = rng.standard_normal(E).astype(np.float32)
    dti, dta, A, WB, WC, Dv = _params(D, N, 3)
    _run_and_check(u, k, cu, int(n.max()), dti, dta, A, WB, WC, D=Dv)


def test_staged_multi_chunk():
    c = CONFIGS["c0"].with_(B=16, D=2, N=16, L=5000, rho=0.8, seed=17)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 2048
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 11)
    res, _ = _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)
    assert res[1].shape[1] == (mx + 2047) // 2048


def test_staged_sparse_gaps_past_table():
    """rho = 0.02: many gaps exceed the 128-row decay table."""
    c = CONFIGS["c0"].with_(B=16, D=4, N=16, L=3000, rho=0.02, seed=18)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert (k > 128).any()
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 12)
    _run_and_check(u, k, cu, mx, 0.05 * dti, 0.05 * dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_staged_16bit(dtype):
    c = CONFIGS["c0"].with_(B=16, D=8, N=16, L=300, rho=0.3, seed=19)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 13)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv, dtype=dtype, tol=TOL_16)


def test_staged_gate_no_skip():
    c = CONFIGS["c0"].with_(B=16, D=8, N=16, L=300, rho=0.3, seed=20)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, _ = _params(c.D, c.N, 14)
    z = np.random.default_rng(5).standard_normal(u.size).astype(np.float32)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=None, z=z)


def test_staged_growing_states():
    """A > 0 for some states and large dt, so decaying states hit the -126
    exponent clamp: the forward must apply the clamps to prod(a) exactly."""
    c = CONFIGS["c0"].with_(B=16, D=4, N=8, L=200, rho=0.3, seed=21)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 15)
    A = A.copy()
    A[:, ::3] = 1e-4          # slowly growing states: prod(a) must keep every clamp
    _run_and_check(u, k, cu, mx, 30 * dti, 30 * dta, A, 0.3 * WB, 0.3 * WC, D=Dv)


def test_staged_c3_shape_rows():
    """The c3 layout (N = 64, bursty Markov spikes) on a short sequence."""
    c = CONFIGS["c3"].with_(B=16, D=8, L=300)
    inp, ch, t, k, cu, mx, u = _events(c)
    p = lambda n: inp[n].numpy()
    _run_and_check(u, k, cu, mx, p("dt_idle"), p("dt_active"), p("A"), p("W_B"), p("W_C"), D=p("D"))
