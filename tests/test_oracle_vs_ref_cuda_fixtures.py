"""CPU tests: the oracle pinned to outputs of the reference's own CUDA
extensions (built from its sources by oracle/build_ref.py and run on a B200
by tests/golden/make_ref_cuda_fixtures.py, which wrote the ref_cuda_*.npz
fixtures).  Event streams, expansion, gather and the restore forward are
compared exactly; sums the reference accumulates in fp32 (restore backward,
scan) within TOL_F32 = 1e-5 of the float64 oracle."""
from pathlib import Path

import numpy as np
import pytest

from helpers import TOL_F32, assert_close, assert_exact
from oracle import events as ev
from oracle import restore as rs
from oracle import scan as sc

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["c0", "markov_small", "sparse_small"]


def _load(name):
    return np.load(GOLDEN / f"ref_cuda_{name}.npz")


@pytest.mark.parametrize("name", CASES)
def test_events_match_reference_cuda(name):
    f = _load(name)
    B, d_model, expand = int(f["B"]), int(f["d_model"]), int(f["expand"])
    got = ev.extract_base_events(f["v"], float(f["threshold"]))
    for g, key in zip(got, ["base_ch", "base_t", "base_k", "base_cu", "base_counts", "base_max"]):
        assert_exact(np.asarray(g).reshape(-1), f[key].reshape(-1), key)
    ex = ev.expand_base_events(*got[:4], B, d_model, expand)
    for g, key in zip(ex, ["ch", "t", "k", "cu", "max_seqlen"]):
        assert_exact(np.asarray(g).reshape(-1), f[key].reshape(-1), key)
    uf = ev.gather_events_fwd(f["u"], f["ch"], f["t"])
    assert_exact(uf, f["u_flat"], "gather")


@pytest.mark.parametrize("name", CASES)
def test_restore_matches_reference_cuda(name):
    f = _load(name)
    D, L = int(f["D"]), int(f["L"])
    dense = rs.restore_dense_fwd(f["out"], f["t"], f["cu"], D, L, out_dtype=np.float32)
    assert_exact(dense, f["dense"], "restore fwd")
    dy = rs.restore_dense_bwd(f["dout"], f["t"], f["cu"], D, L)
    assert_close(dy, f["dy"], TOL_F32, "restore bwd")


@pytest.mark.parametrize("name", CASES)
def test_scan_matches_reference_cuda(name):
    f = _load(name)
    a = (f["u_flat"], f["k"], f["cu"], int(f["max_seqlen"]), f["dt_idle"], f["dt_active"], f["A"],
         f["W_B"], f["W_C"])
    out, x, _ = sc.scan_fwd(*a, D=f["Dskip"], is_depthwise_bc=True)
    assert_close(out, f["out"], TOL_F32, "out")
    assert_close(x, f["x"], TOL_F32, "x")
    g = sc.scan_bwd(*a, f["dy"], D=f["Dskip"], is_depthwise_bc=True)
    for v, key in zip(g, ["du", "dA", "dW_B", "dW_C", "ddt_idle", "ddt_active", "dD"]):
        assert_close(v, f[key], TOL_F32, key)
