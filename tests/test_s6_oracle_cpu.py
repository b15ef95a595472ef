"""The float64 dense-S6 oracle (oracle/s6.py) against golden vectors from the
reference's own selective_scan_ref (tests/golden/make_s6_ref_fixtures.py):
output, last state (the oracle's last chunk state, times B for fixed B) and
every gradient, within 1e-5 of the reference's float32 values (relative to
the largest magnitude).  Also the chunk products and the 2048-position chunk
boundary on a long sequence."""
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_close
from oracle import s6

GOLD = Path(__file__).resolve().parent / "golden"
NAMES = ["fixed", "var_groups", "mixed_n4", "var_b_fixed_c"]


def _load(name):
    f = np.load(GOLD / f"s6_ref_{name}.npz")
    return {k: f[k] for k in f.files}


def _kw(r):
    return dict(D=r.get("D"), z=r.get("z"), delta_bias=r.get("delta_bias"), delta_softplus=bool(r["softplus"]))


@pytest.mark.parametrize("name", NAMES)
def test_s6_oracle_forward_vs_reference(name):
    r = _load(name)
    out, x, out_z, _ = s6.s6_fwd(r["u"], r["delta"], r["A"], r["B"], r["C"], **_kw(r))
    assert_close(out_z if out_z is not None else out, r["out"], 1e-5, "out")
    h_last = x[:, :, -1, 1::2]
    if r["B"].ndim == 2:     # the reference's state carries B; the chunk state does not
        h_last = h_last * r["B"][None]
    assert_close(h_last, r["last_state"], 1e-5, "last state")


@pytest.mark.parametrize("name", NAMES)
def test_s6_oracle_backward_vs_reference(name):
    r = _load(name)
    g = s6.s6_bwd(r["u"], r["delta"], r["A"], r["B"], r["C"], r["dout"], **_kw(r))
    for k in ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]:
        if "d" + k in r:
            assert_close(g["d" + k], r["d" + k], 1e-5, "d" + k)


def test_s6_oracle_chunk_states():
    rng = np.random.default_rng(5)
    b, d, L, N = 1, 2, 2100, 4
    u = rng.standard_normal((b, d, L))
    delta = 0.001 + 0.002 * rng.random((b, d, L))
    A = -np.tile(np.arange(1, N + 1, dtype=np.float64), (d, 1))
    B = rng.standard_normal((d, N))
    C = rng.standard_normal((d, N))
    out, x, _, hs = s6.s6_fwd(u, delta, A, B, C)
    assert x.shape == (b, d, 2, 2 * N)
    for c, t in ((0, 2047), (1, L - 1)):
        np.testing.assert_allclose(x[:, :, c, 0::2], np.exp(A[None] * delta[:, :, : t + 1].sum(-1)[:, :, None]),
                                   rtol=1e-12)
        np.testing.assert_allclose(x[:, :, c, 1::2], hs[:, :, t], rtol=0, atol=0)
