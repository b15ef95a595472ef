"""CPU pin of the decode oracle: decoding a sequence token by token
(oracle/decode.py) equals the training path on the same inputs — extraction,
expansion, the depthwise flat-channel scan and the restore (oracle/events.py,
oracle/scan.py, oracle/restore.py), with and without the conv-state update
(against oracle/conv.py) and across the restore's 4095-event cap."""
import numpy as np
import pytest

from oracle import conv as cv
from oracle import decode as dc
from oracle import events as ev
from oracle import restore as rs
from oracle import scan as sc


def _params(D, N, seed):
    rng = np.random.default_rng(seed)
    sp = lambda x: np.log1p(np.exp(x))
    return dict(dt_idle=sp(rng.standard_normal(D) - 2).astype(np.float32),
                dt_active=sp(rng.standard_normal(D) - 1).astype(np.float32),
                A=-np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)) * 0.3,
                W_B=rng.standard_normal((D, N)).astype(np.float32),
                W_C=rng.standard_normal((D, N)).astype(np.float32),
                D=rng.standard_normal(D).astype(np.float32))


def _event_path(xs, spikes, thr, p, conv=None):
    """Training path: (B, L, D) restored outputs."""
    B, D, L = xs.shape
    d_model = spikes.shape[1]
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(spikes, thr)
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, B, d_model, D // d_model)
    if conv is None:
        u = ev.gather_events_fwd(xs, ch, t)
    else:
        u = cv.conv_events_fwd(xs, conv[0], conv[1], ch, t)
    if t.size == 0:
        return np.zeros((B, L, D))
    out, _, _ = sc.scan_fwd(u, k, cu, int(np.asarray(mx).reshape(-1)[0]), p["dt_idle"], p["dt_active"], p["A"],
                            p["W_B"], p["W_C"], D=p["D"], is_depthwise_bc=True)
    return rs.restore_dense_fwd(out, t, cu, D, L)


@pytest.mark.parametrize("B,d_model,expand,N,L,rho", [(2, 3, 2, 4, 60, 0.3), (1, 4, 1, 7, 90, 0.05),
                                                       (3, 2, 3, 16, 40, 0.9)])
def test_decode_equals_event_path(B, d_model, expand, N, L, rho):
    rng = np.random.default_rng(B * 100 + N + L)
    D = d_model * expand
    xs = rng.standard_normal((B, D, L)).astype(np.float32)
    spikes = (rng.random((B, d_model, L)) < rho).astype(np.float32)
    p = _params(D, N, L)
    got = dc.decode_sequence(xs, spikes, 0.5, **p)
    ref = _event_path(xs, spikes, 0.5, p)
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def test_decode_with_conv_state():
    rng = np.random.default_rng(5)
    B, d_model, expand, N, L, K = 2, 3, 2, 8, 50, 4
    D = d_model * expand
    xs = rng.standard_normal((B, D, L)).astype(np.float32)
    spikes = (rng.random((B, d_model, L)) < 0.4).astype(np.float32)
    w = rng.standard_normal((D, K)).astype(np.float32)
    bias = rng.standard_normal(D).astype(np.float32)
    p = _params(D, N, 6)
    got = dc.decode_sequence(xs, spikes, 0.5, **p, conv_weight=w, conv_bias=bias)
    ref = _event_path(xs, spikes, 0.5, p, conv=(w, bias))
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def test_decode_holds_after_restore_cap():
    """A channel that fires at every token: after 4095 events the restore holds
    event 4094's output, and so does the decode."""
    B, d_model, N, L = 1, 1, 2, 4200
    rng = np.random.default_rng(7)
    xs = rng.standard_normal((B, 1, L)).astype(np.float32)
    spikes = np.ones((B, d_model, L), np.float32)
    p = _params(1, N, 8)
    got = dc.decode_sequence(xs, spikes, 0.5, **p)
    ref = _event_path(xs, spikes, 0.5, p)
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)
    assert np.all(got[0, 4094:, 0] == got[0, 4094, 0])
