"""CPU tests: the oracle pinned against the reference's own golden vectors and
hand-derived known answers; the torch restatement of selective_scan_ref
against the numpy oracle.  No GPU needed."""
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_close, assert_exact
from oracle import events as ev
from oracle import restore as rs
from oracle import scan as sc
from oracle.scan_ref import compact, depthwise_event_scan
from bc_mamba_b200.workloads import CONFIGS, make_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"
# golden vectors are fp32 results of the reference; the oracle is float64
GOLD_TOL = 2e-6


@pytest.mark.parametrize("name", ["c0_depthwise", "c0_legacy_bc", "c0_depthwise_z", "small_n4_sparse"])
def test_oracle_matches_reference_selective_scan_ref(name):
    f = np.load(GOLDEN / f"scan_ref_{name}.npz")
    legacy = "B" in f
    B = f["B"] if legacy else f["W_B"]
    C = f["C"] if legacy else f["W_C"]
    z = f["z_flat"] if "z_flat" in f else None
    a = (f["u_flat"], f["k_flat"], f["cu_seqlens"], int(f["max_seqlen"]), f["dt_idle"], f["dt_active"], f["A"], B, C)
    out, x, oz = sc.scan_fwd(*a, D=f["D"], z=z, is_depthwise_bc=not legacy)
    assert_close(oz if z is not None else out, f["out_flat"], GOLD_TOL, "out")
    g = sc.scan_bwd(*a, f["dout_flat"], D=f["D"], z=z, out=out, is_depthwise_bc=not legacy)
    names = ["du", "dA", "dB" if legacy else "dW_B", "dC" if legacy else "dW_C", "ddt_idle", "ddt_active", "dD"]
    if z is not None:
        names.append("dz")
    for v, n in zip(g, names):
        assert_close(v, f[n], GOLD_TOL, n)


def test_extract_known_answer():
    x = np.array([[[0.1, 0.9, 0.6, 0.2, 0.7]]], np.float32)
    ch, t, k, cu, counts, mx = ev.extract_base_events(x, 0.5)
    assert t.tolist() == [1, 2, 4] and k.tolist() == [2, 1, 2] and ch.tolist() == [0, 0, 0]
    assert cu.tolist() == [0, 3] and counts.tolist() == [3] and int(mx) == 3


def test_expand_known_answer():
    # two base channels with 2 and 1 events, expand 2 -> replicas contiguous per base channel
    bch = np.array([0, 0, 1], np.int32)
    bt = np.array([1, 3, 0], np.int32)
    bk = np.array([2, 2, 1], np.int32)
    bcu = np.array([0, 2, 3], np.int32)
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, 1, 2, 2)
    assert ch.tolist() == [0, 0, 1, 1, 2, 3]
    assert t.tolist() == [1, 3, 1, 3, 0, 0]
    assert cu.tolist() == [0, 2, 4, 5, 6] and int(mx) == 2


def test_restore_known_answer():
    # events at t = 1, 2, 4 with y = [10, 20, 30]: ZOH [0, 10, 20, 20, 30]
    y = np.array([10.0, 20.0, 30.0])
    ts = np.array([1, 2, 4], np.int32)
    cu = np.array([0, 3], np.int32)
    out = rs.restore_dense_fwd(y, ts, cu, 1, 5)
    assert out[0, :, 0].tolist() == [0, 10, 20, 20, 30]
    dy = rs.restore_dense_bwd(np.arange(1, 6, dtype=np.float64).reshape(1, 5, 1), ts, cu, 1, 5)
    assert dy.tolist() == [2.0, 3.0 + 4.0, 5.0]


def test_restore_search_cap_known_answer():
    L = 4200
    ts = np.arange(L, dtype=np.int32)       # an event at every position
    cu = np.array([0, L], np.int32)
    y = np.arange(L, dtype=np.float64)
    out = rs.restore_dense_fwd(y, ts, cu, 1, L)[0, :, 0]
    assert out[4094] == 4094 and out[4095] == 4094 and out[-1] == 4094
    dy = rs.restore_dense_bwd(np.ones((1, L, 1)), ts, cu, 1, L)
    assert dy[4094] == L - 4094 and np.all(dy[4095:] == 0) and np.all(dy[:4094] == 1)


def test_legacy_mask_head_flags():
    m = np.zeros((1, 3, 6), bool)
    m[0, 0, [1, 4]] = True
    m[0, 2, [0]] = True
    ch, t, k, cu, mx, hf = ev.extract_events(m)
    assert hf.tolist() == [1, 0, 1] and k.tolist() == [2, 3, 1] and int(mx) == 2


def test_scan_ref_restatement_matches_oracle():
    cfg = CONFIGS["c0"]
    inp = make_inputs(cfg)
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(inp["v"].numpy(), inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, cfg.B, cfg.d_model, cfg.expand)
    uf = ev.gather_events_fwd(inp["u"].numpy(), ch, t)
    u_c, km1, mask, idx = compact(uf, k, cu, cfg.B, cfg.D)
    y = depthwise_event_scan(u_c, km1, mask.float(), inp["dt_idle"], inp["dt_active"], inp["A"],
                             inp["W_B"], inp["W_C"], inp["D"])
    msk = mask.numpy().reshape(-1)
    got = np.zeros(uf.size)
    got[idx.reshape(-1)[msk]] = y.detach().numpy().reshape(-1)[msk]
    p = {n: inp[n].numpy() for n in ["dt_idle", "dt_active", "A", "W_B", "W_C", "D"]}
    ref, _, _ = sc.scan_fwd(uf, k, cu, int(mx), p["dt_idle"], p["dt_active"], p["A"], p["W_B"], p["W_C"],
                            D=p["D"], is_depthwise_bc=True)
    assert_close(got, ref, 1e-5, "selective_scan_ref restatement")


def test_multichunk_x_layout():
    # 5000 events in one channel -> 3 chunk states; chunk j holds the state after event 2048(j+1)-1
    rng = np.random.default_rng(0)
    E = 5000
    u = rng.standard_normal(E)
    k = np.ones(E, np.int32)
    cu = np.array([0, E], np.int32)
    A = -np.ones((1, 2))
    out, x, _ = sc.scan_fwd(u, k, cu, E, [0.001], [0.001], A, [[1.0, 0.5]], [[1.0, 1.0]],
                            is_depthwise_bc=True)
    assert x.shape == (1, 3, 4)
    out2, x2, _ = sc.scan_fwd(u[:2048], k[:2048], np.array([0, 2048], np.int32), 2048, [0.001], [0.001], A,
                              [[1.0, 0.5]], [[1.0, 1.0]], is_depthwise_bc=True)
    np.testing.assert_allclose(x[0, 0], x2[0, 0], rtol=1e-12)


def test_oracle_per_feature_thresholds():
    """The oracle's per-feature extraction: feature j fires strictly above
    thr[j]; equal thresholds give the scalar extraction."""
    import numpy as np

    from oracle import events as ev

    rng = np.random.default_rng(3)
    B, dm, L = 3, 7, 50
    x = rng.standard_normal((B, dm, L)).astype(np.float32)
    thr = rng.standard_normal(dm).astype(np.float32)
    thr[2] = x[1, 2, 5]                       # a value equal to its threshold does not fire
    ch, t, k, cu, counts, mx = ev.extract_base_events(x, thr)
    mask = x.reshape(B * dm, L) > np.tile(thr, B)[:, None]
    rows, cols = np.nonzero(mask)
    assert np.array_equal(ch, rows) and np.array_equal(t, cols)
    assert np.array_equal(counts, mask.sum(1))
    assert not mask[1 * dm + 2, 5]
    same = ev.extract_base_events(x, np.full(dm, 0.25, np.float32))
    scal = ev.extract_base_events(x, 0.25)
    for a, b in zip(same, scal):
        assert np.array_equal(np.asarray(a), np.asarray(b))


def test_restore_bitmap_is_the_extraction_mask_transposed():
    """For a stream fresh from extraction and expansion, the restore's event
    bitmap [B, ceil(L/32), D] is the threshold mask [B, d_model, ceil(L/32)]
    transposed, logical channel b*D + d taking base feature d // expand's
    words (what bcm_restore_dense_fwd_mask builds it from, up to 4095
    positions)."""
    import numpy as np

    from oracle import events as ev
    from oracle import restore as rs

    rng = np.random.default_rng(4)
    for B, dm, L, expand, thr in [(2, 5, 70, 3, 0.3), (1, 33, 64, 2, -0.2), (3, 4, 1, 1, 0.0)]:
        x = rng.standard_normal((B, dm, L)).astype(np.float32)
        bch, bt, bk, bcu, _, _ = ev.extract_base_events(x, thr)
        ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, B, dm, expand)
        D = dm * expand
        bm = rs.event_bitmap(t, cu, D, L)
        nw = (L + 31) // 32
        bits = np.zeros((B, dm, nw * 32), dtype=bool)
        bits[:, :, :L] = x > np.float32(thr)
        words = (bits.reshape(B, dm, nw, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(-1)
        mask = words.astype(np.uint32)                               # [B, d_model, nw]
        from_mask = np.repeat(mask.transpose(0, 2, 1), expand, axis=2)   # [B, nw, D]
        assert np.array_equal(bm, from_mask)
