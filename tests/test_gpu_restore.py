"""GPU parity: zero-order-hold restore forward (exact) and backward (fp32
segment sums) through ``restore_dense_cuda_nodecay`` against the oracle
(reference csrc/r_nodecay semantics, including the 4095-event search cap)."""
import numpy as np
import pytest
import torch

from helpers import assert_close, assert_exact
from oracle import events as ev
from oracle import restore as rs
from bc_mamba_b200 import load_ops
from bc_mamba_b200.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"


def _stream(cfg):
    inp = make_inputs(cfg)
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(inp["v"].numpy(), inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, cfg.B, cfg.d_model, cfg.expand)
    return ch, t, k, cu


def _check(t, cu, dim, L, y_dtype=torch.float32, out_dtype=None, seed=0):
    ops = load_ops()
    g = torch.Generator().manual_seed(seed)
    E = t.size
    y = torch.randn(E, generator=g).to(y_dtype)
    ts = torch.as_tensor(t, dtype=torch.int32, device=dev)
    cus = torch.as_tensor(cu, dtype=torch.int32, device=dev)
    out = ops.restore_dense_fwd(y.to(dev), ts, cus, dim, L, out_dtype)
    ref = rs.restore_dense_fwd(y.float().numpy(), t, cu, dim, L)
    exp_dtype = out_dtype or y_dtype
    assert out.dtype == exp_dtype
    ref_t = torch.as_tensor(ref, dtype=torch.float32).to(exp_dtype)
    assert_exact(out, ref_t, "restore fwd")
    # the forward that also writes the event bitmap for the backward
    out_b, bm = ops.restore_dense_fwd_bitmap(y.to(dev), ts, cus, dim, L, out_dtype)
    assert torch.equal(out_b, out)
    bm_ref = rs.event_bitmap(t, cu, dim, L)
    assert bm.dtype == torch.int32 and bm.dim() == 1 and bm.numel() >= bm_ref.size
    words = bm[:bm_ref.size].cpu().numpy().view(np.uint32).reshape(bm_ref.shape)
    assert np.array_equal(words, bm_ref), "event bitmap"
    B = (cu.size - 1) // dim
    dout = torch.randn(B, L, dim, generator=g).to(y_dtype)
    dy_ref = rs.restore_dense_bwd(dout.float().numpy(), t, cu, dim, L)
    for bitmap in (True, False):
        dy = ops.restore_dense_bwd(dout.to(dev), ts, cus, dim, L, bitmap)
        assert dy.dtype == torch.float32
        assert_close(dy, dy_ref, 1e-5, f"restore bwd (bitmap={bitmap})")
        # each kernel sums every interval in one fixed order: run to run identical
        assert torch.equal(dy, ops.restore_dense_bwd(dout.to(dev), ts, cus, dim, L, bitmap))
        if bitmap:
            # same sweep from the forward's bitmap: bit-identical
            assert torch.equal(dy, ops.restore_dense_bwd_bitmap(dout.to(dev), ts, cus, bm, dim, L))


@pytest.mark.parametrize("cfg", ["c0", "c1"])
def test_restore_configs(cfg):
    c = CONFIGS[cfg]
    ch, t, k, cu = _stream(c)
    _check(t, cu, c.D, c.L)


@pytest.mark.parametrize("y_dtype,out_dtype", [(torch.float32, torch.float16), (torch.float32, torch.bfloat16),
                                               (torch.bfloat16, None), (torch.float16, None)])
def test_restore_dtypes(y_dtype, out_dtype):
    c = CONFIGS["c0"]
    ch, t, k, cu = _stream(c)
    _check(t, cu, c.D, c.L, y_dtype, out_dtype)


def _random_stream(NC, L, rho, seed):
    rng = np.random.default_rng(seed)
    ts, cnt = [], []
    for c in range(NC):
        m = rng.random(L) < rho[c % len(rho)]
        tt = np.flatnonzero(m).astype(np.int32)
        ts.append(tt)
        cnt.append(tt.size)
    cu = np.zeros(NC + 1, np.int32)
    cu[1:] = np.cumsum(cnt)
    return np.concatenate(ts), cu


def test_restore_empty_and_dense_channels_and_odd_dims():
    # D not a multiple of 32, empty channels, fully dense channels, ragged L
    t, cu = _random_stream(NC=3 * 37, L=301, rho=[0.0, 1.0, 0.3, 0.02], seed=1)
    _check(t, cu, 37, 301)


def test_restore_search_cap():
    # channels with >= 4096 events: only the first 4095 are addressable
    t, cu = _random_stream(NC=2 * 33, L=5000, rho=[1.0, 0.9, 0.0, 0.5], seed=2)
    assert (cu[1:] - cu[:-1]).max() > 4096
    _check(t, cu, 33, 5000)


def test_restore_long_gaps_cross_parts():
    # very sparse channels: hold intervals span many windows/parts
    t, cu = _random_stream(NC=4 * 64, L=4096, rho=[0.001, 0.0005, 0.01, 0.0], seed=3)
    _check(t, cu, 64, 4096)


def test_restore_errors():
    ops = load_ops()
    ts = torch.zeros(4, dtype=torch.int32, device=dev)
    cu = torch.tensor([0, 4, 4], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="n_channels"):
        ops.restore_dense_fwd(torch.zeros(4, device=dev), ts, cu, 3, 10)
    with pytest.raises(RuntimeError, match="bf16 input only supports bf16 output"):
        ops.restore_dense_fwd(torch.zeros(4, device=dev, dtype=torch.bfloat16), ts, cu, 1, 10, torch.float32)


@pytest.mark.parametrize("dim,L,rho,seed", [
    (36, 5000, [1.0, 0.9, 0.0, 0.5], 4),          # search cap
    (44, 301, [0.0, 1.0, 0.3, 0.02], 5),          # empty / dense channels, ragged L
    (132, 4096, [0.001, 0.0005, 0.01, 0.0], 6),   # two feature blocks (one partial), long gaps
    (4, 97, [0.5], 7),                            # a single 4-feature lane
])
def test_restore_more_shapes(dim, L, rho, seed):
    """More feature counts (partial 32-feature blocks, two blocks, a single
    feature group) through the same edge cases, fp32 and bf16."""
    t, cu = _random_stream(NC=2 * dim, L=L, rho=rho, seed=seed)
    _check(t, cu, dim, L)
    _check(t, cu, dim, L, torch.bfloat16, None, seed=seed)


@pytest.mark.parametrize("B,dm,L,expand,thr", [(1, 1, 1, 1, 0.0), (2, 5, 31, 2, 0.3), (3, 40, 777, 2, 0.5),
                                                (4, 96, 1000, 3, -0.5), (2, 128, 4000, 2, 1.28),
                                                (2, 33, 4095, 2, 0.0)])
def test_restore_from_extraction_mask(B, dm, L, expand, thr):
    """restore_dense_fwd_bitmap(base_mask=) transposes the extraction's
    threshold mask into the event bitmap: the same dense output, bitmap
    buffer (words and sweep start indices) and backward as the bitmap built
    from the event times; ragged shapes, dense and empty streams."""
    ops = load_ops()
    g = torch.Generator().manual_seed(B * 31 + dm + L)
    x = torch.randn(B, L, dm, generator=g).to(dev)
    res, _mx = ops.extract_expanded_events(x, thr, expand, bld=True, keep_mask=True)
    ch, ts, kf, cu = res[:4]
    mask = res[5]
    D = dm * expand
    y = torch.randn(ch.numel(), generator=g).to(dev)
    out_e, bm_e = ops.restore_dense_fwd_bitmap(y, ts, cu, D, L)
    out_m, bm_m = ops.restore_dense_fwd_bitmap(y, ts, cu, D, L, base_mask=mask, expand=expand)
    assert torch.equal(out_m, out_e)
    assert torch.equal(bm_m, bm_e)
    dout = torch.randn(B, L, D, generator=g).to(dev)
    assert torch.equal(ops.restore_dense_bwd_bitmap(dout, ts, cu, bm_m, D, L),
                       ops.restore_dense_bwd_bitmap(dout, ts, cu, bm_e, D, L))


def test_restore_from_extraction_mask_limits():
    ops = load_ops()
    x = torch.randn(1, 4096, 4, device=dev)
    res, _mx = ops.extract_expanded_events(x, 0.0, 2, bld=True, keep_mask=True)
    y = torch.randn(res[0].numel(), device=dev)
    with pytest.raises(RuntimeError, match="seqlen above"):
        ops.restore_dense_fwd_bitmap(y, res[1], res[3], 8, 4096, base_mask=res[5], expand=2)
    with pytest.raises(RuntimeError, match="multiple of expand"):
        ops.restore_dense_fwd_bitmap(y, res[1], res[3], 8, 4096, base_mask=res[5], expand=3)
