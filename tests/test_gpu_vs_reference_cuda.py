"""GPU parity against the reference's own CUDA extensions, compiled from its
sources into oracle/_ref (oracle/build_ref.py), on identical seeded inputs.
Event streams, expansion, gather and the restore map are compared bit-exactly;
the restore backward (reference: fp32 atomics) and the scan within 1e-5 (fp32)
or 2e-2 (bf16).  Skipped when oracle/_ref was not built."""
import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32, assert_close, assert_exact
from oracle import build_ref
from bc_mamba_b200 import load_ops
from bc_mamba_b200.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.fixture(scope="module")
def ref():
    mods = {n: build_ref.load(n) for n in build_ref.SOURCES}
    if any(m is None for m in mods.values()):
        pytest.skip("reference CUDA extensions not built (python oracle/build_ref.py)")
    return mods


# one block of configs[4] at the top of its density sweep with bursty spikes:
# B = 128, L = 4000, rho = 0.5 Markov: about a quarter of the channels hold
# more than 2048 events (two chunk states)
VARIANTS = {"c4_markov50": ("c4", dict(rho=0.5, spikes="markov"))}


def _run_both(ref, cfg_name, rho=None):
    if cfg_name in VARIANTS:
        base, kw = VARIANTS[cfg_name]
        cfg = CONFIGS[base].with_(**kw)
    else:
        cfg = CONFIGS[cfg_name] if rho is None else CONFIGS[cfg_name].with_(rho=rho)
    ops = load_ops()
    inp = make_inputs(cfg, device=dev)
    ee = ref["extract_events_cuda"]
    base = inp["v"].contiguous()
    ours = ops.extract_base_events(base, inp["threshold"])
    theirs = ee.extract_base_events(base, inp["threshold"])
    for a, b, n in zip(ours, theirs, ["ch", "t", "k", "cu", "counts", "max"]):
        assert_exact(a, b, "extract " + n)
    ex_o = ops.expand_base_events(*ours[:4], cfg.B, cfg.d_model, cfg.expand)
    ex_t = ee.expand_base_events(*theirs[:4], cfg.B, cfg.d_model, cfg.expand)
    for a, b, n in zip(ex_o, ex_t, ["ch", "t", "k", "cu", "max"]):
        assert_exact(a, b, "expand " + n)
    ch, ts, kf, cu, mx = ex_o
    uf = ops.gather_events_fwd(inp["u"], ch, ts)[0]
    assert_exact(uf, ee.gather_events_fwd(inp["u"], ch, ts)[0], "gather fwd")
    g = torch.randn(uf.shape, device=dev).to(uf.dtype)
    assert_exact(ops.gather_events_bwd(g, ch, ts, cfg.B * cfg.D, cfg.L)[0],
                 ee.gather_events_bwd(g, ch, ts, cfg.B * cfg.D, cfg.L)[0], "gather bwd")
    return cfg, inp, ch, ts, kf, cu, int(mx), uf


@pytest.mark.parametrize("cfg_name", ["c0", "c1", "c2", "c3", "c4_markov50"])
def test_against_reference_cuda(ref, cfg_name):
    cfg, inp, ch, ts, kf, cu, mx, uf = _run_both(ref, cfg_name)
    if cfg_name == "c4_markov50":
        assert mx > 2048   # multi-chunk channels are exercised
    ops = load_ops()
    ss = ref["selective_scan_cuda"]
    rd = ref["restore_dense_cuda_nodecay"]
    tol = TOL_F32 if cfg.dtype == torch.float32 else TOL_16
    ps = [inp[n] for n in ["dt_idle", "dt_active", "A", "W_B", "W_C"]]
    out_o, x_o = ops.fwd_flat_ch(uf, kf, cu, mx, *ps, inp["D"], None, None, 0, True)
    out_t, x_t = ss.fwd_flat_ch(uf, kf, cu, mx, *ps, inp["D"], None, None, 0, True)
    assert_close(out_o, out_t.float().cpu().numpy(), tol, "scan out")
    assert_close(x_o, x_t.cpu().numpy(), tol, "scan x")
    dense_o = ops.restore_dense_fwd(out_o, ts, cu, cfg.D, cfg.L)
    dense_t = rd.restore_dense_fwd(out_o, ts, cu, cfg.D, cfg.L)
    assert_exact(dense_o, dense_t, "restore fwd")
    dy_o = ops.restore_dense_bwd(inp["dout"], ts, cu, cfg.D, cfg.L)
    dy_t = rd.restore_dense_bwd(inp["dout"], ts, cu, cfg.D, cfg.L)
    assert_close(dy_o, dy_t.cpu().numpy(), TOL_F32, "restore bwd")
    dy = dy_o.to(out_o.dtype)
    g_o = ops.bwd_flat_ch(uf, kf, cu, mx, *ps, dy, x_o, inp["D"], None, None, None, 0, True)
    g_t = ss.bwd_flat_ch(uf, kf, cu, mx, *ps, dy, x_t, inp["D"], None, None, None, 0, True)
    # At c4_markov50 every parameter gradient entry sums ~256k events (128 rows
    # x ~2000 events).  This build's two scan kernel families (sequential
    # per-channel walk, and event-parallel scan) agree with each other there
    # to 1.3e-6 of the largest entry, while the reference's fp32 atomics land
    # up to 1e-5 of it away from both; the reduced gradients are compared at
    # 3e-5 for that case, every per-event output at the usual tolerance.
    big = cfg_name == "c4_markov50"
    for a, b, n in zip(g_o, g_t, ["du", "dA", "dW_B", "dW_C", "ddt_idle", "ddt_active", "dD"]):
        assert_close(a, b.float().cpu().numpy(), 3e-5 if (big and n != "du") else tol, n)


def test_against_reference_cuda_legacy_bc(ref):
    cfg, inp, ch, ts, kf, cu, mx, uf = _run_both(ref, "c0")
    ops = load_ops()
    ss = ref["selective_scan_cuda"]
    E = uf.numel()
    gen = torch.Generator(device="cpu").manual_seed(3)
    B = torch.randn(cfg.N, E, generator=gen).to(dev)
    C = torch.randn(cfg.N, E, generator=gen).to(dev)
    z = torch.randn(E, generator=gen).to(dev)
    ps = [inp[n] for n in ["dt_idle", "dt_active", "A"]]
    r_o = ops.fwd_flat_ch(uf, kf, cu, mx, *ps, B, C, inp["D"], z, None, 0, False)
    r_t = ss.fwd_flat_ch(uf, kf, cu, mx, *ps, B, C, inp["D"], z, None, 0, False)
    for a, b, n in zip(r_o, r_t, ["out", "x", "out_z"]):
        assert_close(a, b.cpu().numpy(), TOL_F32, n)
    dout = torch.randn(E, generator=gen).to(dev)
    g_o = ops.bwd_flat_ch(uf, kf, cu, mx, *ps, B, C, dout, r_o[1], inp["D"], z, r_o[0], None, 0, False)
    g_t = ss.bwd_flat_ch(uf, kf, cu, mx, *ps, B, C, dout, r_t[1], inp["D"], z, r_t[0], None, 0, False)
    for a, b, n in zip(g_o, g_t, ["du", "dA", "dB", "dC", "ddt_idle", "ddt_active", "dD", "dz"]):
        assert_close(a, b.cpu().numpy(), TOL_F32, n)


def test_against_reference_cuda_restore_cap(ref):
    """Channels with more than 4095 events: both sides cap the search."""
    ops = load_ops()
    rd = ref["restore_dense_cuda_nodecay"]
    L, D, B = 5000, 8, 2
    rng = np.random.default_rng(0)
    ts_l, cnt = [], []
    for c in range(B * D):
        m = rng.random(L) < (1.0 if c % 3 == 0 else 0.3)
        tt = np.flatnonzero(m).astype(np.int32)
        ts_l.append(tt)
        cnt.append(tt.size)
    cu = torch.as_tensor(np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32), device=dev)
    ts = torch.as_tensor(np.concatenate(ts_l), device=dev)
    y = torch.randn(ts.numel(), device=dev)
    assert_exact(ops.restore_dense_fwd(y, ts, cu, D, L), rd.restore_dense_fwd(y, ts, cu, D, L), "fwd")
    dout = torch.randn(B, L, D, device=dev)
    assert_close(ops.restore_dense_bwd(dout, ts, cu, D, L), rd.restore_dense_bwd(dout, ts, cu, D, L).cpu().numpy(),
                 TOL_F32, "bwd")
