"""GPU parity: flat-channel sparse selective scan forward/backward through the
drop-in ``selective_scan_cuda.fwd_flat_ch / bwd_flat_ch`` against
  (1) golden vectors from the reference's own selective_scan_ref, and
  (2) the float64 oracle (oracle/scan.py) for every B/C mode, dstate, chunking
      and dtype.
Tolerance: |x - ref| <= tol*|ref| + tol*max|ref|, tol = 1e-5 (fp32 u) or
2e-2 (bf16/fp16 u); fp32 parameters and state throughout."""
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32, assert_close
from oracle import events as ev
from oracle import scan as sc
from bc_mamba_b200 import load_ops
from bc_mamba_b200.workloads import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


def T(x, dtype=None):
    t = torch.as_tensor(np.asarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev).contiguous()


@pytest.mark.parametrize("name", ["c0_depthwise", "c0_legacy_bc", "c0_depthwise_z", "small_n4_sparse"])
def test_scan_vs_reference_golden(name):
    """Against the reference's selective_scan_ref run on the same inputs."""
    f = np.load(GOLDEN / f"scan_ref_{name}.npz")
    ops = load_ops()
    legacy = "B" in f
    B = T(f["B"] if legacy else f["W_B"])
    C = T(f["C"] if legacy else f["W_C"])
    z = T(f["z_flat"]) if "z_flat" in f else None
    args = (T(f["u_flat"]), T(f["k_flat"]), T(f["cu_seqlens"]), int(f["max_seqlen"]),
            T(f["dt_idle"]), T(f["dt_active"]), T(f["A"]), B, C)
    res = ops.fwd_flat_ch(*args, T(f["D"]), z, None, 0, not legacy)
    prim = res[2] if z is not None else res[0]
    assert_close(prim, f["out_flat"], TOL_F32, "out")
    g = ops.bwd_flat_ch(*args, T(f["dout_flat"]), res[1], T(f["D"]), z, res[0] if z is not None else None,
                        None, 0, not legacy)
    names = ["du", "dA", "dB" if legacy else "dW_B", "dC" if legacy else "dW_C", "ddt_idle", "ddt_active", "dD"]
    if z is not None:
        names.append("dz")
    for got, n in zip(g, names):
        assert_close(got, f[n], TOL_F32, n)


def _events(cfg):
    inp = make_inputs(cfg)
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(inp["v"].numpy(), inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, cfg.B, cfg.d_model, cfg.expand)
    u = ev.gather_events_fwd(inp["u"].float().numpy(), ch, t)
    return inp, ch, t, k, cu, int(mx), u


def _run_and_check(u, k, cu, mx, dti, dta, A, B, C, D=None, z=None, toff=None, dw=True,
                   pw=None, dtype=torch.float32, tol=TOL_F32, seed=0, fp32_decay=False):
    ops = load_ops()
    g = torch.Generator().manual_seed(seed)
    E = u.size
    u16 = torch.as_tensor(u, dtype=torch.float32).to(dtype)
    u_ref = u16.float().numpy()  # the values the kernel actually sees
    zt = None if z is None else torch.as_tensor(z, dtype=torch.float32).to(dtype)
    z_ref = None if z is None else zt.float().numpy()
    pwB, pwC = (None, None) if pw is None else pw
    args = (u16.to(dev), T(k), T(cu), mx, T(dti), T(dta), T(A), T(B), T(C))
    Dt = None if D is None else T(D)
    res = ops.fwd_flat_ch(*args, Dt, None if zt is None else zt.to(dev),
                          None if toff is None else T(toff), 0, dw,
                          None if pwB is None else T(pwB), None if pwC is None else T(pwC))
    out, x, oz = sc.scan_fwd(u_ref, k, cu, mx, dti, dta, A, B, C, D=D, z=z_ref, tile_offsets=toff,
                             is_depthwise_bc=dw, pw_B=pwB, pw_C=pwC, fp32_decay=fp32_decay)
    assert_close(res[0], out, tol, "out")
    assert_close(res[1], x, tol, "x")
    if z is not None:
        assert_close(res[2], oz, tol, "out_z")
    dout = torch.randn(E, generator=g).to(dtype)
    gr = ops.bwd_flat_ch(*args, dout.to(dev), res[1], Dt, None if zt is None else zt.to(dev),
                         res[0] if z is not None else None, None if toff is None else T(toff), 0, dw,
                         None if pwB is None else T(pwB), None if pwC is None else T(pwC))
    ref = sc.scan_bwd(u_ref, k, cu, mx, dti, dta, A, B, C, dout.float().numpy(), D=D, z=z_ref,
                      out=res[0].float().cpu().numpy(), tile_offsets=toff, is_depthwise_bc=dw,
                      pw_B=pwB, pw_C=pwC, fp32_decay=fp32_decay)
    names = ["du", "dA", "dB", "dC", "ddt_idle", "ddt_active", "dD", "dz", "dpw_B", "dpw_C"]
    names = names[:6] + (["dD"] if D is not None else []) + (["dz"] if z is not None else []) + \
        (["dpw_B", "dpw_C"] if pw is not None else [])
    assert len(gr) == len(ref) == len(names)
    for a, b, n in zip(gr, ref, names):
        assert_close(a, b, tol, n)
    # the forward that also keeps the state checkpoints, and the backward that
    # reads them instead of re-running the recurrence (staged kernels only)
    res_ck = ops.fwd_flat_ch_ckpt(*args, Dt, None if zt is None else zt.to(dev),
                                  None if toff is None else T(toff), 0, dw,
                                  None if pwB is None else T(pwB), None if pwC is None else T(pwC))
    assert len(res_ck) == len(res) + 1
    for a, b in zip(res_ck[:-1], res):
        assert torch.equal(a, b)
    ck = res_ck[-1]
    if ck.numel() > 0:
        gr_ck = ops.bwd_flat_ch(*args, dout.to(dev), res[1], Dt, None if zt is None else zt.to(dev),
                                res[0] if z is not None else None, None if toff is None else T(toff), 0, dw,
                                None if pwB is None else T(pwB), None if pwC is None else T(pwC), ck)
        for a, b, n in zip(gr_ck, ref, names):
            assert_close(a, b, tol, n + " (forward checkpoints)")
        if mx <= 2048:   # one chunk: the same states as the recomputation, bit for bit
            for a, b, n in zip(gr_ck, gr, names):
                assert torch.equal(a, b), n
    return res, gr


def _params(D, N, seed):
    rng = np.random.default_rng(seed)
    sp = lambda x: np.log1p(np.exp(x))
    return (sp(rng.standard_normal(D) - 1).astype(np.float32), sp(rng.standard_normal(D) - 1).astype(np.float32),
            -np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1)),
            rng.standard_normal((D, N)).astype(np.float32), rng.standard_normal((D, N)).astype(np.float32),
            np.ones(D, np.float32))


def test_depthwise_c0_vs_oracle():
    c = CONFIGS["c0"]
    inp, ch, t, k, cu, mx, u = _events(c)
    p = lambda n: inp[n].numpy()
    _run_and_check(u, k, cu, mx, p("dt_idle"), p("dt_active"), p("A"), p("W_B"), p("W_C"), D=p("D"))


def test_depthwise_c0_bf16():
    c = CONFIGS["c0"]
    inp, ch, t, k, cu, mx, u = _events(c)
    p = lambda n: inp[n].numpy()
    _run_and_check(u, k, cu, mx, p("dt_idle"), p("dt_active"), p("A"), p("W_B"), p("W_C"), D=p("D"),
                   dtype=torch.bfloat16, tol=TOL_16)


@pytest.mark.parametrize("N", [1, 3, 4, 8, 16, 32, 64, 100, 128, 256])
def test_dstate_layouts(N):
    c = CONFIGS["c0"].with_(B=1, D=16, N=N, L=300, rho=0.3, seed=11)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, N, N)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


def test_no_D_and_gate_and_pointwise():
    c = CONFIGS["c0"].with_(B=2, D=24, N=16, L=200, rho=0.3, seed=12)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 3)
    rng = np.random.default_rng(4)
    z = rng.standard_normal(u.size).astype(np.float32)
    pw = (0.2 * rng.standard_normal((c.D, c.D))).astype(np.float32), (0.2 * rng.standard_normal((c.D, c.D))).astype(np.float32)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=None)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv, z=z)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv, z=z, pw=pw)


def test_legacy_per_event_bc():
    c = CONFIGS["c0"].with_(B=2, D=16, N=16, L=300, rho=0.25, seed=13)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, _, _, Dv = _params(c.D, c.N, 5)
    rng = np.random.default_rng(6)
    Bev = rng.standard_normal((c.N, u.size)).astype(np.float32)
    Cev = rng.standard_normal((c.N, u.size)).astype(np.float32)
    _run_and_check(u, k, cu, mx, dti, dta, A, Bev, Cev, D=Dv, dw=False)
    z = rng.standard_normal(u.size).astype(np.float32)
    _run_and_check(u, k, cu, mx, dti, dta, A, Bev, Cev, D=Dv, z=z, dw=False)


@pytest.mark.parametrize("rho", [0.1, 0.45])
def test_tiled_bc(rho):
    c = CONFIGS["c0"].with_(B=2, D=8, N=8, L=1200, rho=rho, seed=14)
    inp, ch, t, k, cu, mx, u = _events(c)
    dti, dta, A, _, _, Dv = _params(c.D, c.N, 7)
    cs = sc.ref_chunk_size(mx)
    n = cu[1:] - cu[:-1]
    tiles = (n + cs - 1) // cs
    toff = np.zeros(n.size, np.int32)
    toff[1:] = np.cumsum(tiles)[:-1]
    rng = np.random.default_rng(8)
    Bt = rng.standard_normal((int(tiles.sum()), c.N, cs)).astype(np.float32)
    Ct = rng.standard_normal((int(tiles.sum()), c.N, cs)).astype(np.float32)
    _run_and_check(u, k, cu, mx, dti, dta, A, Bt, Ct, D=Dv, toff=toff, dw=False)


def test_multi_chunk_channels():
    """Channels with > 2048 events: chunk states in x and the backward restart.

    Small dt (memory of ~300 events at a ~ 0.997) and near-uniform gaps make the
    fp32 rounding of the per-gap decay compound coherently, so the oracle uses
    the fp32 decays the reference kernel forms (fp32_decay=True); the
    remaining arithmetic is float64."""
    c = CONFIGS["c0"].with_(B=1, D=6, N=16, L=7000, rho=0.9, seed=15)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 4096
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 9)
    dti = dti * 0.01
    dta = dta * 0.01
    res, _ = _run_and_check(u, k, cu, mx, dti, dta, A, 0.3 * WB, 0.3 * WC, D=Dv, fp32_decay=True)
    assert res[1].shape[1] == (mx + 2047) // 2048


def test_multi_chunk_short_memory_exact_decay():
    """Multi-chunk channels with the model's typical dt: float64 decays."""
    c = CONFIGS["c0"].with_(B=1, D=4, N=16, L=6000, rho=0.8, seed=16)
    inp, ch, t, k, cu, mx, u = _events(c)
    assert mx > 2048
    dti, dta, A, WB, WC, Dv = _params(c.D, c.N, 10)
    _run_and_check(u, k, cu, mx, dti, dta, A, WB, WC, D=Dv)


@pytest.mark.parametrize("max_len", [127, 128, 129, 256, 257, 512, 513, 1024, 1025, 2048, 2049])
def test_seqlen_dispatch_boundaries(max_len):
    rng = np.random.default_rng(max_len)
    NC, D, N = 8, 4, 16
    n = rng.integers(0, max_len + 1, NC)
    n[0] = max_len
    cu = np.zeros(NC + 1, np.int32)
    cu[1:] = np.cumsum(n)
    k = rng.integers(1, 6, int(cu[-1])).astype(np.int32)
    u = rng.standard_normal(int(cu[-1])).astype(np.float32)
    dti, dta, A, WB, WC, Dv = _params(D, N, 1)
    _run_and_check(u, k, cu, int(max_len), 0.05 * dti, 0.05 * dta, A, 0.5 * WB, 0.5 * WC, D=Dv)


def test_empty_channels_and_no_events():
    ops = load_ops()
    dti, dta, A, WB, WC, Dv = _params(4, 16, 2)
    cu = np.array([0, 0, 3, 3, 5, 5, 5, 9, 9], np.int32)
    rng = np.random.default_rng(3)
    u = rng.standard_normal(9).astype(np.float32)
    k = rng.integers(1, 4, 9).astype(np.int32)
    _run_and_check(u, k, cu, 4, dti, dta, A, WB, WC, D=Dv)
    # E == 0: outputs are empty, parameter gradients are zero
    e = torch.zeros(0, device=dev)
    args = (e, torch.zeros(0, dtype=torch.int32, device=dev), T(np.zeros(9, np.int32)), 0, T(dti), T(dta),
            T(A), T(WB), T(WC))
    out, x = ops.fwd_flat_ch(*args, T(Dv), None, None, 0, True)
    assert out.numel() == 0 and x.shape == (8, 1, 32) and float(x.abs().sum()) == 0.0
    g = ops.bwd_flat_ch(*args, e, x, T(Dv), None, None, None, 0, True)
    assert all(float(t.abs().sum()) == 0.0 for t in g[1:])


def test_scan_argument_errors():
    ops = load_ops()
    dti, dta, A, WB, WC, Dv = _params(4, 16, 2)
    u = torch.zeros(3, device=dev)
    k = torch.ones(3, dtype=torch.int32, device=dev)
    cu = torch.tensor([0, 3], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="A must be float32"):
        ops.fwd_flat_ch(u, k, cu, 3, T(dti), T(dta), T(A).double(), T(WB), T(WC), None, None, None, 0, True)
    with pytest.raises(RuntimeError, match="W_B must be"):
        ops.fwd_flat_ch(u, k, cu, 3, T(dti), T(dta), T(A), T(WB)[:, :8].contiguous(), T(WC), None, None, None, 0, True)
    with pytest.raises(RuntimeError, match="dstate must be <= 256"):
        A2 = torch.zeros(4, 300, device=dev)
        ops.fwd_flat_ch(u, k, cu, 3, T(dti), T(dta), A2, A2, A2, None, None, None, 0, True)
    with pytest.raises(RuntimeError, match="x.size\\(1\\) must equal n_chunks"):
        x = torch.zeros(1, 2, 32, device=dev)
        ops.bwd_flat_ch(u, k, cu, 3, T(dti), T(dta), T(A), T(WB), T(WC), u, x, None, None, None, None, 0, True)
