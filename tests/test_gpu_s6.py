"""GPU parity of the dense selective scan (bcm_s6_fwd / bcm_s6_bwd through the
shim's selective_scan_cuda.fwd / .bwd, the reference's argument order and
outputs) against the float64 oracle (oracle/s6.py, itself pinned to the
reference's selective_scan_ref), against the reference's golden vectors, and
against the reference's own compiled fwd/bwd (oracle/_ref; skipped when not
built).  Fixed and variable (grouped) B / C, D, the z gate, delta_bias and
softplus, every lane layout (dstate 1 .. 256), sequences across the
2048-position chunk boundary, 16-bit inputs.  Tolerance 1e-5 (fp32) / 2e-2
(16-bit) relative to the largest magnitude, as tests/helpers.py."""
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import TOL_16, TOL_F32, assert_close
from oracle import s6
from bc_mamba_b200 import load_ops

pytestmark = pytest.mark.gpu
dev = "cuda"
GOLD = Path(__file__).resolve().parent / "golden"


def _inputs(b, d, L, N, bk, ck, groups, has_d, has_z, has_bias, softplus, seed):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, d, L, generator=g)
    delta = (0.5 * torch.randn(b, d, L, generator=g) - 1.0) if softplus else \
        (0.01 + 0.2 * torch.rand(b, d, L, generator=g))
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(d, 1) * (0.5 + torch.rand(d, 1, generator=g))
    B = torch.randn(d, N, generator=g) if bk == "fixed" else torch.randn(b, groups, N, L, generator=g)
    C = torch.randn(d, N, generator=g) if ck == "fixed" else torch.randn(b, groups, N, L, generator=g)
    D = torch.randn(d, generator=g) if has_d else None
    z = torch.randn(b, d, L, generator=g) if has_z else None
    # without softplus delta' = delta + bias must stay positive (decaying states)
    bias = (0.3 * torch.randn(d, generator=g) if softplus else 0.05 * torch.rand(d, generator=g)) \
        if has_bias else None
    dout = torch.randn(b, d, L, generator=g)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=bias, dout=dout, softplus=softplus)


def _np(t):
    return None if t is None else t.float().numpy()


def _run(inp, dtype=torch.float32, tol=TOL_F32):
    ops = load_ops()
    to = lambda t, dt=dtype: None if t is None else t.to(dt).to(dev)
    var_b, var_c = inp["B"].dim() >= 3, inp["C"].dim() >= 3
    u, delta, z, dout = to(inp["u"]), to(inp["delta"]), to(inp["z"]), to(inp["dout"])
    A = to(inp["A"], torch.float32)
    B = to(inp["B"], dtype if var_b else torch.float32)
    C = to(inp["C"], dtype if var_c else torch.float32)
    D, bias = to(inp["D"], torch.float32), to(inp["delta_bias"], torch.float32)
    sp = inp["softplus"]
    res = ops.fwd(u, delta, A, B, C, D, z, bias, sp)
    # the oracle on the values the kernel sees (16-bit inputs rounded)
    ref_in = [_np(x.cpu()) for x in (u, delta, A, B, C)]
    kw = dict(D=_np(inp["D"]), z=None if z is None else _np(z.cpu()), delta_bias=_np(inp["delta_bias"]),
              delta_softplus=sp)
    out, x, out_z, _ = s6.s6_fwd(*ref_in, **kw)
    assert_close(res[0], out, tol, "out")
    assert_close(res[1], x, tol, "x")
    if z is not None:
        assert_close(res[2], out_z, tol, "out_z")
    g = ops.bwd(u, delta, A, B, C, D, z, bias, dout, res[1], res[0] if z is not None else None, None, sp,
                z is not None)
    ref = s6.s6_bwd(*ref_in, _np(dout.cpu()), **kw)
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"]
    for n, a in zip(names, g[:7]):
        if ref[n] is None:
            assert a is None, n
        else:
            assert_close(a, ref[n], tol, n)
    if z is not None:
        assert_close(g[7], ref["dz"], tol, "dz")
        assert_close(g[8], out_z, tol, "recomputed out_z")
    return res, g


@pytest.mark.parametrize("N", [1, 3, 4, 8, 16, 17, 32, 33, 64, 100, 256])
def test_s6_dstates(N):
    _run(_inputs(2, 5, 130, N, "var", "var", 1, True, False, True, True, seed=N))


@pytest.mark.parametrize("bk,ck,groups", [("fixed", "fixed", 1), ("var", "var", 2), ("fixed", "var", 1),
                                          ("var", "fixed", 6), ("var", "var", 6)])
def test_s6_bc_modes(bk, ck, groups):
    _run(_inputs(2, 6, 257, 16, bk, ck, groups, True, True, True, True, seed=groups * 7))


@pytest.mark.parametrize("has_d,has_z,has_bias,softplus", [(False, False, False, False), (True, True, False, False),
                                                           (False, True, True, True), (True, False, True, False)])
def test_s6_options(has_d, has_z, has_bias, softplus):
    _run(_inputs(3, 4, 96, 16, "var", "var", 2, has_d, has_z, has_bias, softplus, seed=11))


@pytest.mark.parametrize("L", [1, 31, 32, 33, 2048, 2100])
def test_s6_lengths(L):
    _run(_inputs(1, 4, L, 16, "var", "fixed", 1, True, True, True, True, seed=L))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_s6_16bit(dtype):
    _run(_inputs(2, 8, 300, 16, "var", "var", 2, True, True, True, True, seed=21), dtype=dtype, tol=TOL_16)


@pytest.mark.parametrize("name", ["fixed", "var_groups", "mixed_n4", "var_b_fixed_c"])
def test_s6_reference_golden(name):
    """The reference's own selective_scan_ref outputs and gradients."""
    f = np.load(GOLD / f"s6_ref_{name}.npz")
    r = {k: f[k] for k in f.files}
    ops = load_ops()
    T_ = lambda k: torch.as_tensor(r[k]).to(dev) if k in r else None
    u, delta, A, B, C, D, z, bias = (T_(k) for k in ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"])
    sp = bool(r["softplus"])
    res = ops.fwd(u, delta, A, B, C, D, z, bias, sp)
    assert_close(res[2] if z is not None else res[0], r["out"], TOL_F32, "out")
    g = ops.bwd(u, delta, A, B, C, D, z, bias, T_("dout"), res[1], res[0] if z is not None else None, None, sp,
                False)
    got = dict(zip(["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"], g[:7]))
    if z is not None:
        got["dz"] = g[7]
    for k, v in got.items():
        if k in r:   # the fixture holds the gradient of every input it was given
            assert_close(v, r[k], TOL_F32, k)
        else:
            assert v is None, k


def test_s6_against_reference_cuda():
    """The reference's compiled selective_scan_cuda.fwd/bwd on the same inputs."""
    from oracle import build_ref
    ref = build_ref.load("selective_scan_cuda")
    if ref is None:
        pytest.skip("reference CUDA extensions not built (python oracle/build_ref.py)")
    ops = load_ops()
    for spec, seed in [((2, 16, 1000, 16, "var", "var", 1, True, True, True, True), 31),
                       ((2, 8, 2500, 16, "fixed", "fixed", 1, True, False, False, False), 32),
                       ((1, 12, 600, 4, "var", "fixed", 3, False, True, True, True), 33)]:
        inp = _inputs(*spec, seed=seed)
        args = [None if inp[k] is None else inp[k].to(dev) for k in ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]]
        sp = inp["softplus"]
        mine = ops.fwd(*args, sp)
        theirs = ref.fwd(*args, sp)
        for a, b, n in zip(mine, theirs, ["out", "x", "out_z"]):
            assert_close(a, b.cpu().numpy(), TOL_F32, n)
        dout = inp["dout"].to(dev)
        has_z = inp["z"] is not None
        gm = ops.bwd(*args, dout, mine[1], mine[0] if has_z else None, None, sp, False)
        gt = ref.bwd(*args, dout, theirs[1], theirs[0] if has_z else None, None, sp, False)
        for a, b, n in zip(gm, gt, ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias", "dz"]):
            if b is None:
                assert a is None, n
            else:
                assert_close(a, b.cpu().numpy(), TOL_F32, n)


def test_s6_errors():
    """The reference binding's checks: dstate, complex weights, dtypes, and
    (n_groups taken from B) a grouped variable C beside a fixed B."""
    ops = load_ops()
    u = torch.randn(1, 4, 10, device=dev)
    A = -torch.ones(4, 8, device=dev)
    B = torch.randn(4, 8, device=dev)
    with pytest.raises(RuntimeError, match="state dimension <= 256"):
        ops.fwd(u, u, -torch.ones(4, 300, device=dev), torch.randn(4, 300, device=dev),
                torch.randn(4, 300, device=dev), None, None, None, False)
    with pytest.raises(RuntimeError, match="complex weights"):
        ops.fwd(u, u, A.to(torch.complex64), B.to(torch.complex64), B.to(torch.complex64), None, None, None, False)
    with pytest.raises(RuntimeError):
        ops.fwd(u, u.half(), A, B, B, None, None, None, False)
    with pytest.raises(RuntimeError, match="C must have shape"):
        ops.fwd(u, u, A, B, torch.randn(1, 2, 8, 10, device=dev), None, None, None, False)
