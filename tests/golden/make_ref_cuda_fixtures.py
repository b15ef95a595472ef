"""Generate golden vectors from the reference's own CUDA extensions.

Runs on a GPU box with the extensions built by oracle/build_ref.py (from the
reference sources) present in oracle/_ref:
    python tests/golden/make_ref_cuda_fixtures.py <outdir>
It writes ref_cuda_<case>.npz with the inputs and the reference outputs of
extract_base_events, expand_base_events, gather_events_fwd,
restore_dense_fwd/bwd and fwd_flat_ch/bwd_flat_ch (depthwise) for small
seeded cases; the CPU tests pin the oracle to them (event streams and the
restore map bit-exactly).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from bc_mamba_b200.workloads import CONFIGS, make_inputs  # noqa: E402
from oracle import build_ref  # noqa: E402


def case(name, cfg, outdir: Path):
    ee = build_ref.load("extract_events_cuda")
    ss = build_ref.load("selective_scan_cuda")
    rd = build_ref.load("restore_dense_cuda_nodecay")
    dev = "cuda"
    inp = make_inputs(cfg, device=dev)
    v = inp["v"].contiguous()
    bch, bt, bk, bcu, counts, bmx = ee.extract_base_events(v, inp["threshold"])
    ch, ts, kf, cu, mx = ee.expand_base_events(bch, bt, bk, bcu, cfg.B, cfg.d_model, cfg.expand)
    uf = ee.gather_events_fwd(inp["u"], ch, ts)[0]
    ps = [inp[n] for n in ["dt_idle", "dt_active", "A", "W_B", "W_C"]]
    out, x = ss.fwd_flat_ch(uf, kf, cu, int(mx), *ps, inp["D"], None, None, 0, True)
    dense = rd.restore_dense_fwd(out, ts, cu, cfg.D, cfg.L)
    dy = rd.restore_dense_bwd(inp["dout"], ts, cu, cfg.D, cfg.L)
    g = ss.bwd_flat_ch(uf, kf, cu, int(mx), *ps, dy.to(out.dtype), x, inp["D"], None, None, None, 0, True)
    c = lambda t: t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()
    rec = dict(v=c(v), threshold=np.float64(inp["threshold"]), u=c(inp["u"]), dout=c(inp["dout"]),
               B=cfg.B, d_model=cfg.d_model, expand=cfg.expand, D=cfg.D, L=cfg.L,
               dt_idle=c(ps[0]), dt_active=c(ps[1]), A=c(ps[2]), W_B=c(ps[3]), W_C=c(ps[4]), Dskip=c(inp["D"]),
               base_ch=c(bch), base_t=c(bt), base_k=c(bk), base_cu=c(bcu), base_counts=c(counts),
               base_max=c(bmx), ch=c(ch), t=c(ts), k=c(kf), cu=c(cu), max_seqlen=c(mx), u_flat=c(uf),
               out=c(out), x=c(x), dense=c(dense), dy=c(dy), du=c(g[0]), dA=c(g[1]), dW_B=c(g[2]),
               dW_C=c(g[3]), ddt_idle=c(g[4]), ddt_active=c(g[5]), dD=c(g[6]))
    np.savez_compressed(outdir / f"ref_cuda_{name}.npz", **rec)
    print("wrote", name, int(ch.numel()))


def main():
    outdir = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
    outdir.mkdir(parents=True, exist_ok=True)
    c0 = CONFIGS["c0"]
    case("c0", c0, outdir)
    case("markov_small", CONFIGS["c3"].with_(B=2, D=32, N=16, L=300), outdir)
    case("sparse_small", c0.with_(B=2, D=16, L=700, rho=0.03, seed=21), outdir)


if __name__ == "__main__":
    main()
