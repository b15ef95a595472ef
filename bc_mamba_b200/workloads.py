"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is used: the reference publishes no
kernel benchmark suite, so these stand in for it).

Per configuration (B batch, D = d_model*expand logical features, N states,
L positions, rho spike density):
  * membrane v ~ N(0,1) of shape (B, d_model, L); the threshold is the exact
    (1 - rho) order statistic of v, so ~rho of positions fire (i.i.d.);
    "markov" configs use a per-channel two-state chain with P(on->off) = 1/8
    (on-runs of mean 8) and P(off->on) set for density rho (1/12 at rho =
    0.4), from its stationary start, v in {0, 1}, threshold 0.5;
  * x_conv u ~ N(0,1) of shape (B, D, L);
  * dt_idle, dt_active = softplus(N(0,1) - 1), shape (D,);
  * A = -(1..N) for every feature (A_log = log(1..N), the S4D-real init);
  * W_B, W_C ~ N(0,1), shape (D, N); D skip = 1;
  * upstream gradient dout ~ N(0,1), shape (B, L, D).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    D: int
    N: int
    L: int
    rho: float
    dtype: torch.dtype = torch.float32
    spikes: str = "iid"      # "iid" | "markov"
    seed: int = 0
    expand: int = 2
    blocks: int = 1

    @property
    def d_model(self) -> int:
        return self.D // self.expand

    def with_(self, **kw) -> "Config":
        return replace(self, **kw)


CONFIGS = {
    "c0": Config("c0_tiny", B=2, D=64, N=16, L=256, rho=0.25, seed=0),
    "c1": Config("c1_long", B=32, D=256, N=16, L=2048, rho=0.20, seed=1),
    "c2": Config("c2_bf16", B=16, D=512, N=16, L=4096, rho=0.10, dtype=torch.bfloat16, seed=2),
    "c3": Config("c3_bursty", B=64, D=256, N=64, L=1024, rho=0.40, spikes="markov", seed=3),
    "c4": Config("c4_stack", B=128, D=256, N=16, L=4000, rho=0.10, seed=4, blocks=4),
}


def markov_rates(rho: float = 0.4):
    """(P(off->on), P(on->off)) of the two-state spike chain: on-runs of mean
    length 8 and stationary density rho (rho = 0.4: off-runs of mean 12)."""
    if rho == 0.4:
        return 1.0 / 12.0, 1.0 / 8.0
    return rho / (8.0 * (1.0 - rho)), 1.0 / 8.0


def markov_chain(state: torch.Tensor, r: torch.Tensor, rho: float = 0.4) -> torch.Tensor:
    """Run the chain from `state` (rows,) bool over the uniforms r (rows, L);
    returns the (rows, L) bool on/off path (works on any device)."""
    p_off_on, p_on_off = markov_rates(rho)
    out = torch.empty(r.shape, dtype=torch.bool, device=r.device)
    for t in range(r.shape[1]):
        out[:, t] = state
        flip_off = state & (r[:, t] < p_on_off)
        flip_on = (~state) & (r[:, t] < p_off_on)
        state = (state & ~flip_off) | flip_on
    return out


def _markov(shape, gen, rho: float = 0.4) -> torch.Tensor:
    """Two-state chain per row: on-run mean 8, stationary density rho (0.4:
    off-run mean 12), started from its stationary distribution."""
    rows, L = shape
    p_off_on, p_on_off = markov_rates(rho)
    p_on = p_off_on / (p_off_on + p_on_off)
    state = torch.rand(rows, generator=gen) < p_on
    r = torch.rand(rows, L, generator=gen)
    return markov_chain(state, r, rho)


def spikes_membrane(cfg: Config, gen: torch.Generator):
    """(v, threshold): membrane (B, d_model, L) float32 and the firing threshold."""
    shape = (cfg.B, cfg.d_model, cfg.L)
    if cfg.spikes == "markov":
        v = _markov((cfg.B * cfg.d_model, cfg.L), gen, cfg.rho).reshape(shape).float()
        return v, 0.5
    v = torch.randn(shape, generator=gen)
    n = v.numel()
    kth = max(1, min(n, int(round((1.0 - cfg.rho) * n))))
    thr = float(v.reshape(-1).kthvalue(kth).values)
    return v, thr


def make_inputs(cfg: Config, device="cpu", rank: int = 0) -> dict:
    """All tensors of one step of the pipeline for `cfg` (rank offsets the seed)."""
    gen = torch.Generator().manual_seed(cfg.seed * 1000 + rank)
    v, thr = spikes_membrane(cfg, gen)
    u = torch.randn(cfg.B, cfg.D, cfg.L, generator=gen)
    dt_idle = F.softplus(torch.randn(cfg.D, generator=gen) - 1.0)
    dt_active = F.softplus(torch.randn(cfg.D, generator=gen) - 1.0)
    A = -torch.arange(1, cfg.N + 1, dtype=torch.float32).repeat(cfg.D, 1).contiguous()
    W_B = torch.randn(cfg.D, cfg.N, generator=gen)
    W_C = torch.randn(cfg.D, cfg.N, generator=gen)
    Dskip = torch.ones(cfg.D)
    dout = torch.randn(cfg.B, cfg.L, cfg.D, generator=gen)
    t = dict(v=v, u=u.to(cfg.dtype), dt_idle=dt_idle, dt_active=dt_active, A=A, W_B=W_B,
             W_C=W_C, D=Dskip, dout=dout.to(cfg.dtype))
    out = {k: x.to(device) for k, x in t.items()}
    out["threshold"] = thr
    return out
