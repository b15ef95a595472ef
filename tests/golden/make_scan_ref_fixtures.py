"""Generate golden vectors for the scan from the reference's own pure-PyTorch
scan, ``selective_scan_ref`` (spike_mamba/selective_scan_interface.py:708-774).

Run in the build container, where the reference is mounted read-only:
    python tests/golden/make_scan_ref_fixtures.py [/path/to/reference]
The reference module imports mamba_ssm / selective_scan_cuda at top level
(:5, :18, :20), which are not installed; stub modules satisfy those imports
and nothing else from them is used.  The event stream comes from the numpy
restatement of extraction (oracle/events.py, itself pinned by known answers),
the scan runs through the reference function on event-compacted tensors
(construction documented in oracle/scan_ref.py), forward plus autograd
backward, in float32.  Output: tests/golden/scan_ref_*.npz.
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from bc_mamba_b200.workloads import CONFIGS, make_inputs  # noqa: E402
from oracle import events as ev  # noqa: E402


def import_reference(ref_root: Path):
    stub_names = ["mamba_ssm", "mamba_ssm.utils", "mamba_ssm.utils.torch", "mamba_ssm.ops",
                  "mamba_ssm.ops.triton", "mamba_ssm.ops.triton.layer_norm", "selective_scan_cuda"]
    for n in stub_names:
        sys.modules.setdefault(n, types.ModuleType(n))
    sys.modules["mamba_ssm.utils.torch"].custom_fwd = lambda *a, **k: (a[0] if a and callable(a[0]) else (lambda f: f))
    sys.modules["mamba_ssm.utils.torch"].custom_bwd = lambda *a, **k: (a[0] if a and callable(a[0]) else (lambda f: f))
    sys.modules["mamba_ssm.ops.triton.layer_norm"]._layer_norm_fwd = None
    sys.path.insert(0, str(ref_root / "spike_mamba"))
    import selective_scan_interface as ssi  # noqa: E402
    return ssi


def make_case(ssi, name, cfg, legacy_bc=False, with_z=False, dense_seed=123):
    inp = make_inputs(cfg)
    v = inp["v"].numpy()
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(v, inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, cfg.B, cfg.d_model, cfg.expand)
    u = inp["u"].float().numpy()
    u_flat = ev.gather_events_fwd(u, ch, t).astype(np.float32)
    E = u_flat.size
    n = cu[1:] - cu[:-1]
    Lmax = int(n.max())
    j = np.arange(Lmax)
    mask = j[None, :] < n[:, None]
    idx = np.where(mask, cu[:-1, None] + j[None, :], 0)
    shp = (cfg.B, cfg.D, Lmax)

    u_c = torch.tensor(u_flat[idx] * mask, dtype=torch.float32).reshape(shp).requires_grad_(True)
    km1 = torch.tensor((k[idx] - 1) * mask, dtype=torch.float32).reshape(shp)
    m = torch.tensor(mask, dtype=torch.float32).reshape(shp)
    dti = inp["dt_idle"].clone().requires_grad_(True)
    dta = inp["dt_active"].clone().requires_grad_(True)
    A = inp["A"].clone().requires_grad_(True)
    Dv = inp["D"].clone().requires_grad_(True)
    delta = (dti[None, :, None] * km1 + dta[None, :, None]) * m
    g = torch.Generator().manual_seed(dense_seed)
    if legacy_bc:
        # per-event B/C [N, E] from dense (B, N, L) draws at each event's (b, t)
        Bd = torch.randn(cfg.B, cfg.N, cfg.L, generator=g)
        Cd = torch.randn(cfg.B, cfg.N, cfg.L, generator=g)
        b_of = ch // cfg.D
        B_ev = Bd[torch.as_tensor(b_of).long(), :, torch.as_tensor(t).long()].T.contiguous()
        C_ev = Cd[torch.as_tensor(b_of).long(), :, torch.as_tensor(t).long()].T.contiguous()
        B_leaf = B_ev.clone().requires_grad_(True)
        C_leaf = C_ev.clone().requires_grad_(True)
        idx_t = torch.as_tensor(idx)
        Bc = B_leaf[:, idx_t].permute(1, 0, 2).reshape(cfg.B, cfg.D, cfg.N, Lmax) * m.unsqueeze(2)
        Cc = C_leaf[:, idx_t].permute(1, 0, 2).reshape(cfg.B, cfg.D, cfg.N, Lmax) * m.unsqueeze(2)
    else:
        W_B = inp["W_B"].clone().requires_grad_(True)
        W_C = inp["W_C"].clone().requires_grad_(True)
        Bc = u_c.unsqueeze(2) * W_B[None, :, :, None]
        Cc = u_c.unsqueeze(2) * W_C[None, :, :, None]
    z_c = None
    if with_z:
        z_flat = torch.randn(E, generator=g)
        z_c = (z_flat[torch.as_tensor(idx)] * torch.as_tensor(mask)).reshape(shp).requires_grad_(True)
    y = ssi.selective_scan_ref(u_c, delta, A, Bc, Cc, D=Dv, z=z_c)
    dout_flat = torch.randn(E, generator=g)
    dout_c = (dout_flat[torch.as_tensor(idx)] * torch.as_tensor(mask)).reshape(shp)
    (y * dout_c).sum().backward()
    flat_mask = mask.reshape(-1)
    sel = idx.reshape(-1)[flat_mask]

    def to_flat(tc):
        out = np.zeros(E, np.float32)
        out[sel] = tc.detach().reshape(-1).numpy()[flat_mask]
        return out

    rec = dict(u_flat=u_flat, k_flat=k.astype(np.int32), cu_seqlens=cu.astype(np.int32),
               max_seqlen=np.int32(mx), dt_idle=inp["dt_idle"].numpy(),
               dt_active=inp["dt_active"].numpy(), A=inp["A"].numpy(), D=inp["D"].numpy(),
               dout_flat=dout_flat.numpy(), out_flat=to_flat(y), du=to_flat(u_c.grad),
               dA=A.grad.numpy(), ddt_idle=dti.grad.numpy(), ddt_active=dta.grad.numpy(),
               dD=Dv.grad.numpy())
    if legacy_bc:
        rec.update(B=B_ev.numpy(), C=C_ev.numpy(), dB=B_leaf.grad.numpy(), dC=C_leaf.grad.numpy())
    else:
        rec.update(W_B=inp["W_B"].numpy(), W_C=inp["W_C"].numpy(), dW_B=W_B.grad.numpy(),
                   dW_C=W_C.grad.numpy())
    if with_z:
        rec.update(z_flat=z_flat.numpy(), dz=to_flat(z_c.grad))
    np.savez_compressed(HERE / f"scan_ref_{name}.npz", **rec)
    print(f"wrote scan_ref_{name}.npz  E={E} NC={cu.size - 1} Lmax={Lmax}")


def main():
    from oracle.build_ref import default_root

    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else default_root()
    ssi = import_reference(ref)
    torch.manual_seed(0)
    c0 = CONFIGS["c0"]
    make_case(ssi, "c0_depthwise", c0)
    make_case(ssi, "c0_legacy_bc", c0, legacy_bc=True)
    make_case(ssi, "c0_depthwise_z", c0, with_z=True)
    make_case(ssi, "small_n4_sparse", c0.with_(B=1, D=8, N=4, L=512, rho=0.05, seed=7))


if __name__ == "__main__":
    main()
