"""Generate golden vectors for the dense selective scan (S6) from the
reference's own ``selective_scan_ref`` (spike_mamba/selective_scan_interface.py:
708-774): forward (with return_last_state) and its autograd backward, in the
reference's float32, on seeded inputs.

Run in the build container, where the reference is mounted read-only:
    python tests/golden/make_s6_ref_fixtures.py [/path/to/reference]
(stubs for the absent third-party imports as make_scan_ref_fixtures.py).
Output: tests/golden/s6_ref_*.npz.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from make_scan_ref_fixtures import import_reference  # noqa: E402

CASES = {
    # name: (batch, dim, seqlen, dstate, B kind, C kind, groups, D, z, delta_bias, softplus)
    "fixed": (2, 8, 300, 16, "fixed", "fixed", 1, True, False, False, False),
    "var_groups": (2, 8, 300, 16, "var", "var", 2, True, True, True, True),
    "mixed_n4": (1, 6, 200, 4, "fixed", "var", 1, False, False, True, True),
    "var_b_fixed_c": (2, 4, 150, 8, "var", "fixed", 4, True, True, False, True),
}


def make_case(ssi, name, spec, seed):
    bsz, dim, L, N, bk, ck, groups, has_d, has_z, has_bias, softplus = spec
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(bsz, dim, L, generator=g)
    if softplus:
        delta = 0.5 * torch.randn(bsz, dim, L, generator=g) - 1.0
    else:
        delta = 0.01 + 0.2 * torch.rand(bsz, dim, L, generator=g)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(dim, 1) * (0.5 + torch.rand(dim, 1, generator=g))
    B = torch.randn(dim, N, generator=g) if bk == "fixed" else torch.randn(bsz, groups, N, L, generator=g)
    C = torch.randn(dim, N, generator=g) if ck == "fixed" else torch.randn(bsz, groups, N, L, generator=g)
    D = torch.randn(dim, generator=g) if has_d else None
    z = torch.randn(bsz, dim, L, generator=g) if has_z else None
    bias = 0.3 * torch.randn(dim, generator=g) if has_bias else None
    dout = torch.randn(bsz, dim, L, generator=g)
    leaves = {k: v.clone().requires_grad_(True) for k, v in
              dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=bias).items() if v is not None}
    out, last = ssi.selective_scan_ref(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                       D=leaves.get("D"), z=leaves.get("z"), delta_bias=leaves.get("delta_bias"),
                                       delta_softplus=softplus, return_last_state=True)
    (out * dout).sum().backward()
    rec = {k: v.detach().numpy() for k, v in dict(u=u, delta=delta, A=A, B=B, C=C, dout=dout).items()}
    for k, v in dict(D=D, z=z, delta_bias=bias).items():
        if v is not None:
            rec[k] = v.numpy()
    rec.update(out=out.detach().numpy(), last_state=last.detach().numpy(), softplus=np.int32(softplus))
    for k, v in leaves.items():
        rec["d" + k] = v.grad.numpy()
    np.savez_compressed(HERE / f"s6_ref_{name}.npz", **rec)
    print(f"wrote s6_ref_{name}.npz  {spec}")


def main():
    from oracle.build_ref import default_root

    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else default_root()
    ssi = import_reference(ref)
    for i, (name, spec) in enumerate(CASES.items()):
        make_case(ssi, name, spec, seed=100 + i)


if __name__ == "__main__":
    main()
