"""Drop-in for the reference's ``selective_scan_cuda`` extension module
(csrc/selective_scan/selective_scan.cpp:1155-1197), backed by libbcm_b200.so."""
from bc_mamba_b200._native import load_ops as _load

_ops = _load()
fwd = _ops.fwd
bwd = _ops.bwd
fwd_flat_ch = _ops.fwd_flat_ch
bwd_flat_ch = _ops.bwd_flat_ch
__file__native__ = _ops.__file__
