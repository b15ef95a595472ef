"""Drop-in for the reference's ``restore_dense_cuda_nodecay`` extension module
(csrc/r_nodecay/restore_dense.cpp:206-226), backed by libbcm_b200.so."""
from bc_mamba_b200._native import load_ops as _load

_ops = _load()
restore_dense_fwd = _ops.restore_dense_fwd
restore_dense_bwd = _ops.restore_dense_bwd
__file__native__ = _ops.__file__
