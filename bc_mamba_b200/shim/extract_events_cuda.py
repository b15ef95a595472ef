"""Drop-in for the reference's ``extract_events_cuda`` extension module
(csrc/extract/extract_events_cuda.cu:759-798), backed by libbcm_b200.so."""
from bc_mamba_b200._native import load_ops as _load

_ops = _load()
extract_events = _ops.extract_events
extract_base_events = _ops.extract_base_events
expand_base_events = _ops.expand_base_events
gather_events_fwd = _ops.gather_events_fwd
gather_events_bwd = _ops.gather_events_bwd
__file__native__ = _ops.__file__
