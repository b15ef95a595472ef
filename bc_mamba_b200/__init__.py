"""bc_mamba_b200 — B200-native (sm_100a) event-scan pipeline of BC_mamba.

Hot path: threshold -> event extraction -> sparse selective scan fwd/bwd with
inter-spike decay -> causal zero-order-hold restore, as hand-written CUDA in
``libbcm_b200.so`` behind the C ABI ``include/bcm_b200.h``, exposed through the
reference's own module names and autograd Functions (``interface``).
"""
from ._native import ABI_SYMBOLS, LIB_PATH, load_library, load_ops  # noqa: F401

__all__ = ["ABI_SYMBOLS", "LIB_PATH", "load_library", "load_ops"]
