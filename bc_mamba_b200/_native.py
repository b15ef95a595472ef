"""Locate and load the native parts built in-tree by ``bc_mamba_b200.build``.

``libbcm_b200.so`` holds the CUDA kernels behind the C ABI of
``include/bcm_b200.h``; ``_bcm_torch*.so`` is the pybind11 host shim linked to
it.  Nothing here falls back to Python or CPU code: if the native build is
missing, importing the ops raises.
"""
from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libbcm_b200.so"

# Every symbol include/bcm_b200.h declares (checked by the CPU test suite).
ABI_SYMBOLS = (
    "bcm_last_error",
    "bcm_abi_version",
    "bcm_extract_workspace_bytes",
    "bcm_extract_base_count",
    "bcm_extract_base_fill",
    "bcm_extract_base_count_bld",
    "bcm_expand_base_events",
    "bcm_gather_events_fwd",
    "bcm_gather_bwd_workspace_bytes",
    "bcm_gather_events_bwd",
    "bcm_gather_events_bwd_noalloc",
    "bcm_conv_events_fwd",
    "bcm_conv_events_bwd_workspace_bytes",
    "bcm_conv_events_bwd",
    "bcm_flat_ch_ckpt_bytes",
    "bcm_flat_ch_fwd_workspace_bytes",
    "bcm_flat_ch_bwd_workspace_bytes",
    "bcm_flat_ch_fwd",
    "bcm_flat_ch_bwd",
    "bcm_event_decode_step",
    "bcm_extract_expand_fill",
    "bcm_extract_expanded",
    "bcm_extract_expanded_ft",
    "bcm_gather_events_bwd_rows",
    "bcm_restore_workspace_bytes",
    "bcm_restore_bitmap_bytes",
    "bcm_restore_dense_fwd_bitmap",
    "bcm_restore_dense_fwd_mask",
    "bcm_restore_dense_bwd_bitmap",
    "bcm_restore_dense_fwd",
    "bcm_restore_dense_bwd",
    "bcm_s6_fwd",
    "bcm_s6_bwd_workspace_bytes",
    "bcm_s6_bwd",
    "bcm_event_params_fwd",
    "bcm_event_params_bwd",
)

_ops = None
_lib = None


class NativeBuildMissing(ImportError):
    pass


def load_library() -> ctypes.CDLL:
    """dlopen libbcm_b200.so (works without a GPU)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeBuildMissing(
                f"{LIB_PATH} is missing; run `python -m bc_mamba_b200.build` first")
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.bcm_last_error.restype = ctypes.c_char_p
        _lib.bcm_abi_version.restype = ctypes.c_int
    return _lib


def load_ops():
    """Import the pybind11 shim (requires torch; kernels need a CUDA device)."""
    global _ops
    if _ops is None:
        import torch  # noqa: F401  (loads libc10/libtorch the shim links against)

        load_library()
        cands = sorted(PKG.glob("_bcm_torch*.so"))
        if not cands:
            raise NativeBuildMissing(
                f"no _bcm_torch*.so in {PKG}; run `python -m bc_mamba_b200.build` first")
        name = "bc_mamba_b200._bcm_torch"
        loader = importlib.machinery.ExtensionFileLoader("_bcm_torch", str(cands[0]))
        spec = importlib.util.spec_from_file_location("_bcm_torch", str(cands[0]), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules[name] = mod
        _ops = mod
    return _ops
