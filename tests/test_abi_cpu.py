"""CPU tests of the drop-in boundary: the C-ABI library loads without a GPU
and exports every symbol include/bcm_b200.h declares; the pybind11 shim
exposes every entry point of the reference's three extension modules; the
drop-in modules resolve by the reference's names.  No kernel is launched."""
import re
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "bcm_b200.h").read_text()
    return sorted(set(re.findall(r"BCM_API\s+[\w\s\*]+?\b(bcm_\w+)\s*\(", text)))


def test_header_matches_package_list():
    import bc_mamba_b200

    assert declared_symbols() == sorted(bc_mamba_b200.ABI_SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    import ctypes

    import bc_mamba_b200

    lib = bc_mamba_b200.load_library()
    for s in declared_symbols():
        assert isinstance(getattr(lib, s), ctypes._CFuncPtr), s
    # the allocation-free gather backward is declared and exported like the rest
    assert "bcm_gather_events_bwd_noalloc" in declared_symbols()
    assert isinstance(lib.bcm_gather_events_bwd_noalloc, ctypes._CFuncPtr)
    assert lib.bcm_abi_version() == 1
    assert lib.bcm_last_error() == b""


def test_workspace_queries_without_gpu():
    import ctypes

    import bc_mamba_b200

    lib = bc_mamba_b200.load_library()
    lib.bcm_extract_workspace_bytes.restype = ctypes.c_size_t
    lib.bcm_extract_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    # one bit per base channel and position, plus a 256-byte {total, max} slot
    assert lib.bcm_extract_workspace_bytes(4096, 2048) == 4096 * 64 * 4 + 256
    lib.bcm_restore_workspace_bytes.restype = ctypes.c_size_t
    lib.bcm_restore_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    assert lib.bcm_restore_workspace_bytes(8192, 2048) == 8192 * 64 * 4
    assert lib.bcm_restore_workspace_bytes(3, 33) == 256


def test_shim_exports_reference_entry_points():
    import bc_mamba_b200

    ops = bc_mamba_b200.load_ops()
    for name in ["fwd", "bwd", "fwd_flat_ch", "bwd_flat_ch", "extract_events", "extract_base_events",
                 "expand_base_events", "gather_events_fwd", "gather_events_bwd", "restore_dense_fwd",
                 "restore_dense_bwd"]:
        assert callable(getattr(ops, name)), name
    # the product's own fused entry points beside them
    for name in ["extract_expanded_events", "extract_base_events_host_max", "restore_dense_fwd_bitmap",
                 "restore_dense_bwd_bitmap", "conv_events_fwd", "conv_events_bwd"]:
        assert callable(getattr(ops, name)), name
    doc = ops.fwd_flat_ch.__doc__
    for arg in ["u_flat", "k_flat", "cu_seqlens", "max_seqlen", "dt_idle", "dt_active", "tile_offsets",
                "tile_chunk_size", "is_depthwise_bc", "pw_B", "pw_C"]:
        assert arg in doc, arg


def test_dropin_module_names():
    from bc_mamba_b200 import interface

    interface.install_shim()
    import extract_events_cuda
    import restore_dense_cuda_nodecay
    import selective_scan_cuda

    assert hasattr(extract_events_cuda, "gather_events_fwd")  # e_model's _HAS_GATHER_CUDA probe
    assert hasattr(restore_dense_cuda_nodecay, "restore_dense_fwd")
    assert hasattr(selective_scan_cuda, "fwd_flat_ch")


def test_dense_scan_entry_points_and_cpu_errors():
    """selective_scan_cuda.fwd/bwd take the reference's arguments and check
    them before any kernel runs (CPU tensors are rejected)."""
    import torch

    import bc_mamba_b200

    ops = bc_mamba_b200.load_ops()
    u = torch.zeros(1, 2, 4)
    A = -torch.ones(2, 4)
    with pytest.raises(RuntimeError):
        ops.fwd(u, u, A, A, A, None, None, None, False)
    with pytest.raises(RuntimeError, match="complex weights"):
        ops.fwd(u, u, A.to(torch.complex64), A.to(torch.complex64), A.to(torch.complex64), None, None, None, False)
    with pytest.raises(RuntimeError):
        ops.bwd(u, u, A, A, A, None, None, None, u, None, None, None, False, False)


def test_event_params_entry_points_and_cpu_errors():
    """The fused block-parameter transforms are exported and reject CPU
    tensors before any kernel runs."""
    import torch

    import bc_mamba_b200

    ops = bc_mamba_b200.load_ops()
    A_log, W_BC, a = torch.zeros(4, 8), torch.zeros(4, 16), torch.zeros(4)
    with pytest.raises(RuntimeError, match="A_log must be a contiguous float32 CUDA tensor"):
        ops.event_params_fwd(A_log, W_BC, a, a, 1e-6)
    with pytest.raises(RuntimeError, match="A must be a contiguous float32 CUDA tensor"):
        ops.event_params_bwd(A_log, a, a, None, None, None, None, None)


def test_argument_errors_without_gpu():
    """The entry points added beside the reference's reject bad arguments
    before any CUDA call: BCM_ERR_INVALID_ARGUMENT (1) and the reason in
    bcm_last_error()."""
    import ctypes

    import bc_mamba_b200

    lib = bc_mamba_b200.load_library()
    lib.bcm_last_error.restype = ctypes.c_char_p
    P, I, E = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

    f = lib.bcm_event_params_fwd
    f.restype = E
    f.argtypes = [P, P, P, P, I, I, ctypes.c_float] + [P] * 6
    assert f(None, None, None, None, 0, 16, 1e-6, *([None] * 6)) == 1
    assert b"event_params_fwd: bad sizes" in lib.bcm_last_error()

    f = lib.bcm_event_params_bwd
    f.restype = E
    f.argtypes = [P] * 8 + [I, I] + [P] * 5
    assert f(*([None] * 8), 4, 16, *([None] * 5)) == 1
    assert b"event_params_bwd: null pointer" in lib.bcm_last_error()

    f = lib.bcm_restore_dense_fwd_mask
    f.restype = E
    f.argtypes = [P, E, P, P, I, I, I, I, P, E, P, I, P, P]
    assert f(None, 0, None, None, 10, 8, 8, 100, None, 0, None, 2, None, None) == 1
    assert b"null event_bitmap or base_mask" in lib.bcm_last_error()

    f = lib.bcm_extract_expanded_ft
    f.restype = E
    f.argtypes = [P, E, I, I, I, P, I, P, P, P, P, ctypes.c_size_t, I, P, P, P, P, P, E, P, P, P, P]
    assert f(None, 0, 1, 4, 8, None, 2, None, None, None, None, 0, 0, None, None, None, None, None, 0,
             None, None, None, None) == 1
    assert b"null feature thresholds" in lib.bcm_last_error()
