"""GPU test of bcm_gather_events_bwd_noalloc, the gather backward for callers
that may not allocate device memory (an FFI host whose device memory all
comes from its own arena, or code where cudaMalloc/cudaFree would stall the
GPU).  It keeps its scratch in a fixed array inside the library instead of a
caller-supplied workspace.

Both entry points are called through the C ABI with ctypes, on two calls in a
row with different shapes, dtypes and event orders, so the second call runs
on scratch the first one left behind.  The gather backward is a copy, so the
outputs must agree bit for bit.  The file name makes pytest collect it last;
it passes alone in a fresh process as well."""
import ctypes

import numpy as np
import pytest
import torch

from bc_mamba_b200 import load_library
from bc_mamba_b200.workloads import CONFIGS, make_inputs
from oracle import events as ev

pytestmark = pytest.mark.gpu
dev = "cuda"
MAX_CHANNELS = 262144   # BCM_GATHER_BWD_NOALLOC_MAX_CHANNELS
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


def _lib():
    lib = load_library()
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.bcm_gather_events_bwd.restype = I
    lib.bcm_gather_events_bwd.argtypes = [P, I, P, P, I64, I64, I64, P, P, ctypes.c_size_t, P]
    lib.bcm_gather_events_bwd_noalloc.restype = I
    lib.bcm_gather_events_bwd_noalloc.argtypes = [P, I, P, P, I64, I64, I64, P, P]
    lib.bcm_gather_bwd_workspace_bytes.restype = ctypes.c_size_t
    lib.bcm_gather_bwd_workspace_bytes.argtypes = [I64]
    return lib


def _case(cfg, dtype, shuffle, seed):
    """Event stream of cfg (oracle extraction) and a random grad per event."""
    inp = make_inputs(cfg)
    r = ev.extract_base_events(inp["v"].numpy(), inp["threshold"])
    ch, t, _k, _cu, _mx = ev.expand_base_events(*r[:4], cfg.B, cfg.d_model, cfg.expand)
    if shuffle:
        perm = np.random.default_rng(seed).permutation(ch.size)
        ch, t = ch[perm], t[perm]
    g = torch.randn(ch.size, generator=torch.Generator().manual_seed(seed)).to(dtype)
    return (g.to(dev), torch.as_tensor(ch).to(dev), torch.as_tensor(t).to(dev),
            cfg.B * cfg.D, cfg.L)


def _garbage(n_ch, L, dtype):
    return torch.full((n_ch, L), float("nan"), dtype=dtype, device=dev)


def _run_existing(lib, g, ch, t, n_ch, L):
    dx = _garbage(n_ch, L, g.dtype)
    ws = torch.empty(lib.bcm_gather_bwd_workspace_bytes(n_ch), dtype=torch.uint8, device=dev)
    st = lib.bcm_gather_events_bwd(g.data_ptr(), DTYPES[g.dtype], ch.data_ptr(), t.data_ptr(), ch.numel(),
                                   n_ch, L, dx.data_ptr(), ws.data_ptr(), ws.numel(),
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.bcm_last_error()
    return dx


def _run_noalloc(lib, g, ch, t, n_ch, L):
    dx = _garbage(n_ch, L, g.dtype)
    st = lib.bcm_gather_events_bwd_noalloc(g.data_ptr(), DTYPES[g.dtype], ch.data_ptr(), t.data_ptr(),
                                           ch.numel(), n_ch, L, dx.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.bcm_last_error()
    return dx


def test_noalloc_matches_existing_entry_two_calls_in_a_row():
    lib = _lib()
    cases = [
        # first call: shuffled stream -> the order flag is raised in the scratch
        _case(CONFIGS["c0"].with_(B=4, D=256, L=1000), torch.float32, shuffle=True, seed=11),
        # second call: extraction order, other shape and dtype, on the leftover scratch
        _case(CONFIGS["c3"].with_(B=3, D=128, N=16, L=250), torch.bfloat16, shuffle=False, seed=12),
    ]
    outs = []
    for g, ch, t, n_ch, L in cases:
        outs.append(_run_noalloc(lib, g, ch, t, n_ch, L))
    torch.cuda.synchronize()
    for (g, ch, t, n_ch, L), got in zip(cases, outs):
        want = _run_existing(lib, g, ch, t, n_ch, L)
        torch.cuda.synchronize()
        assert not torch.isnan(got).any()
        assert torch.equal(got, want)


def test_noalloc_call_allocates_no_device_memory():
    """After a first call on the device (which may load the library's module
    and with it the fixed array), a call changes neither the caching
    allocator's counters nor the device's free memory: it allocates nothing."""
    lib = _lib()
    g, ch, t, n_ch, L = _case(CONFIGS["c0"].with_(B=4, D=128, L=777), torch.float32, shuffle=False, seed=13)
    dx = _garbage(n_ch, L, g.dtype)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        st = lib.bcm_gather_events_bwd_noalloc(g.data_ptr(), DTYPES[g.dtype], ch.data_ptr(), t.data_ptr(),
                                               ch.numel(), n_ch, L, dx.data_ptr(), stream)
        assert st == 0, lib.bcm_last_error()

    call()                      # warm: module loaded, symbol address cached
    torch.cuda.synchronize()
    alloc0, reserved0 = torch.cuda.memory_allocated(), torch.cuda.memory_reserved()
    free0, _total = torch.cuda.mem_get_info()
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    free1, _total = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert torch.cuda.memory_reserved() == reserved0
    # a device allocation shows as at least one 2 MiB page of free memory gone
    assert free1 >= free0 - (1 << 20), (free0, free1)
    assert not torch.isnan(dx).any()


def test_noalloc_rejects_more_channels_than_its_scratch_holds():
    lib = _lib()
    torch.zeros(1, device=dev)
    st = lib.bcm_gather_events_bwd_noalloc(None, 0, None, None, 1, MAX_CHANNELS + 1, 8, None, None)
    assert st == 1   # BCM_ERR_INVALID_ARGUMENT
    assert b"exceeds the fixed scratch limit" in lib.bcm_last_error()
