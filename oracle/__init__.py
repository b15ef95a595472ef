"""CPU oracle for the BC_mamba event pipeline — TEST INFRASTRUCTURE ONLY.

Plain numpy (and, for the CPU baseline, torch) restatements of the reference's
algorithms for this path, each function citing the reference file:line it
follows.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import anything from here, and only as the checker or the
timed CPU reference — never as part of the product path, which is the CUDA
code in ``bc_mamba_b200`` and has no CPU fallback.

Parity pinning: the scan oracle is checked against golden vectors produced by
the reference's own ``selective_scan_ref`` (tests/golden/make_scan_ref_fixtures.py)
and, for the integer streams and the restore maps, against hand-derived known
answers plus fixtures produced by the reference's CUDA extensions compiled
from its sources (oracle/build_ref.py, tests/golden/make_ref_cuda_fixtures.py).
"""
