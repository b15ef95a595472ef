"""Compile the reference's three CUDA extensions from its own sources into
``oracle/_ref/`` — a GPU-side checker (TEST INFRASTRUCTURE ONLY).

The reference ships no binaries; its hot path is CUDA C++ built as PyTorch
extensions (csrc/extract, csrc/selective_scan, csrc/r_nodecay).  Instead of
its setup.py / build_extensions.sh, this recipe hands the listed source files
directly to torch's extension compiler for sm_100 and writes the modules to
oracle/_ref/<name>/ (git-ignored; travels to the GPU box with the tree).
Nothing is copied out of the reference tree.

    python oracle/build_ref.py [/path/to/reference]

Only tests and fixture generation load these modules, to compare our kernels
with the reference's on identical inputs.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def default_root() -> Path:
    """The reference checkout: $BCM_REFERENCE_ROOT, else the mount point of
    the build container."""
    return Path(os.environ.get("BCM_REFERENCE_ROOT", "/root/reference"))

SOURCES = {
    "extract_events_cuda": ["csrc/extract/extract_events_cuda.cu"],
    "restore_dense_cuda_nodecay": [
        "csrc/r_nodecay/restore_dense.cpp",
        "csrc/r_nodecay/restore_dense_fwd_fp16.cu",
        "csrc/r_nodecay/restore_dense_fwd_bf16.cu",
        "csrc/r_nodecay/restore_dense_fwd_fp32.cu",
        "csrc/r_nodecay/restore_dense_bwd_fp16.cu",
        "csrc/r_nodecay/restore_dense_bwd_bf16.cu",
        "csrc/r_nodecay/restore_dense_bwd_fp32.cu",
    ],
    "selective_scan_cuda": [
        "csrc/selective_scan/selective_scan.cpp",
        "csrc/selective_scan/selective_scan_fwd_fp16.cu",
        "csrc/selective_scan/selective_scan_fwd_bf16.cu",
        "csrc/selective_scan/selective_scan_fwd_fp32.cu",
        "csrc/selective_scan/selective_scan_bwd_fp16_real.cu",
        "csrc/selective_scan/selective_scan_bwd_bf16_real.cu",
        "csrc/selective_scan/selective_scan_bwd_fp32_real.cu",
        "csrc/selective_scan/selective_scan_bwd_fp16_complex.cu",
        "csrc/selective_scan/selective_scan_bwd_bf16_complex.cu",
        "csrc/selective_scan/selective_scan_bwd_fp32_complex.cu",
    ],
}

# The reference's own flags for each module (setup.py files), arch pinned to sm_100.
FLAGS = {
    "extract_events_cuda": ["-O3", "-std=c++17", "--use_fast_math"],
    "restore_dense_cuda_nodecay": ["-O3"],
    "selective_scan_cuda": ["-O3"],
}


def build(ref_root: Path, names=None) -> None:
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils import cpp_extension

    for name, srcs in SOURCES.items():
        if names and name not in names:
            continue
        bdir = OUT / name
        bdir.mkdir(parents=True, exist_ok=True)
        paths = [str(ref_root / s) for s in srcs]
        print(f"building {name} from {len(paths)} reference sources", flush=True)
        cpp_extension.load(name=name, sources=paths, build_directory=str(bdir),
                           extra_cflags=["-O3"], extra_cuda_cflags=FLAGS[name],
                           with_cuda=True, verbose=False)


def load(name: str):
    """Import a built reference module (None when it was not built)."""
    import importlib.machinery
    import importlib.util

    so = OUT / name / f"{name}.so"
    if not so.exists():
        return None
    import torch  # noqa: F401

    loader = importlib.machinery.ExtensionFileLoader(name, str(so))
    spec = importlib.util.spec_from_file_location(name, str(so), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else default_root()
    build(root, sys.argv[2:] or None)
