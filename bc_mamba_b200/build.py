"""In-tree build of the native parts of bc_mamba_b200.

Two artefacts, both written next to this file so they travel with the tree:

* ``libbcm_b200.so``  — every CUDA kernel plus the ``extern "C"`` ABI declared
  in ``include/bcm_b200.h``; compiled by nvcc for sm_100a only, cudart linked
  statically, no torch dependency.
* ``_bcm_torch*.so``  — the pybind11 host shim (``csrc/torch_shim.cpp``) that
  mirrors the reference's three extension modules on top of the C ABI.

Run ``python -m bc_mamba_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libbcm_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["abi.cu", "extract.cu", "restore.cu", "scan_fwd.cu", "scan_bwd.cu", "scan_dw.cu", "scan_v3.cu", "scan_seg.cu",
              "conv_events.cu", "decode.cu", "s6_dense.cu", "param_prep.cu"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC),
]


def _hash(paths) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(Path(p).read_bytes())
    h.update(" ".join(NVCC_FLAGS + ARCH).encode())
    return h.hexdigest()[:16]


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    deps = [CSRC / s for s in CU_SOURCES] + list(CSRC.glob("*.cuh")) + [INCLUDE / "bcm_b200.h"]
    stamp = BUILD / "libbcm_b200.stamp"
    key = _hash(deps)
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == key:
        return LIB
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(CSRC / s, verbose), CU_SOURCES))
    tmp = BUILD / "libbcm_b200.so.tmp"
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "-soname=libbcm_b200.so",
           "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(key)
    return LIB


def build_torch_shim(force: bool = False, verbose: bool = False) -> Path:
    """Compile the pybind11 shim against torch and link it to libbcm_b200.so."""
    from torch.utils import cpp_extension

    src = CSRC / "torch_shim.cpp"
    key = _hash([src, INCLUDE / "bcm_b200.h"])
    stamp = BUILD / "torch_shim.stamp"
    existing = sorted(PKG.glob("_bcm_torch*.so"))
    if not force and existing and stamp.exists() and stamp.read_text() == key:
        return existing[0]
    shim_build = BUILD / "torch_shim"
    if shim_build.exists():
        shutil.rmtree(shim_build)
    shim_build.mkdir(parents=True)
    # torch imports the module from the build directory right after linking;
    # the soname of an already-loaded libbcm_b200.so satisfies its dependency.
    import ctypes

    ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)
    cpp_extension.load(
        name="_bcm_torch",
        sources=[str(src)],
        extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O3", "-std=c++17"],
        # `\$$` survives ninja and the shell as a literal $ORIGIN
        extra_ldflags=[f"-L{PKG}", "-lbcm_b200", "-Wl,-rpath,\\$$ORIGIN"],
        build_directory=str(shim_build),
        with_cuda=True,
        verbose=verbose,
    )
    built = sorted(shim_build.glob("_bcm_torch*.so"))
    if not built:
        raise RuntimeError("torch shim build produced no .so")
    for old in existing:
        old.unlink()
    dst = PKG / built[0].name
    shutil.copy2(built[0], dst)
    stamp.write_text(key)
    return dst


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_torch_shim(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", LIB)
