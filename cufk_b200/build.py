"""Builds the two native artefacts of cufk_b200 in-tree, for sm_100a only.

* ``cufk_b200/libcufkb.so``: every CUDA kernel plus the C ABI declared in ``include/cufkb.h``
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, static CUDA runtime, no torch).
* ``cufk_b200/_C.so``: the PyTorch extension (host C++ only) holding the autograd ``apply``
  wrappers; it links ``libcufkb.so`` through an ``$ORIGIN`` run path.

Both are rebuilt only when a source is newer than the artefact (or with ``force``).  Nothing is
written outside the package directory and its ``_build/`` folder.

Usage: ``python cufk_b200/build.py [--force]`` (run as a script, so that the package and its old
native libraries are not imported before they are rebuilt).
"""

from __future__ import annotations

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
LIB = PKG / "libcufkb.so"
EXT = PKG / "_C.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", *ARCH]
CUDA_SOURCES = [CSRC / "cufkb_api.cu"]
CUDA_DEPENDS = [CSRC / "nerf_device.cuh", CSRC / "nerf_kernels.cuh", CSRC / "nerf_long.cuh", CSRC / "nerf_math.cuh", CSRC / "nerf_vec.cuh", INCLUDE / "cufkb.h"]
EXT_SOURCES = [CSRC / "torch_ext.cpp"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else "nvcc"


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the kernels and the C ABI into libcufkb.so."""
    if not force and not _stale(LIB, CUDA_SOURCES + CUDA_DEPENDS):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *map(str, CUDA_SOURCES), "-o", str(tmp), "-Xlinker", "-soname=libcufkb.so"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the PyTorch autograd wrapper (host code) into _C.so, linked to libcufkb.so."""
    if not force and not _stale(EXT, EXT_SOURCES + [INCLUDE / "cufkb.h", LIB]):
        return EXT
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    BUILD.mkdir(parents=True, exist_ok=True)
    # load() imports the result; make libcufkb.so resolvable by soname from the build folder
    import ctypes

    ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)
    load(
        name="_C",
        sources=[str(s) for s in EXT_SOURCES],
        extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O2", "-std=c++17"],
        # "$ORIGIN" escaped for ninja ($$) and for the shell ninja runs the link in (\\$)
        extra_ldflags=[f"-L{PKG}", "-lcufkb", "-Wl,-rpath,\\$$ORIGIN"],
        build_directory=str(BUILD),
        with_cuda=True,
        verbose=verbose,
        is_python_module=False,
        is_standalone=False,
    )
    built = BUILD / "_C.so"
    tmp = EXT.with_suffix(".so.tmp")
    shutil.copy(built, tmp)  # fresh mtime: the artefact is newer than libcufkb.so it was linked against
    os.replace(tmp, EXT)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_extension(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
