"""Recipe that compiles the reference's own CUDA kernels for sm_100a into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY.  The product (``cufk_b200``) never imports, links or runs anything
under ``oracle/``; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may.  The built extensions are the parity pin for the float64 restatement in
``oracle/nerf64.py``: the reference ships no tests or golden vectors, so its own kernels, run on
a B200, are the only ground truth for "the reference's result on these inputs".

What is compiled (from the files where they lie in the read-only reference checkout; nothing is
copied into this repository):

* ``src/cufk/csrc/block.cu`` -> ``oracle/_ref/block/cufk_ref_block.so``.  The reference builds it
  with ``-O3 -std=c++20`` (``setup.py:14-24``); the same flags are used here plus an explicit
  ``-gencode arch=compute_100a,code=sm_100a``, which is what ``TORCH_CUDA_ARCH_LIST=10.0a`` gives.
* ``src/cufk/csrc/torsion.cu`` -> ``oracle/_ref/torsion/cufk_ref_torsion.so`` for ONE constant
  set (the backbone constants of the benchmark configuration).  The flags restate
  ``src/cufk/torsion.py:59-86``: ``-O3 -std=c++20 --use_fast_math`` and the six ``-D`` macros, whose values
  are formatted with ``.17g`` and whose angle sin/cos come from Python's ``math`` in double.

This does not run the reference's build system (its ``setup.py``); it calls nvcc through
``torch.utils.cpp_extension.load`` with the flags above.  Re-running is a no-op when the outputs
exist and ``--force`` is not given.

Usage: ``python oracle/build_ref.py [--force] [--reference PATH]``.
"""

from __future__ import annotations

import argparse
import math
import os
import shutil
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"

# Backbone constants of the torsion benchmark configuration (N-CA, CA-C, C-N lengths in nm and
# N-CA-C, CA-C-N, C-N-CA angles in rad).  Mirrors the example in the reference README.
TORSION_BOND_LENGTHS = (0.14685231, 0.15365194, 0.13405086)
TORSION_BOND_ANGLES = (1.9676635, 2.062335, 2.164016)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _fmt(value: float) -> str:
    return format(float(value), ".17g")


def torsion_flags(lengths, angles) -> list[str]:
    """Restates ``_compile_flags`` (``src/cufk/torsion.py:81-86``)."""
    flags = ["-O3", "-std=c++20", "--use_fast_math"]
    for i, length in enumerate(lengths):
        flags.append(f"-DCUFK_TORSION_BOND_{i}_LENGTH={_fmt(length)}")
    for i, angle in enumerate(angles):
        flags.append(f"-DCUFK_TORSION_ANGLE_{i}_SIN={_fmt(math.sin(angle))}")
        flags.append(f"-DCUFK_TORSION_ANGLE_{i}_COS={_fmt(math.cos(angle))}")
    return flags


def _build(name: str, source: Path, cuda_flags: list[str], out_dir: Path, force: bool) -> Path:
    from torch.utils.cpp_extension import load

    target = out_dir / f"{name}.so"
    if target.exists() and not force:
        print(f"[build_ref] {target} exists; skipping")
        return target
    build_dir = out_dir / "build"
    if force and build_dir.exists():
        shutil.rmtree(build_dir)
    build_dir.mkdir(parents=True, exist_ok=True)
    t0 = time.time()
    load(
        name=name,
        sources=[str(source)],
        extra_cuda_cflags=cuda_flags + ARCH_FLAGS,
        extra_cflags=["-O3"],
        build_directory=str(build_dir),
        with_cuda=True,
        verbose=False,
        is_python_module=True,
    )
    built = build_dir / f"{name}.so"
    shutil.copy2(built, target)
    print(f"[build_ref] built {target} in {time.time() - t0:.0f}s")
    return target


def build(reference: Path, force: bool = False, which: str = "all") -> None:
    csrc = reference / "src" / "cufk" / "csrc"
    if not csrc.is_dir():
        raise FileNotFoundError(f"reference sources not found under {csrc}")
    # torch's JIT picks the arch list from this variable; pin it so no host-visible GPU is probed.
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    if which in ("all", "block"):
        _build("cufk_ref_block", csrc / "block.cu", ["-O3", "-std=c++20"], REF_OUT / "block", force)
    if which in ("all", "torsion"):
        _build(
            "cufk_ref_torsion",
            csrc / "torsion.cu",
            torsion_flags(TORSION_BOND_LENGTHS, TORSION_BOND_ANGLES),
            REF_OUT / "torsion",
            force,
        )


def reference_checkout() -> Path | None:
    """The cufk checkout to compile: $CUFKB_REFERENCE when set, else a directory named "reference"
    beside this repository; None when neither exists."""
    env = os.environ.get("CUFKB_REFERENCE")
    candidate = Path(env) if env else Path(__file__).resolve().parent.parent.parent / "reference"
    return candidate if candidate.is_dir() else None


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=None, help="cufk checkout (default: $CUFKB_REFERENCE, else ../reference)")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--which", choices=["all", "block", "torsion"], default="all")
    args = ap.parse_args(argv)
    ref = Path(args.reference) if args.reference else reference_checkout()
    if ref is None:
        print("no reference checkout: set CUFKB_REFERENCE")
        return 1
    build(ref, force=args.force, which=args.which)
    return 0


if __name__ == "__main__":
    sys.exit(main())
