"""Generates the golden vectors in this folder from the reference's own kernels.

TEST INFRASTRUCTURE ONLY.  The reference (xsjk/cufk) ships no golden vectors or known-answer tests,
so these fixtures are outputs of its CUDA kernels, compiled from its sources by
``oracle/build_ref.py`` into ``oracle/_ref/`` and run on a B200:

* ``block_*``: ``ReconstructAutograd`` forward and backward (src/cufk/csrc/block.cu:393-445) through
  the Python layer of src/cufk/reconstruct.py:29-81 (``oracle.ref_kernels.ref_reconstruct``);
* ``torsion_*``: the torsion extension compiled for the benchmark constants
  (src/cufk/csrc/torsion.cu:419-447, src/cufk/torsion.py:89-135).

Inputs come from ``oracle.nerf64.make_inputs`` / ``make_torsion_inputs`` (seeded, CPU float64, then
cast).  ``tests/test_oracle.py`` checks the float64 oracle against every file on the CPU.  Run on a
GPU machine after ``python oracle/build_ref.py``::

    python tests/golden/make_golden.py [--out DIR]
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import nerf64, ref_kernels  # noqa: E402

BOND_LENGTHS = (0.14685231, 0.15365194, 0.13405086)
BOND_ANGLES = (1.9676635, 2.062335, 2.164016)
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")

# (name, batch, points, dtype, anchors, single-chain)
BLOCK_CASES = [
    ("block_f32_b4_n4", 4, 4, torch.float32, False, False),
    ("block_f32_b3_n5_anchors", 3, 5, torch.float32, True, False),
    ("block_f32_b4_n33", 4, 33, torch.float32, False, False),
    ("block_f32_b4_n384", 4, 384, torch.float32, False, False),
    ("block_f32_b2_n2051_anchors", 2, 2051, torch.float32, True, False),
    ("block_f32_single_n100_anchors", 1, 100, torch.float32, True, True),
    ("block_f64_b3_n7_anchors", 3, 7, torch.float64, True, False),
    ("block_f64_b2_n257", 2, 257, torch.float64, False, False),
]
# (name, batch, points, dtype)
TORSION_CASES = [
    ("torsion_f32_b4_n4", 4, 4, torch.float32),
    ("torsion_f32_b3_n34", 3, 34, torch.float32),
    ("torsion_f32_b2_n768", 2, 768, torch.float32),
    ("torsion_f64_b2_n100", 2, 100, torch.float64),
]


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def block_case(name, batch, points, dtype, anchors, single):
    inp = nerf64.make_inputs(batch, points, seed=sum(map(ord, name)), dtype=dtype, anchors=anchors)
    if single:
        for k in ("lengths", "angles", "dihedrals", "grad"):
            inp[k] = inp[k][0]
    L, A, D = (inp[k].cuda().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: inp[k].cuda() for k in ANCHOR_KEYS} if anchors else {}
    xyz = ref_kernels.ref_reconstruct(L, A, D, **kw)
    xyz.backward(inp["grad"].cuda())
    out = {"kind": "block", "dtype": str(dtype).split(".")[1], **{k: _np(v) for k, v in inp.items()}}
    out.update(xyz=_np(xyz), grad_lengths=_np(L.grad), grad_angles=_np(A.grad), grad_dihedrals=_np(D.grad))
    return out


def torsion_case(name, batch, points, dtype):
    inp = nerf64.make_torsion_inputs(batch, points, seed=sum(map(ord, name)), dtype=dtype)
    raw = inp["raw"].cuda().requires_grad_(True)
    xyz = ref_kernels.ref_torsion(raw)
    xyz.backward(inp["grad"].cuda())
    return {"kind": "torsion", "dtype": str(dtype).split(".")[1], "raw": _np(inp["raw"]), "grad": _np(inp["grad"]),
            "bond_lengths": np.array(BOND_LENGTHS), "bond_angles": np.array(BOND_ANGLES), "xyz": _np(xyz), "grad_raw": _np(raw.grad)}


def main() -> None:
    out_dir = Path(sys.argv[sys.argv.index("--out") + 1]) if "--out" in sys.argv else HERE
    out_dir.mkdir(parents=True, exist_ok=True)
    if not torch.cuda.is_available() or not ref_kernels.available("block") or not ref_kernels.available("torsion"):
        raise SystemExit("needs a CUDA device and the reference kernels built by oracle/build_ref.py")
    for case in BLOCK_CASES:
        np.savez_compressed(out_dir / f"{case[0]}.npz", **block_case(*case))
    for case in TORSION_CASES:
        np.savez_compressed(out_dir / f"{case[0]}.npz", **torsion_case(*case))
    print("wrote", len(BLOCK_CASES) + len(TORSION_CASES), "golden files to", out_dir)


if __name__ == "__main__":
    main()
