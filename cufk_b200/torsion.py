"""``compile_torsion``: the drop-in for ``cufk.compile_torsion`` (src/cufk/torsion.py:89-135).

The reference JIT-compiles one extension per constant set, with the constants as ``-D`` macros
(torsion.py:72-86, ~5 minutes per set).  Here the constants are a run-time argument of one
prebuilt sm_100a kernel, so "compiling" is instantaneous; the returned callable is still cached
per (bond_lengths, bond_angles), exactly as the reference caches it (torsion.py:50, 119-135).
Bond lengths are rounded to float32 inside the library, as the reference's compiled constants are,
and the angle sine/cosine are taken in double on the host (torsion.py:81-86).
"""

from __future__ import annotations

import math
from typing import Protocol

import torch

from ._native import _C


class TorsionReconstructor(Protocol):
    def __call__(self, raw_pairs: torch.Tensor) -> torch.Tensor:
        r"""Reconstruct ``(B, N, 3)`` coordinates from raw ``(B, 2 * (N - 3))`` torsion pairs.

        ``raw_pairs`` interleaves unnormalised ``[sin_raw, cos_raw]`` per dihedral; each pair is
        normalised inside the kernel.  Rows may have any stride, elements within a row are
        contiguous.  Gradients flow to ``raw_pairs``.
        """
        ...


_TORSION_CALLS: dict[tuple[tuple[float, float, float], tuple[float, float, float]], TorsionReconstructor] = {}


def _as_triple(values, label: str) -> tuple[float, float, float]:
    assert len(values) == 3, f"{label} must have 3 elements"
    return (values[0], values[1], values[2])


def torsion_constants(lengths: tuple[float, float, float], angles: tuple[float, float, float]) -> list[float]:
    """[3 lengths, 3 angle sines, 3 angle cosines] as passed to the kernels."""
    return [float(x) for x in lengths] + [math.sin(float(a)) for a in angles] + [math.cos(float(a)) for a in angles]


class _Reconstructor:
    __slots__ = ("constants", "bond_lengths", "bond_angles")

    def __init__(self, lengths, angles):
        self.bond_lengths = lengths
        self.bond_angles = angles
        self.constants = torsion_constants(lengths, angles)

    def __call__(self, raw_pairs: torch.Tensor) -> torch.Tensor:
        return _C.torsion_apply(raw_pairs, self.constants)

    def __repr__(self) -> str:
        return f"TorsionReconstructor(bond_lengths={self.bond_lengths}, bond_angles={self.bond_angles})"


def compile_torsion(
    bond_lengths: tuple[float, float, float],
    bond_angles: tuple[float, float, float],
) -> TorsionReconstructor:
    r"""Return the cached torsion-only reconstructor for a fixed backbone geometry.

    Args:
        bond_lengths: Three repeating bond lengths (step k uses ``bond_lengths[(k + 2) % 3]``).
        bond_angles: Three repeating bond angles in radians (step k uses ``(k + 1) % 3``).

    Returns:
        A callable ``reconstruct(raw_pairs) -> xyz``; repeated calls with equal constants return
        the same object.
    """
    lengths = _as_triple(bond_lengths, "bond_lengths")
    angles = _as_triple(bond_angles, "bond_angles")
    key = (lengths, angles)
    if key not in _TORSION_CALLS:
        _TORSION_CALLS[key] = _Reconstructor(lengths, angles)
    return _TORSION_CALLS[key]
