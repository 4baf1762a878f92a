"""Loader for the reference's own kernels compiled by ``oracle/build_ref.py`` into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY (imported by ``tests/`` and ``tests/golden/make_golden.py``; never by
the product).  Mirrors the reference's Python layer around its extensions:
``ref_reconstruct`` restates ``cufk.reconstruct`` (src/cufk/reconstruct.py:8-81: single-chain
batching, default anchors built with ``torch.tensor(..., device, dtype)``, ``.contiguous()``), and
``ref_torsion`` calls the ``apply`` of the torsion extension built for the benchmark constants.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
from functools import lru_cache
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
BLOCK_SO = HERE / "_ref" / "block" / "cufk_ref_block.so"
TORSION_SO = HERE / "_ref" / "torsion" / "cufk_ref_torsion.so"


def available(which: str = "block") -> bool:
    return (BLOCK_SO if which == "block" else TORSION_SO).exists()


def _load(name: str, path: Path):
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


@lru_cache(maxsize=None)
def block_module():
    return _load("cufk_ref_block", BLOCK_SO)


@lru_cache(maxsize=None)
def torsion_module():
    return _load("cufk_ref_torsion", TORSION_SO)


def ref_reconstruct(lengths, angles, dihedrals, p0=None, first_direction=None, initial_normal=None):
    single = lengths.dim() == 1
    if single:
        lengths, angles, dihedrals = lengths[None], angles[None], dihedrals[None]

    def anchor(x, vals):
        return torch.tensor(vals, device=lengths.device, dtype=lengths.dtype) if x is None else x

    xyz = block_module().apply(
        lengths.contiguous(),
        angles.contiguous(),
        dihedrals.contiguous(),
        anchor(p0, (0.0, 0.0, 0.0)),
        anchor(first_direction, (1.0, 0.0, 0.0)),
        anchor(initial_normal, (0.0, 0.0, 1.0)),
    )
    return xyz[0] if single else xyz


def ref_torsion(raw_pairs):
    return torsion_module().apply(raw_pairs)
