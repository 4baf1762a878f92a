"""``reconstruct``: the drop-in for ``cufk.reconstruct`` (src/cufk/reconstruct.py:29-81).

Same signature, shapes, dtypes, defaults and error behaviour.  The work runs in the sm_100a
kernels of ``libcufkb.so`` through the C++ autograd wrapper ``_C.apply``.  Omitted anchors are
passed as ``None``; the kernels then use the reference defaults directly instead of building three
small device tensors per call (reconstruct.py:19-26, 69-71).
"""

from __future__ import annotations

import torch

from . import anchors
from ._native import _C

BLOCK_SCAN_MAX_POINT_COUNT = 2051


def _batched_inputs(
    lengths: torch.Tensor,
    angles: torch.Tensor,
    dihedrals: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, bool]:
    single = lengths.dim() == 1
    if single:
        lengths, angles, dihedrals = lengths[None], angles[None], dihedrals[None]
    return lengths, angles, dihedrals, single


def reconstruct(
    lengths: torch.Tensor,
    angles: torch.Tensor,
    dihedrals: torch.Tensor,
    p0: torch.Tensor | None = None,
    first_direction: torch.Tensor | None = None,
    initial_normal: torch.Tensor | None = None,
    *,
    anchor_grads: bool = False,
) -> torch.Tensor:
    r"""Reconstruct Cartesian coordinates from full internal coordinates.

    Args:
        lengths: Bond lengths. CUDA tensor shaped ``(N - 1,)`` for one chain or ``(B, N - 1)``.
        angles: Bond angles in radians, ``(N - 2,)`` or ``(B, N - 2)``.
        dihedrals: Dihedral angles in radians, ``(N - 3,)`` or ``(B, N - 3)``.
        p0: Optional first point, shaped ``(3,)``; default ``(0, 0, 0)``.
        first_direction: Optional first-bond direction, ``(3,)``; default ``(1, 0, 0)``.
        initial_normal: Optional initial plane normal, ``(3,)``; default ``(0, 0, 1)``.

    Returns:
        ``(N, 3)`` for one chain or ``(B, N, 3)``, with the dtype of ``lengths``.

    Notes:
        Inputs are CUDA tensors of one dtype among float16, bfloat16, float32 and float64, with
        4 <= N <= 2051.  Gradients flow to lengths, angles and dihedrals.  Anchors take none and an
        anchor that requires grad raises, as in the reference, unless ``anchor_grads=True`` (an
        extension the reference does not have, see ``anchors.py``): then anchors that require
        grad receive theirs.  16-bit inputs are computed in float32 and rounded once on output.
    """
    lengths, angles, dihedrals, single = _batched_inputs(lengths, angles, dihedrals)
    lengths, angles, dihedrals = lengths.contiguous(), angles.contiguous(), dihedrals.contiguous()
    if anchor_grads and any(a is not None and a.requires_grad for a in (p0, first_direction, initial_normal)):
        xyz = anchors.AnchorGradReconstruct.apply(lengths, angles, dihedrals, p0, first_direction, initial_normal)
    else:
        xyz = _C.apply(lengths, angles, dihedrals, p0, first_direction, initial_normal)
    return xyz[0] if single else xyz


def reconstruct_long(
    lengths: torch.Tensor,
    angles: torch.Tensor,
    dihedrals: torch.Tensor,
    p0: torch.Tensor | None = None,
    first_direction: torch.Tensor | None = None,
    initial_normal: torch.Tensor | None = None,
) -> torch.Tensor:
    r"""``reconstruct`` for chains of any length N >= 4 (float32 and float64).

    The reference stops at ``BLOCK_SCAN_MAX_POINT_COUNT`` points and leaves longer chains to a scan
    it does not ship (README.md:52).  Here each chain is split into balanced segments of at most
    2048 steps, one CTA each; the segments exchange their frame products through a workspace that
    the wrapper allocates per call.  Arguments, shapes, anchors and gradients are those of
    ``reconstruct``.  The backward needs an orthonormal base frame: a collinear first angle or
    degenerate anchors give NaN gradients.
    """
    lengths, angles, dihedrals, single = _batched_inputs(lengths, angles, dihedrals)
    xyz = _C.apply_long(lengths.contiguous(), angles.contiguous(), dihedrals.contiguous(), p0, first_direction, initial_normal)
    return xyz[0] if single else xyz


def reconstruct_packed(
    lengths: torch.Tensor,
    angles: torch.Tensor,
    dihedrals: torch.Tensor,
    chain_points: torch.Tensor,
    p0: torch.Tensor | None = None,
    first_direction: torch.Tensor | None = None,
    initial_normal: torch.Tensor | None = None,
    max_points: int | None = None,
) -> torch.Tensor:
    r"""``reconstruct`` for a packed (ragged) batch: chains of different lengths in one call.

    The reference takes (B, N) batches only (block.cu:367-378).  Here chain b owns the points
    ``[chain_points[b], chain_points[b+1])`` of the packed output, and its rows sit packed the same
    way in the 1-D inputs: ``lengths`` has ``total - B`` entries (chain b's start at
    ``chain_points[b] - b``), ``angles`` ``total - 2B`` (from ``chain_points[b] - 2b``) and
    ``dihedrals`` ``total - 3B`` (from ``chain_points[b] - 3b``).

    Args:
        chain_points: ``(B + 1,)`` int64 offsets, ``chain_points[0] = 0``, nondecreasing, every chain
            with 4 to 2051 points; on the device of ``lengths``.
        max_points: the largest chain's point count.  When omitted it is read from
            ``chain_points`` (one device-to-host copy, which also validates the offsets); pass it to
            keep the call free of host synchronisation (then chains outside ``[4, max_points]`` are
            skipped, their outputs left unset).

    Returns:
        ``(total, 3)`` packed coordinates, ``total = chain_points[-1]``.  Gradients flow to the packed
        lengths, angles and dihedrals; anchors as in ``reconstruct``.
    """
    if max_points is None:
        offsets = chain_points.detach().to("cpu", torch.int64)
        counts = offsets[1:] - offsets[:-1]
        if offsets.numel() < 1 or int(offsets[0]) != 0:
            raise RuntimeError("chain_points must start at 0")
        if counts.numel() and (int(counts.min()) < 4 or int(counts.max()) > BLOCK_SCAN_MAX_POINT_COUNT):
            raise RuntimeError(f"every packed chain needs 4 to {BLOCK_SCAN_MAX_POINT_COUNT} points")
        if int(offsets[-1]) != lengths.numel() + counts.numel():
            raise RuntimeError("chain_points[-1] must equal the packed point count (lengths.numel() + B)")
        max_points = int(counts.max()) if counts.numel() else 4
    return _C.apply_packed(
        lengths.contiguous(), angles.contiguous(), dihedrals.contiguous(), chain_points, int(max_points), p0, first_direction, initial_normal
    )
