"""The reconstruction path as ``torch.library`` custom operators.

``cufk_b200.reconstruct`` keeps the reference's binding: a C++ ``torch::autograd::Function``
reached through pybind (src/cufk/csrc/block.cu:393-445).  Such a binding is opaque to
``torch.compile``, which graph-breaks around it.  The operators below run the same kernels of
``libcufkb.so`` (through the same checked ``_C`` entry points) but are registered with
``torch.library``, each with a fake implementation for shape inference and a registered autograd
formula.  ``torch.compile(fullgraph=True)`` therefore traces through them, and their forward and
backward capture into CUDA graphs like any ATen operator.  The operator is not in the reference
(its path stops at the pybind ``apply``).

Operators (namespace ``cufk_b200``):

* ``reconstruct(lengths, angles, dihedrals, p0?, first_direction?, initial_normal?) -> xyz``:
  ``(B, N-1)``, ``(B, N-2)``, ``(B, N-3)`` in, ``(B, N, 3)`` out;
* ``reconstruct_xyz32(lengths, angles, dihedrals, p0?, first_direction?, initial_normal?) ->
  (xyz, xyz32)``: float16/bfloat16 only; ``xyz`` as ``reconstruct`` gives it and ``xyz32`` the
  float32 positions before rounding, which its autograd formula hands to the backward (a 16-bit
  position is too coarse for the bond directions the backward takes from it);
* ``reconstruct_backward(lengths, angles, dihedrals, p0?, first_direction?, initial_normal?, xyz,
  grad_xyz) -> (grad_lengths, grad_angles, grad_dihedrals)``: reads the forward's output, as the
  C++ wrapper's backward does: ``xyz`` in the inputs' dtype (16-bit types then recompute inside the
  library) or, for float16/bfloat16, the float32 ``xyz32``;
* ``torsion_reconstruct(raw_pairs, constants) -> xyz`` and ``torsion_backward(raw_pairs,
  constants, xyz, grad_xyz) -> grad_raw_pairs``, with ``constants`` the nine floats of
  ``torsion.torsion_constants``; ``torsion_reconstruct_xyz32`` is the float16/bfloat16 forward
  that also returns the float32 positions its backward reads (as ``reconstruct_xyz32``).

Python helpers with the public signatures: ``reconstruct`` (1-D single-chain inputs included; the
16-bit types go through ``reconstruct_xyz32``, the kernels of the C++ wrapper) and
``torsion(raw_pairs, bond_lengths, bond_angles)``.  Anchors take no gradient; an anchor that
requires grad raises the reference's error, as ``cufk_b200.reconstruct`` does.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from ._native import _C
from .torsion import torsion_constants

__all__ = ["reconstruct", "torsion"]


def _check_anchor_grads(p0, first_direction, initial_normal) -> None:
    # the reference's message (src/cufk/csrc/extension_utils.cuh:81)
    for name, t in (("p0", p0), ("first_direction", first_direction), ("initial_normal", initial_normal)):
        if t is not None and t.requires_grad:
            raise RuntimeError(f"{name} gradients are not supported")


def _fake_geometry(lengths: Tensor, angles: Tensor, dihedrals: Tensor) -> tuple[int, int]:
    torch._check(lengths.dim() == 2, lambda: "lengths must have shape (B, N-1)")
    torch._check(angles.dim() == 2, lambda: "angles must have shape (B, N-2)")
    torch._check(dihedrals.dim() == 2, lambda: "dihedrals must have shape (B, N-3)")
    batch, points = lengths.shape[0], lengths.shape[1] + 1
    torch._check(angles.shape[0] == batch and angles.shape[1] == points - 2, lambda: "bad angles shape")
    torch._check(dihedrals.shape[0] == batch and dihedrals.shape[1] == points - 3, lambda: "bad dihedrals shape")
    return batch, points


# ---------------------------------------------------------------------------------------------
# block path
# ---------------------------------------------------------------------------------------------
@torch.library.custom_op("cufk_b200::reconstruct", mutates_args=())
def _reconstruct_op(
    lengths: Tensor,
    angles: Tensor,
    dihedrals: Tensor,
    p0: Optional[Tensor],
    first_direction: Optional[Tensor],
    initial_normal: Optional[Tensor],
) -> Tensor:
    return _C.block_forward(lengths, angles, dihedrals, p0, first_direction, initial_normal)


@_reconstruct_op.register_fake
def _(lengths, angles, dihedrals, p0, first_direction, initial_normal):
    batch, points = _fake_geometry(lengths, angles, dihedrals)
    return lengths.new_empty((batch, points, 3))


@torch.library.custom_op("cufk_b200::reconstruct_backward", mutates_args=())
def _reconstruct_backward_op(
    lengths: Tensor,
    angles: Tensor,
    dihedrals: Tensor,
    p0: Optional[Tensor],
    first_direction: Optional[Tensor],
    initial_normal: Optional[Tensor],
    xyz: Tensor,
    grad_xyz: Tensor,
) -> tuple[Tensor, Tensor, Tensor]:
    if xyz.dtype != lengths.dtype:
        # float16/bfloat16 with the float32 positions of reconstruct_xyz32 (the C++ entry checks both)
        gl, ga, gd = _C.block_backward_from_xyz32(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz.contiguous())
    else:
        gl, ga, gd = _C.block_backward_from_xyz(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz.contiguous())
    return gl, ga, gd


@_reconstruct_backward_op.register_fake
def _(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz):
    _fake_geometry(lengths, angles, dihedrals)
    return torch.empty_like(lengths), torch.empty_like(angles), torch.empty_like(dihedrals)


def _reconstruct_setup(ctx, inputs, output):
    lengths, angles, dihedrals, p0, first_direction, initial_normal = inputs
    ctx.save_for_backward(lengths, angles, dihedrals, p0, first_direction, initial_normal, output)


def _reconstruct_grad(ctx, grad_xyz):
    lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz = ctx.saved_tensors
    gl, ga, gd = _reconstruct_backward_op(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz)
    return gl, ga, gd, None, None, None


_reconstruct_op.register_autograd(_reconstruct_grad, setup_context=_reconstruct_setup)


@torch.library.custom_op("cufk_b200::reconstruct_xyz32", mutates_args=())
def _reconstruct_xyz32_op(
    lengths: Tensor,
    angles: Tensor,
    dihedrals: Tensor,
    p0: Optional[Tensor],
    first_direction: Optional[Tensor],
    initial_normal: Optional[Tensor],
) -> tuple[Tensor, Tensor]:
    xyz, xyz32 = _C.block_forward_xyz32(lengths, angles, dihedrals, p0, first_direction, initial_normal)
    return xyz, xyz32


@_reconstruct_xyz32_op.register_fake
def _(lengths, angles, dihedrals, p0, first_direction, initial_normal):
    batch, points = _fake_geometry(lengths, angles, dihedrals)
    torch._check(lengths.dtype in (torch.float16, torch.bfloat16), lambda: "block_forward_xyz32 supports float16 and bfloat16")
    return lengths.new_empty((batch, points, 3)), lengths.new_empty((batch, points, 3), dtype=torch.float32)


def _reconstruct_xyz32_setup(ctx, inputs, output):
    lengths, angles, dihedrals, p0, first_direction, initial_normal = inputs
    ctx.mark_non_differentiable(output[1])
    ctx.save_for_backward(lengths, angles, dihedrals, p0, first_direction, initial_normal, output[1])


def _reconstruct_xyz32_grad(ctx, grad_xyz, _grad_xyz32):
    lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz32 = ctx.saved_tensors
    gl, ga, gd = _reconstruct_backward_op(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz32, grad_xyz)
    return gl, ga, gd, None, None, None


_reconstruct_xyz32_op.register_autograd(_reconstruct_xyz32_grad, setup_context=_reconstruct_xyz32_setup)


def reconstruct(
    lengths: Tensor,
    angles: Tensor,
    dihedrals: Tensor,
    p0: Tensor | None = None,
    first_direction: Tensor | None = None,
    initial_normal: Tensor | None = None,
) -> Tensor:
    """``cufk_b200.reconstruct`` through the ``cufk_b200::reconstruct`` operator (same arguments,
    shapes, results and gradients)."""
    _check_anchor_grads(p0, first_direction, initial_normal)
    single = lengths.dim() == 1
    if single:
        lengths, angles, dihedrals = lengths[None], angles[None], dihedrals[None]
    args = (lengths.contiguous(), angles.contiguous(), dihedrals.contiguous(), p0, first_direction, initial_normal)
    if lengths.dtype in (torch.float16, torch.bfloat16):
        xyz = _reconstruct_xyz32_op(*args)[0]
    else:
        xyz = _reconstruct_op(*args)
    return xyz[0] if single else xyz


# ---------------------------------------------------------------------------------------------
# torsion-only path
# ---------------------------------------------------------------------------------------------
def _fake_pairs(raw_pairs: Tensor) -> tuple[int, int]:
    torch._check(raw_pairs.dim() == 2, lambda: "raw_pairs must have shape (B, K)")
    torch._check(raw_pairs.shape[1] % 2 == 0, lambda: "raw_pairs second dimension must be even")
    return raw_pairs.shape[0], raw_pairs.shape[1] // 2 + 3


@torch.library.custom_op("cufk_b200::torsion_reconstruct", mutates_args=())
def _torsion_op(raw_pairs: Tensor, constants: list[float]) -> Tensor:
    return _C.torsion_forward(raw_pairs, constants)


@_torsion_op.register_fake
def _(raw_pairs, constants):
    batch, points = _fake_pairs(raw_pairs)
    return raw_pairs.new_empty((batch, points, 3))


@torch.library.custom_op("cufk_b200::torsion_backward", mutates_args=())
def _torsion_backward_op(raw_pairs: Tensor, constants: list[float], xyz: Tensor, grad_xyz: Tensor) -> Tensor:
    # the gradient copies raw_pairs' strides (empty_strided_like, extension_utils.cuh:162-164)
    if xyz.dtype != raw_pairs.dtype:
        # float16/bfloat16 with the float32 positions of torsion_reconstruct_xyz32
        return _C.torsion_backward_from_xyz32(raw_pairs, constants, xyz, grad_xyz.contiguous())
    return _C.torsion_backward_from_xyz(raw_pairs, constants, xyz, grad_xyz.contiguous())


@_torsion_backward_op.register_fake
def _(raw_pairs, constants, xyz, grad_xyz):
    _fake_pairs(raw_pairs)
    return torch.empty_strided(raw_pairs.shape, raw_pairs.stride(), dtype=raw_pairs.dtype, device=raw_pairs.device)


def _torsion_setup(ctx, inputs, output):
    raw_pairs, constants = inputs
    ctx.constants = constants
    ctx.save_for_backward(raw_pairs, output)


def _torsion_grad(ctx, grad_xyz):
    raw_pairs, xyz = ctx.saved_tensors
    return _torsion_backward_op(raw_pairs, ctx.constants, xyz, grad_xyz), None


_torsion_op.register_autograd(_torsion_grad, setup_context=_torsion_setup)


@torch.library.custom_op("cufk_b200::torsion_reconstruct_xyz32", mutates_args=())
def _torsion_xyz32_op(raw_pairs: Tensor, constants: list[float]) -> tuple[Tensor, Tensor]:
    xyz, xyz32 = _C.torsion_forward_xyz32(raw_pairs, constants)
    return xyz, xyz32


@_torsion_xyz32_op.register_fake
def _(raw_pairs, constants):
    batch, points = _fake_pairs(raw_pairs)
    torch._check(raw_pairs.dtype in (torch.float16, torch.bfloat16), lambda: "torsion_forward_xyz32 supports float16 and bfloat16")
    return raw_pairs.new_empty((batch, points, 3)), raw_pairs.new_empty((batch, points, 3), dtype=torch.float32)


def _torsion_xyz32_setup(ctx, inputs, output):
    raw_pairs, constants = inputs
    ctx.constants = constants
    ctx.mark_non_differentiable(output[1])
    ctx.save_for_backward(raw_pairs, output[1])


def _torsion_xyz32_grad(ctx, grad_xyz, _grad_xyz32):
    raw_pairs, xyz32 = ctx.saved_tensors
    return _torsion_backward_op(raw_pairs, ctx.constants, xyz32, grad_xyz), None


_torsion_xyz32_op.register_autograd(_torsion_xyz32_grad, setup_context=_torsion_xyz32_setup)


def torsion(raw_pairs: Tensor, bond_lengths: tuple[float, float, float], bond_angles: tuple[float, float, float]) -> Tensor:
    """``compile_torsion(bond_lengths, bond_angles)(raw_pairs)`` through the
    ``cufk_b200::torsion_reconstruct`` operator (16-bit types: ``torsion_reconstruct_xyz32``, the
    kernels of the C++ wrapper)."""
    consts = torsion_constants(tuple(bond_lengths), tuple(bond_angles))
    if raw_pairs.dtype in (torch.float16, torch.bfloat16):
        return _torsion_xyz32_op(raw_pairs, consts)[0]
    return _torsion_op(raw_pairs, consts)
