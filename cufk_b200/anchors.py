"""Gradients of the anchors (p0, first_direction, initial_normal): an extension of the path.

The reference rejects anchors that require grad (src/cufk/csrc/extension_utils.cuh:81,
README.md:39).  ``reconstruct(..., anchor_grads=True)`` gives them gradients instead.

Every atom j >= 3 of a chain is x_j = p2 + F v_j, where (F, p2) is the chain's first frame
(block.cu:113-148) and v_j its local position, which the anchors do not move.  Given the
gradient g of the loss with respect to xyz, the anchors therefore see the loss only through

    S = g_0 . p0 + g_1 . p1 + (g_2 + G) . p2 + <M F0, F>,
    G = sum_{j>=3} g_j,   M = sum_{j>=3} g_j (x_j - p2)^T,

with F0 the frame's value (v_j = F0^T (x_j - p2) for an orthonormal frame), summed over the
chains.  The kernels do the work that scales with the atoms: the forward, and the backward for
lengths, angles and dihedrals (unchanged).  Here one batched contraction forms G and M from the
forward's xyz and the incoming gradient.  Torch's autograd then differentiates S through the
first-frame construction below: a few dozen operations per chain, in float64.

Limit: the frame is orthonormal unless the first bond angle is 0 or pi (sin(angles[0]) = 0).  At
such a degenerate frame the anchor gradients are not defined and come out non-finite or wrong.
"""

from __future__ import annotations

import torch

from ._native import _C

_F64 = torch.float64
# frame_utils.cuh:7 / block.cu:41: the clamp of every normalisation is the float literal 1e-12f
_EPS = float(torch.tensor(1.0e-12, dtype=torch.float32).item())


def _normalized(v: torch.Tensor) -> torch.Tensor:
    # v / sqrt(max(|v|^2, 1e-12)) (frame_utils.cuh:17-20)
    return v / torch.sqrt(torch.clamp((v * v).sum(-1, keepdim=True), min=_EPS))


def first_frame(l0, l1, a0, p0, first_direction, initial_normal):
    """The chain's first frame (block.cu:113-148), differentiable in the anchors.

    ``l0, l1, a0``: (B,) lengths[0], lengths[1], angles[0]; anchors: (3,).  Returns p1, p2 (B, 3)
    and F (B, 3, 3) with columns [dir1 | normal x dir1 | normal].
    """
    dir0 = _normalized(first_direction)
    n0 = initial_normal - (initial_normal * dir0).sum() * dir0
    if float((n0 * n0).sum()) < _EPS:
        # stable_perpendicular (frame_utils.cuh:22-31): dir0 x e_x, or dir0 x e_y when |dir0_x| >= 0.9
        helper = torch.zeros_like(dir0)
        helper[1 if float(dir0[0].abs()) >= 0.9 else 0] = 1.0
        n0 = torch.linalg.cross(dir0, helper)
    n0 = _normalized(n0)
    turn0 = _normalized(torch.linalg.cross(n0, dir0))
    p1 = p0 + l0[:, None] * dir0
    dir1 = -torch.cos(a0)[:, None] * dir0 + torch.sin(a0)[:, None] * turn0
    p2 = p1 + l1[:, None] * dir1
    normal = _normalized(torch.linalg.cross(dir0.expand_as(dir1), dir1, dim=-1))
    side = torch.linalg.cross(normal, dir1, dim=-1)
    return p1, p2, torch.stack([dir1, side, normal], dim=-1)


_DEFAULTS = ((0.0, 0.0, 0.0), (1.0, 0.0, 0.0), (0.0, 0.0, 1.0))  # reconstruct.py:69-71


def anchor_gradients(lengths, angles, anchors, xyz, grad_xyz, needs):
    """Gradients of (p0, first_direction, initial_normal) for the anchors flagged in ``needs``
    (None for the others), from the forward's ``xyz`` and the gradient ``grad_xyz``, both (B, N, 3)."""
    dev = lengths.device
    compute = _F64 if lengths.dtype == _F64 else torch.float32
    with torch.enable_grad():
        leaves = []
        values = []
        for t, default, need in zip(anchors, _DEFAULTS, needs):
            v = torch.tensor(default, dtype=_F64, device=dev) if t is None else t.detach().to(_F64)
            if need:
                v = v.clone().requires_grad_(True)
                leaves.append(v)
            values.append(v)
        p0, fd, nn = values
        l0, l1, a0 = (x.detach().to(_F64) for x in (lengths[:, 0], lengths[:, 1], angles[:, 0]))
        p1, p2, F = first_frame(l0, l1, a0, p0, fd, nn)
        g = grad_xyz.to(compute)
        rel = xyz[:, 3:].to(compute) - p2.detach().to(compute)[:, None, :]
        M = torch.einsum("bjk,bjl->bkl", g[:, 3:], rel).to(_F64)
        G = g[:, 3:].sum(1).to(_F64)
        g = g[:, :3].to(_F64)
        S = (g[:, 0].sum(0) * p0).sum() + (g[:, 1] * p1).sum() + ((g[:, 2] + G) * p2).sum() + ((M @ F.detach()) * F).sum()
        grads = iter(torch.autograd.grad(S, leaves, allow_unused=True)) if leaves else iter(())
    out = []
    for t, need in zip(anchors, needs):
        if not need:
            out.append(None)
            continue
        # an anchor the frame does not use (the initial normal when it is parallel to the first
        # direction: stable_perpendicular replaces it) has a zero gradient
        gr = next(grads)
        out.append(torch.zeros_like(t) if gr is None else gr.to(t.dtype))
    return out


class AnchorGradReconstruct(torch.autograd.Function):
    """The block path with anchor gradients: the kernels for xyz and for the gradients of lengths,
    angles and dihedrals (the same as ``_C.apply``), ``anchor_gradients`` for the anchors."""

    @staticmethod
    def forward(ctx, lengths, angles, dihedrals, p0, first_direction, initial_normal):
        anchors = [None if a is None else a.detach() for a in (p0, first_direction, initial_normal)]
        xyz = _C.block_forward(lengths.detach(), angles.detach(), dihedrals.detach(), *anchors)
        ctx.save_for_backward(lengths, angles, dihedrals, xyz)
        ctx.anchors = anchors
        return xyz

    @staticmethod
    def backward(ctx, grad_xyz):
        lengths, angles, dihedrals, xyz = ctx.saved_tensors
        grad_xyz = grad_xyz.contiguous()
        gl, ga, gd = _C.block_backward_from_xyz(lengths, angles, dihedrals, *ctx.anchors, xyz, grad_xyz)
        gp = anchor_gradients(lengths, angles, ctx.anchors, xyz, grad_xyz, ctx.needs_input_grad[3:6])
        return (gl, ga, gd, *gp)
