"""A fused downstream consumer: reconstruction and a coordinate loss in one kernel.

``reconstruct_mse(lengths, angles, dihedrals, target)`` returns each chain's mean squared distance
to a target structure, (1/N) sum_j |x_j - t_j|^2, with x the chain ``reconstruct`` would give.  The
reference's path ends at xyz; a caller then writes xyz to memory, reads it back for the loss,
writes dL/dxyz, and reads xyz and dL/dxyz again in the backward.  Here one kernel per call
(``block_mse_kernel``) keeps each chain in shared memory from its parameters to its loss and, when
gradients are needed, to d loss / d (lengths, angles, dihedrals).  So HBM sees only the parameters,
the target and those gradients: 36 B per atom in float32, against ~120 B for the unfused
sequence.  The gradients are formed in the forward call, as fused cross-entropy kernels do.  The
autograd backward only scales them by the incoming per-chain gradient.

float32 and float64.  Anchors as in ``reconstruct`` (no anchor gradients); the target takes no
gradient.
"""

from __future__ import annotations

import torch

from ._native import _C


class _MseReconstruct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lengths, angles, dihedrals, target, p0, first_direction, initial_normal):
        need = any(ctx.needs_input_grad[:3])
        loss, gl, ga, gd = _C.block_mse(
            lengths.detach(), angles.detach(), dihedrals.detach(), p0, first_direction, initial_normal, target.detach(), need
        )
        if need:
            ctx.save_for_backward(gl, ga, gd)
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        gl, ga, gd = ctx.saved_tensors
        scale = grad_loss[:, None]
        return gl * scale, ga * scale, gd * scale, None, None, None, None


def reconstruct_mse(
    lengths: torch.Tensor,
    angles: torch.Tensor,
    dihedrals: torch.Tensor,
    target: torch.Tensor,
    p0: torch.Tensor | None = None,
    first_direction: torch.Tensor | None = None,
    initial_normal: torch.Tensor | None = None,
) -> torch.Tensor:
    r"""Mean squared distance of each chain's reconstruction to ``target``, fused in one kernel.

    Args:
        lengths, angles, dihedrals, p0, first_direction, initial_normal: as for ``reconstruct``
            (``(B, N-1)``/``(B, N-2)``/``(B, N-3)`` or one chain), float32 or float64.
        target: ``(B, N, 3)`` (or ``(N, 3)`` for one chain), the dtype of ``lengths``.

    Returns:
        ``(B,)`` losses (a 0-d tensor for one chain); differentiable with respect to lengths,
        angles and dihedrals.
    """
    if target.requires_grad:
        raise RuntimeError("reconstruct_mse: target gradients are not supported")
    single = lengths.dim() == 1
    if single:
        lengths, angles, dihedrals, target = lengths[None], angles[None], dihedrals[None], target[None]
    loss = _MseReconstruct.apply(
        lengths.contiguous(), angles.contiguous(), dihedrals.contiguous(), target.contiguous(), p0, first_direction, initial_normal
    )
    return loss[0] if single else loss
