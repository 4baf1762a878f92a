"""Parity on whole configuration batches, every chain checked: configs 2, 3 and 4 at their full
sizes through the public API (autograd), against the float64 oracle run on the GPU (the oracle's
arithmetic is device-independent; on the CPU its sequential loop over steps takes minutes at these
sizes).  The other tests check these shapes on batch slices; these cover every chain of the batch
the benchmark times, per chain.  Config 1 is checked in full in test_gpu_block.py."""

from __future__ import annotations

import math

import pytest
import torch

import cufk_b200 as cufk
from oracle import nerf64

pytestmark = pytest.mark.gpu

DEV = "cuda"
F64 = torch.float64
ANCHORS = ("p0", "first_direction", "initial_normal")
# xyz: max-abs error (scaled by max |x| for the 16-bit types); gradients: relative L2 per chain
BLOCK_TOL = {torch.float32: (5e-4, 1e-4), F64: (1e-9, 1e-9), torch.float16: (2.0**-10, 2.0**-8), torch.bfloat16: (2.0**-7, 2.0**-5)}


def per_chain_rel(got, want):
    """Largest relative L2 error over the chains (rows of the leading dimension)."""
    num = (got.to(F64) - want).flatten(1).norm(dim=1)
    den = want.flatten(1).norm(dim=1).clamp_min(1e-300)
    return float((num / den).max())


def check_block(batch, points, dtype, anchors, seed):
    inp = nerf64.make_inputs(batch, points, seed=seed, anchors=anchors)
    # the oracle sees exactly the values the kernels see (the inputs rounded to dtype)
    cast = {k: v.to(DEV, dtype) for k, v in inp.items()}
    L, A, D = (cast[k].clone().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: cast[k] for k in ANCHORS} if anchors else {}
    xyz = cufk.reconstruct(L, A, D, **kw)
    xyz.backward(cast["grad"])
    ref = nerf64.reconstruct64_with_grads(
        cast["lengths"].to(F64), cast["angles"].to(F64), cast["dihedrals"].to(F64), cast["grad"].to(F64), **{k: v.to(F64) for k, v in kw.items()}
    )
    xt, gt = BLOCK_TOL[dtype]
    err = float((xyz.detach().to(F64) - ref[0]).abs().max())
    scale = float(ref[0].abs().max())
    if dtype in (torch.float16, torch.bfloat16):
        xt *= scale
    elif dtype == torch.float32:
        # far below the 5e-4 target: an indexing mistake anywhere in the batch shows
        xt = min(xt, 2e-6 * max(1.0, scale) * math.sqrt(points))
    assert err <= xt, (err, xt)
    for name, g, want in zip(("lengths", "angles", "dihedrals"), (L.grad, A.grad, D.grad), ref[1:]):
        r = per_chain_rel(g, want)
        assert r <= gt, (name, r)


@pytest.mark.parametrize("dtype", [torch.float32, F64])
def test_config2_full_batch(dtype):
    # B=2048 chains of N=2051 with anchors, every chain
    check_block(2048, 2051, dtype, anchors=True, seed=2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_config4_full_batch(dtype):
    # B=8192 chains of N=1026, every chain (the 16-bit forward with float32 positions, and the
    # backward from them)
    check_block(8192, 1026, dtype, anchors=False, seed=4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_config3_full_batch(dtype):
    # torsion-only, B=16384 chains of N=768, every chain
    inp = nerf64.make_torsion_inputs(16384, 768, seed=3)
    raw = inp["raw"].to(DEV, dtype)
    grad = inp["grad"].to(DEV, dtype)
    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    r = raw.clone().requires_grad_(True)
    xyz = f(r)
    xyz.backward(grad)
    rxyz, rgraw = nerf64.torsion64_with_grads(raw.to(F64), grad.to(F64), nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    xt, gt = (5e-4, 1e-4) if dtype == torch.float32 else (2.0**-7, 2.0**-5)
    err = float((xyz.detach().to(F64) - rxyz).abs().max())
    if dtype == torch.bfloat16:
        xt *= float(rxyz.abs().max())
    assert err <= xt, err
    assert per_chain_rel(r.grad, rgraw) <= gt
