"""Torsion backward from the forward's xyz (the reference's own torsion backward reads its saved
xyz, src/cufk/csrc/torsion.cu:297-381) against the recompute backward and the float64 oracle."""

from __future__ import annotations

import pytest
import torch

import cufk_b200 as cufk
from cufk_b200 import _native
from cufk_b200.torsion import torsion_constants as _constants
from oracle import nerf64

pytestmark = pytest.mark.gpu

C = _native._C
F64 = torch.float64


def _rel(a, b):
    return float((a.double().cpu() - b.double().cpu()).norm() / b.double().cpu().norm())


def _consts(lengths=nerf64.BACKBONE_LENGTHS, angles=nerf64.BACKBONE_ANGLES):
    return _constants(lengths, angles)


@pytest.mark.parametrize("dtype", [torch.float32, F64])
@pytest.mark.parametrize("batch,points", [(3, 4), (2, 5), (5, 97), (64, 768), (3, 2051), (700, 300)])
def test_from_xyz_matches_recompute_and_oracle(dtype, batch, points):
    inp = nerf64.make_torsion_inputs(batch, points, seed=batch + points, dtype=dtype)
    raw, G = inp["raw"].cuda(), inp["grad"].cuda()
    consts = _consts()
    xyz = C.torsion_forward(raw, consts)
    got = C.torsion_backward_from_xyz(raw, consts, xyz, G)
    rec = C.torsion_backward(raw, consts, G)
    _, want = nerf64.torsion64_with_grads(inp["raw"].double(), inp["grad"].double(), nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    tol = 1e-4 if dtype == torch.float32 else 1e-10
    assert _rel(got, rec) <= tol
    assert _rel(got, want) <= tol


def test_row_strides():
    inp = nerf64.make_torsion_inputs(6, 50, seed=3)
    wide = torch.zeros(6, 2 * 47 + 9, device="cuda")
    wide[:, : 2 * 47] = inp["raw"].cuda()
    raw = wide[:, : 2 * 47]
    consts = _consts()
    xyz = C.torsion_forward(raw, consts)
    got = C.torsion_backward_from_xyz(raw, consts, xyz, inp["grad"].cuda())
    assert got.stride() == raw.stride()
    rec = C.torsion_backward(raw.contiguous(), consts, inp["grad"].cuda())
    assert _rel(got, rec) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, F64])
def test_short_bond_falls_back_to_recompute(dtype):
    # a compiled bond of 1e-9 nm: its direction cannot come from positions, the recompute form runs
    lengths = (0.14685231, 1e-9, 0.13405086)
    inp = nerf64.make_torsion_inputs(4, 200, seed=7, dtype=dtype)
    raw, G = inp["raw"].cuda(), inp["grad"].cuda()
    consts = _consts(lengths)
    xyz = C.torsion_forward(raw, consts)
    got = C.torsion_backward_from_xyz(raw, consts, xyz, G)
    rec = C.torsion_backward(raw, consts, G)
    # the same recompute form, over another split of the steps between threads
    assert _rel(got, rec) <= (1e-6 if dtype == torch.float32 else 1e-12)


@pytest.mark.parametrize("dtype", [torch.float32, F64])
def test_clamped_pair_falls_back_to_recompute(dtype):
    # a (sin, cos) pair below the norm clamp is not a rotation: the chain takes the recompute form;
    # the other chains of the batch keep the xyz form
    inp = nerf64.make_torsion_inputs(5, 300, seed=8, dtype=dtype)
    raw, G = inp["raw"].cuda(), inp["grad"].cuda()
    raw[2, 40:42] = 1e-12
    consts = _consts()
    xyz = C.torsion_forward(raw, consts)
    got = C.torsion_backward_from_xyz(raw, consts, xyz, G)
    rec = C.torsion_backward(raw, consts, G)
    assert bool(torch.isfinite(got).all())
    for b in (0, 1, 3, 4):
        assert _rel(got[b], rec[b]) <= (1e-5 if dtype == torch.float32 else 1e-11), b
    # the clamped chain: the step scales its frame by ~1e-4, so two splits of the steps between
    # threads round differently by far more than a well-conditioned chain's
    assert _rel(got[2], rec[2]) <= (1e-2 if dtype == torch.float32 else 1e-6)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_16bit_recomputes(dtype):
    inp = nerf64.make_torsion_inputs(8, 100, seed=2)
    raw, G = inp["raw"].to("cuda", dtype), inp["grad"].to("cuda", dtype)
    consts = _consts()
    xyz = C.torsion_forward(raw, consts)
    torch.testing.assert_close(C.torsion_backward_from_xyz(raw, consts, xyz, G), C.torsion_backward(raw, consts, G), rtol=0, atol=0)


def test_autograd_saves_xyz_and_detects_inplace_edits():
    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    raw = nerf64.make_torsion_inputs(2, 30, seed=1)["raw"].cuda().requires_grad_(True)
    xyz = f(raw)
    xyz.mul_(2.0)
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        xyz.sum().backward()
