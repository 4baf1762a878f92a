"""CPU checks of the float64 oracle (oracle/nerf64.py) before it is trusted as the parity checker.

* autograd of the restated forward equals the restatement of the reference's explicit backward
  formulas (block.cu:206-313, affine.cuh:64-140);
* finite differences (torch.autograd.gradcheck) agree with autograd;
* geometric invariants: bond lengths, bond angles and dihedrals are reproduced from xyz, and
  anchors act as a rigid motion of the default-anchor chain;
* the torsion restatement equals the block restatement with tiled constants and atan2 dihedrals;
* golden vectors produced by the reference's own kernels on a B200 (tests/golden/*.npz) are
  reproduced, which pins the restatement to the reference.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nerf64

F64 = torch.float64
GOLDEN = Path(__file__).resolve().parent / "golden"


def _dihedral(a, b, c, d):
    b0 = a - b
    b1 = c - b
    b2 = d - c
    b1n = b1 / b1.norm(dim=-1, keepdim=True)
    v = b0 - (b0 * b1n).sum(-1, keepdim=True) * b1n
    w = b2 - (b2 * b1n).sum(-1, keepdim=True) * b1n
    x = (v * w).sum(-1)
    y = (torch.linalg.cross(b1n, v, dim=-1) * w).sum(-1)
    return torch.atan2(y, x)


@pytest.mark.parametrize("points", [4, 5, 7, 33])
@pytest.mark.parametrize("anchors", [False, True])
def test_autograd_matches_reference_backward_formulas(points, anchors):
    inp = nerf64.make_inputs(5, points, seed=points, dtype=F64, anchors=anchors)
    a = {k: inp[k] for k in ("p0", "first_direction", "initial_normal")} if anchors else {}
    _, gl, ga, gd = nerf64.reconstruct64_with_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], **a)
    rl, ra, rd = nerf64.block_backward64(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], **a)
    torch.testing.assert_close(gl, rl, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(ga, ra, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(gd, rd, rtol=1e-10, atol=1e-10)


def test_gradcheck_finite_differences():
    inp = nerf64.make_inputs(2, 7, seed=3, dtype=F64, anchors=True)
    L = inp["lengths"].clone().requires_grad_(True)
    A = inp["angles"].clone().requires_grad_(True)
    D = inp["dihedrals"].clone().requires_grad_(True)

    def f(L, A, D):
        return nerf64.reconstruct64(L, A, D, inp["p0"], inp["first_direction"], inp["initial_normal"])

    assert torch.autograd.gradcheck(f, (L, A, D), eps=1e-6, atol=1e-7)


def test_geometry_is_reproduced():
    inp = nerf64.make_inputs(4, 40, seed=11, dtype=F64)
    xyz = nerf64.reconstruct64(inp["lengths"], inp["angles"], inp["dihedrals"])
    bonds = (xyz[:, 1:] - xyz[:, :-1]).norm(dim=-1)
    torch.testing.assert_close(bonds, inp["lengths"], rtol=0, atol=1e-12)
    u = xyz[:, :-2] - xyz[:, 1:-1]
    v = xyz[:, 2:] - xyz[:, 1:-1]
    ang = torch.acos((u * v).sum(-1) / (u.norm(dim=-1) * v.norm(dim=-1)))
    torch.testing.assert_close(ang, inp["angles"], rtol=0, atol=1e-9)
    dih = _dihedral(xyz[:, :-3], xyz[:, 1:-2], xyz[:, 2:-1], xyz[:, 3:])
    diff = torch.remainder(dih - inp["dihedrals"] + math.pi, 2 * math.pi) - math.pi
    assert diff.abs().max() < 1e-9


def test_anchors_are_a_rigid_motion():
    inp = nerf64.make_inputs(3, 25, seed=5, dtype=F64, anchors=True)
    base = nerf64.reconstruct64(inp["lengths"], inp["angles"], inp["dihedrals"])
    moved = nerf64.reconstruct64(inp["lengths"], inp["angles"], inp["dihedrals"], inp["p0"], inp["first_direction"], inp["initial_normal"])
    d0 = inp["first_direction"] / inp["first_direction"].norm()
    n0 = inp["initial_normal"] - (inp["initial_normal"] @ d0) * d0
    n0 = n0 / n0.norm()
    t0 = torch.linalg.cross(n0, d0, dim=-1)
    rot = torch.stack([d0, t0, torch.linalg.cross(d0, t0, dim=-1)], dim=-1)
    expect = inp["p0"] + base @ rot.T
    torch.testing.assert_close(moved, expect, rtol=0, atol=1e-12)


def test_single_chain_shape():
    inp = nerf64.make_inputs(1, 9, seed=1, dtype=F64)
    one = nerf64.reconstruct64(inp["lengths"][0], inp["angles"][0], inp["dihedrals"][0])
    many = nerf64.reconstruct64(inp["lengths"], inp["angles"], inp["dihedrals"])
    assert one.shape == (9, 3)
    torch.testing.assert_close(one, many[0])


def test_torsion_equals_block_path():
    points = 30
    raw = nerf64.make_torsion_inputs(4, points, seed=2, dtype=F64)["raw"]
    xyz_t = nerf64.torsion64(raw, nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    lengths_f, _ = nerf64.torsion_constants(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    L = torch.tensor(lengths_f, dtype=F64)[torch.arange(points - 1) % 3].expand(4, -1)
    A = torch.tensor(nerf64.BACKBONE_ANGLES, dtype=F64)[torch.arange(points - 2) % 3].expand(4, -1)
    D = torch.atan2(raw[:, 0::2], raw[:, 1::2])
    xyz_b = nerf64.reconstruct64(L, A, D)
    torch.testing.assert_close(xyz_t, xyz_b, rtol=0, atol=1e-12)


def test_torsion_gradient_matches_block_chain_rule():
    points = 12
    inp = nerf64.make_torsion_inputs(3, points, seed=4, dtype=F64)
    raw, g = inp["raw"], inp["grad"]
    _, graw = nerf64.torsion64_with_grads(raw, g, nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    lengths_f, _ = nerf64.torsion_constants(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    L = torch.tensor(lengths_f, dtype=F64)[torch.arange(points - 1) % 3].expand(3, -1)
    A = torch.tensor(nerf64.BACKBONE_ANGLES, dtype=F64)[torch.arange(points - 2) % 3].expand(3, -1)
    r = raw.clone().requires_grad_(True)
    D = torch.atan2(r[:, 0::2], r[:, 1::2])
    xyz = nerf64.reconstruct64(L, A, D)
    (expect,) = torch.autograd.grad(xyz, r, g)
    torch.testing.assert_close(graw, expect, rtol=1e-10, atol=1e-12)


def test_input_generator_is_deterministic():
    a = nerf64.make_inputs(3, 10, seed=0)
    b = nerf64.make_inputs(3, 10, seed=0)
    for k in a:
        assert torch.equal(a[k], b[k])
    assert a["lengths"].dtype == torch.float32 and a["lengths"].shape == (3, 9)


def _golden_files():
    return sorted(GOLDEN.glob("*.npz"))


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_reproduces_reference_golden_vectors(path):
    """Golden vectors are outputs of the reference's own kernels (see tests/golden/make_golden.py)."""
    z = np.load(path)
    kind = str(z["kind"])
    dtype = str(z["dtype"])
    # fp32: the stated tolerances (max-abs xyz 5e-4 nm, gradient relative-L2 1e-4) between the
    # reference's fp32 kernels and float64; fp64: agreement to rounding
    tol_x = {"float64": 1e-10, "float32": 5e-4}[dtype]
    tol_g = {"float64": 1e-9, "float32": 1e-4}[dtype]
    if kind == "block":
        single = z["lengths"].ndim == 1
        args = [torch.from_numpy(z[k]).reshape(1, -1) if single else torch.from_numpy(z[k]) for k in ("lengths", "angles", "dihedrals")]
        anchors = {k: torch.from_numpy(z[k]) for k in ("p0", "first_direction", "initial_normal") if k in z.files}
        grad = torch.from_numpy(z["grad"]).reshape(args[0].shape[0], -1, 3)
        xyz, gl, ga, gd = nerf64.reconstruct64_with_grads(*args, grad, **anchors)
        if single:
            xyz, gl, ga, gd = xyz[0], gl[0], ga[0], gd[0]
        assert xyz.shape == z["xyz"].shape
        assert (xyz - torch.from_numpy(z["xyz"]).to(F64)).abs().max() <= tol_x
        if "grad_lengths" in z.files:
            for ours, key in ((gl, "grad_lengths"), (ga, "grad_angles"), (gd, "grad_dihedrals")):
                ref = torch.from_numpy(z[key]).to(F64)
                rel = (ours - ref).norm() / ref.norm()
                assert rel <= tol_g, (key, float(rel))
    else:
        raw = torch.from_numpy(z["raw"])
        xyz, graw = nerf64.torsion64_with_grads(raw, torch.from_numpy(z["grad"]), tuple(z["bond_lengths"]), tuple(z["bond_angles"]))
        assert (xyz - torch.from_numpy(z["xyz"]).to(F64)).abs().max() <= tol_x
        ref = torch.from_numpy(z["grad_raw"]).to(F64)
        if dtype == "float64":
            # The reference scales step k's torsion gradient by 1.0f / bond_len((k+1) % 3), a float32
            # reciprocal of the float32 length, in every dtype (src/cufk/csrc/torsion.cu:213-217);
            # the exact derivative has 1 / bond_len.  Apply that rounding to pin float64 exactly.
            lf = np.float32(z["bond_lengths"]).astype(np.float32)
            ratio = torch.tensor([float(np.float32(1.0) / lf[(k + 1) % 3]) * float(lf[(k + 1) % 3]) for k in range(3)], dtype=F64)
            steps = graw.shape[-1] // 2
            graw = graw * ratio[torch.arange(steps) % 3].repeat_interleave(2)
        rel = (graw - ref).norm() / ref.norm()
        assert rel <= tol_g, float(rel)
