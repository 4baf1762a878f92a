"""GPU parity of the torsion-only path (cufk_b200.compile_torsion) against the float64 oracle."""

from __future__ import annotations

import math

import pytest
import torch

import cufk_b200 as cufk
from oracle import nerf64

pytestmark = pytest.mark.gpu

F64 = torch.float64
LENGTHS = nerf64.BACKBONE_LENGTHS
ANGLES = nerf64.BACKBONE_ANGLES
TOL = {torch.float32: (5e-4, 1e-4), F64: (1e-10, 1e-10), torch.bfloat16: (2.0**-7, 2.0**-5), torch.float16: (2.0**-10, 2.0**-8)}


def run(raw, grad, dtype, lengths=LENGTHS, angles=ANGLES):
    f = cufk.compile_torsion(lengths, angles)
    r = raw.to("cuda", dtype).requires_grad_(True)
    xyz = f(r)
    xyz.backward(grad.to("cuda", dtype))
    return xyz.detach().cpu(), r.grad.cpu()


def check(raw, grad, dtype, lengths=LENGTHS, angles=ANGLES):
    xyz, graw = run(raw, grad, dtype, lengths, angles)
    rxyz, rgraw = nerf64.torsion64_with_grads(raw.to(dtype).to(F64), grad.to(dtype).to(F64), lengths, angles)
    err = float((xyz.to(F64) - rxyz).abs().max())
    xt, gt = TOL[dtype]
    if dtype in (torch.bfloat16, torch.float16):
        xt *= float(rxyz.abs().max())
    assert err <= xt, err
    rel = float((graw.to(F64) - rgraw).norm() / rgraw.norm())
    assert rel <= gt, rel


@pytest.mark.parametrize("points", [4, 5, 6, 33, 258, 768, 1027, 2051])
def test_fp32(points):
    inp = nerf64.make_torsion_inputs(3, points, seed=points)
    check(inp["raw"], inp["grad"], torch.float32)


@pytest.mark.parametrize("dtype", [F64, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("points", [4, 768, 2051])
def test_other_dtypes(dtype, points):
    inp = nerf64.make_torsion_inputs(2, points, seed=points + 3, dtype=F64)
    check(inp["raw"], inp["grad"], dtype)


def test_benchmark_config_fp32():
    inp = nerf64.make_torsion_inputs(16384, 768, seed=0)
    # parity on a slice; the full batch runs through the same plan
    xyz, graw = run(inp["raw"], inp["grad"], torch.float32)
    sub = slice(0, 512)
    rxyz, rg = nerf64.torsion64_with_grads(inp["raw"][sub].double(), inp["grad"][sub].double(), LENGTHS, ANGLES)
    assert float((xyz[sub].double() - rxyz).abs().max()) <= 5e-4
    assert float((graw[sub].double() - rg).norm() / rg.norm()) <= 1e-4


def test_row_stride_and_gradient_strides():
    points = 100
    width = 2 * (points - 3)
    inp = nerf64.make_torsion_inputs(5, points, seed=1)
    big = torch.randn(5, width + 6, device="cuda")
    big[:, :width] = inp["raw"].cuda()
    view = big[:, :width]
    assert view.stride(0) == width + 6
    f = cufk.compile_torsion(LENGTHS, ANGLES)
    v = view.detach().requires_grad_(True)
    xyz = f(v)
    xyz.backward(inp["grad"].cuda())
    assert v.grad.stride() == v.stride() or v.grad.is_contiguous()
    xyz_c, g_c = run(inp["raw"], inp["grad"], torch.float32)
    torch.testing.assert_close(xyz.detach().cpu(), xyz_c, rtol=0, atol=0)
    torch.testing.assert_close(v.grad.cpu(), g_c, rtol=0, atol=0)


def test_custom_constants():
    lengths = (0.1, 0.2, 0.15)
    angles = (1.5, 2.5, 2.0)
    inp = nerf64.make_torsion_inputs(4, 200, seed=6)
    check(inp["raw"], inp["grad"], torch.float32, lengths, angles)


def test_tiny_pairs_are_clamped():
    inp = nerf64.make_torsion_inputs(2, 20, seed=2, dtype=F64)
    raw = inp["raw"].clone()
    raw[:, 4:6] = 1e-12  # below the 1e-8 norm clamp
    check(raw, inp["grad"], F64)


def test_equals_block_path():
    points = 300
    inp = nerf64.make_torsion_inputs(8, points, seed=5)
    raw = inp["raw"].cuda()
    xyz_t = cufk.compile_torsion(LENGTHS, ANGLES)(raw)
    lf, _ = nerf64.torsion_constants(LENGTHS, ANGLES)
    L = torch.tensor(lf, device="cuda")[torch.arange(points - 1, device="cuda") % 3].expand(8, -1)
    A = torch.tensor(ANGLES, device="cuda")[torch.arange(points - 2, device="cuda") % 3].expand(8, -1)
    D = torch.atan2(raw[:, 0::2], raw[:, 1::2])
    xyz_b = cufk.reconstruct(L, A, D)
    assert float((xyz_t - xyz_b).abs().max()) < 2e-4


def test_errors():
    f = cufk.compile_torsion(LENGTHS, ANGLES)
    with pytest.raises(RuntimeError, match="raw_pairs second dimension must be even"):
        f(torch.ones(2, 7, device="cuda"))
    with pytest.raises(RuntimeError, match=r"raw_pairs must have shape \(B, K\)"):
        f(torch.ones(8, device="cuda"))
    with pytest.raises(RuntimeError, match=r"raw_pairs must have stride\(1\) == 1"):
        f(torch.ones(8, 4, device="cuda").t())
    with pytest.raises(RuntimeError, match="point_count must be >= 4"):
        f(torch.ones(2, 0, device="cuda"))
    with pytest.raises(RuntimeError, match="torsion_pairs supports at most 2048 local transforms"):
        f(torch.ones(1, 2 * 2049, device="cuda"))
    with pytest.raises(AssertionError):
        cufk.compile_torsion((1.0, 2.0), ANGLES)


def test_empty_batch():
    f = cufk.compile_torsion(LENGTHS, ANGLES)
    r = torch.empty(0, 10, device="cuda", requires_grad=True)
    xyz = f(r)
    assert xyz.shape == (0, 8, 3)
    xyz.sum().backward()
    assert r.grad.shape == (0, 10)


def test_angle_constants_in_double():
    c = cufk.compile_torsion(LENGTHS, ANGLES).constants
    assert c[3:6] == [math.sin(a) for a in ANGLES] and c[6:9] == [math.cos(a) for a in ANGLES]
