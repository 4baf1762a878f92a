"""Large (and odd) batch sizes through the public API, every dtype: chains at the start, middle and
end of the batch are checked against the float64 oracle."""

from __future__ import annotations

import pytest
import torch

import cufk_b200 as cufk
from oracle import nerf64

pytestmark = pytest.mark.gpu

F64 = torch.float64
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")
TOL = {torch.float32: (5e-4, 1e-4), torch.bfloat16: (2.0**-7, 2.0**-5), torch.float16: (2.0**-10, 2.0**-8)}


def _rows(b):
    return sorted({0, 1, b // 2, b // 2 + 1, b - 2, b - 1})


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch,points", [(2049, 33), (1999, 768), (1185, 2051), (3001, 4)])
def test_block_large_batch(dtype, batch, points):
    anchors = points != 4
    inp = nerf64.make_inputs(batch, points, seed=batch + points, anchors=anchors)
    L, A, D = (inp[k].to("cuda", dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: inp[k].to("cuda", dtype) for k in ANCHOR_KEYS} if anchors else {}
    xyz = cufk.reconstruct(L, A, D, **kw)
    xyz.backward(inp["grad"].to("cuda", dtype))
    rows = _rows(batch)
    cast = {k: (v[rows] if v.dim() > 1 else v).to(dtype).to(F64) for k, v in inp.items()}
    ref = nerf64.reconstruct64_with_grads(cast["lengths"], cast["angles"], cast["dihedrals"], cast["grad"], **({k: cast[k] for k in ANCHOR_KEYS} if anchors else {}))
    xt, gt = TOL[dtype]
    scale = float(ref[0].abs().max()) if dtype != torch.float32 else 1.0
    assert float((xyz.detach()[rows].double().cpu() - ref[0]).abs().max()) <= xt * scale
    for got, want in zip((L.grad, A.grad, D.grad), ref[1:]):
        rel = float((got[rows].double().cpu() - want).norm() / want.norm())
        assert rel <= gt, rel


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("batch,points", [(2049, 100), (1201, 2051)])
def test_torsion_large_batch(dtype, batch, points):
    inp = nerf64.make_torsion_inputs(batch, points, seed=batch)
    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    raw = inp["raw"].to("cuda", dtype).requires_grad_(True)
    xyz = f(raw)
    xyz.backward(inp["grad"].to("cuda", dtype))
    rows = _rows(batch)
    rx, rg = nerf64.torsion64_with_grads(inp["raw"][rows].to(dtype).double(), inp["grad"][rows].to(dtype).double(), nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    xt, gt = TOL[dtype]
    scale = float(rx.abs().max()) if dtype != torch.float32 else 1.0
    assert float((xyz.detach()[rows].double().cpu() - rx).abs().max()) <= xt * scale
    assert float((raw.grad[rows].double().cpu() - rg).norm() / rg.norm()) <= gt


def test_chain_result_does_not_depend_on_the_batch():
    # a chain computed alone (the plan gives it more warps) and inside a large batch
    inp = nerf64.make_inputs(2400, 300, seed=5)
    L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
    big = cufk.reconstruct(L, A, D)
    for r in (0, 1, 1199, 2399):
        one = cufk.reconstruct(L[r], A[r], D[r])
        assert float((big[r] - one).abs().max()) <= 1e-5


def test_grid_beyond_65535_chains():
    # one CTA per chain: 70000 chains need a grid larger than the 16-bit y/z grid limits
    inp = nerf64.make_inputs(70000, 6, seed=8)
    L, A, D = (inp[k].cuda().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    xyz = cufk.reconstruct(L, A, D)
    xyz.backward(inp["grad"].cuda())
    rows = [0, 1, 35000, 65535, 65536, 69999]
    c = {k: v[rows].double() for k, v in inp.items()}
    ref = nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"])
    assert float((xyz.detach()[rows].double().cpu() - ref[0]).abs().max()) <= 1e-5
    for got, want in zip((L.grad, A.grad, D.grad), ref[1:]):
        assert float((got[rows].double().cpu() - want).norm() / want.norm()) <= 1e-5
