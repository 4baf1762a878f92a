"""Anchor gradients through the public API on the GPU: ``reconstruct(..., anchor_grads=True)``
against float64 autograd through the oracle forward (oracle/nerf64.py), for float32, float64 and the
16-bit types, single chains, partial requests, and the reference's error when the option is off."""

from __future__ import annotations

import pytest
import torch

import cufk_b200 as cufk
from oracle import nerf64

pytestmark = pytest.mark.gpu

DEV = "cuda"
F64 = torch.float64
KEYS = ("p0", "first_direction", "initial_normal")
# anchor-gradient relative L2 error against float64 (16-bit: their xyz and grad rounding)
TOL = {torch.float32: 1e-4, F64: 1e-9, torch.float16: 2e-2, torch.bfloat16: 1e-1}


def rel(a, b):
    return float((a.double().cpu() - b).norm() / b.norm().clamp_min(1e-300))


def run(inp, dtype, need=(True, True, True), points_single=False):
    L, A, D = (inp[k].to(DEV, dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    anchors = [inp[k].to(DEV, dtype).requires_grad_(n) for k, n in zip(KEYS, need)]
    if points_single:
        xyz = cufk.reconstruct(L[0], A[0], D[0], *anchors, anchor_grads=True)
        xyz.backward(inp["grad"][0].to(DEV, dtype))
    else:
        xyz = cufk.reconstruct(L, A, D, *anchors, anchor_grads=True)
        xyz.backward(inp["grad"].to(DEV, dtype))
    return xyz.detach(), (L.grad, A.grad, D.grad), [a.grad for a in anchors]


@pytest.mark.parametrize("dtype", [torch.float32, F64, torch.float16, torch.bfloat16])
def test_anchor_gradients_match_float64(dtype):
    inp = nerf64.make_inputs(48, 300, seed=21, anchors=True)
    cast = {k: v.to(dtype).to(F64) for k, v in inp.items()}
    ref = nerf64.reconstruct64_anchor_grads(cast["lengths"], cast["angles"], cast["dihedrals"], cast["grad"], *(cast[k] for k in KEYS))
    xyz, _, got = run(inp, dtype)
    for g, r in zip(got, ref[1:]):
        assert rel(g, r) <= TOL[dtype], (dtype, rel(g, r))


def test_parameter_gradients_unchanged_by_anchor_grads():
    inp = nerf64.make_inputs(33, 257, seed=22, anchors=True)
    xyz, grads, _ = run(inp, torch.float32)
    L, A, D = (inp[k].to(DEV).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    ref = cufk.reconstruct(L, A, D, *(inp[k].to(DEV) for k in KEYS))
    ref.backward(inp["grad"].to(DEV))
    assert torch.equal(xyz, ref.detach())
    for a, b in zip(grads, (L.grad, A.grad, D.grad)):
        assert torch.equal(a, b)


def test_partial_requests_and_single_chain():
    inp = nerf64.make_inputs(1, 2051, seed=23, anchors=True)
    ref = nerf64.reconstruct64_anchor_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], *(inp[k] for k in KEYS))
    _, _, got = run(inp, torch.float32, need=(True, False, True), points_single=True)
    assert got[1] is None
    assert rel(got[0], ref[1]) <= 1e-4 and rel(got[2], ref[3]) <= 1e-4


def test_reference_error_without_the_option():
    inp = nerf64.make_inputs(2, 20, seed=24, anchors=True)
    L, A, D = (inp[k].to(DEV) for k in ("lengths", "angles", "dihedrals"))
    p0 = inp["p0"].to(DEV).requires_grad_(True)
    with pytest.raises(RuntimeError, match="p0 gradients are not supported"):
        cufk.reconstruct(L, A, D, p0, inp["first_direction"].to(DEV), inp["initial_normal"].to(DEV))
