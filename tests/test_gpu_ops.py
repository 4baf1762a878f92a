"""The torch.library operators (cufk_b200/ops.py) on the GPU: the same kernels as the C++ autograd
wrapper (results and gradients identical), torch.library.opcheck (schema, autograd registration,
fake tensors, AOT dispatch), torch.compile with fullgraph=True, and CUDA-graph capture of the
forward and backward operators."""

from __future__ import annotations

import pytest
import torch

import cufk_b200 as cufk
from cufk_b200 import ops
from oracle import nerf64

pytestmark = pytest.mark.gpu

DEV = "cuda"
ANCHORS = ("p0", "first_direction", "initial_normal")


def inputs(batch, points, dtype, anchors=False, seed=0):
    inp = nerf64.make_inputs(batch, points, seed=seed, anchors=anchors)
    out = {k: v.to(DEV, dtype) for k, v in inp.items()}
    return out


def grads_of(fn, inp, anchors):
    L, A, D = (inp[k].detach().clone().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: inp[k] for k in ANCHORS} if anchors else {}
    xyz = fn(L, A, D, **kw)
    xyz.backward(inp["grad"])
    return xyz.detach(), L.grad, A.grad, D.grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("anchors", [False, True])
def test_operator_matches_autograd_wrapper(dtype, anchors):
    inp = inputs(37, 301, dtype, anchors=anchors, seed=3)
    ref = grads_of(cufk.reconstruct, inp, anchors)
    got = grads_of(ops.reconstruct, inp, anchors)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_single_chain_operator():
    inp = inputs(1, 2051, torch.float32, seed=5)
    L, A, D = (inp[k][0] for k in ("lengths", "angles", "dihedrals"))
    assert torch.equal(ops.reconstruct(L, A, D), cufk.reconstruct(L, A, D))


def test_opcheck_reconstruct():
    inp = inputs(6, 50, torch.float32, anchors=True, seed=7)
    L, A, D = (inp[k].clone().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    torch.library.opcheck(torch.ops.cufk_b200.reconstruct.default, (L, A, D, None, None, None))
    torch.library.opcheck(torch.ops.cufk_b200.reconstruct.default, (L, A, D, inp["p0"], inp["first_direction"], inp["initial_normal"]))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_opcheck_reconstruct_xyz32(dtype):
    inp = inputs(6, 50, dtype, anchors=True, seed=7)
    L, A, D = (inp[k].clone().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    torch.library.opcheck(torch.ops.cufk_b200.reconstruct_xyz32.default, (L, A, D, None, None, None))
    torch.library.opcheck(torch.ops.cufk_b200.reconstruct_xyz32.default, (L, A, D, inp["p0"], inp["first_direction"], inp["initial_normal"]))


def test_opcheck_torsion():
    tin = nerf64.make_torsion_inputs(5, 40, seed=2)
    raw = tin["raw"].to(DEV, torch.float32).requires_grad_(True)
    consts = [float(c) for c in cufk.torsion.torsion_constants(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)]
    torch.library.opcheck(torch.ops.cufk_b200.torsion_reconstruct.default, (raw, consts))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16])
def test_torsion_operator_matches_compile_torsion(dtype):
    tin = nerf64.make_torsion_inputs(9, 130, seed=4)
    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    outs = []
    for fn in (f, lambda r: ops.torsion(r, nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)):
        raw = tin["raw"].to(DEV, dtype).requires_grad_(True)
        xyz = fn(raw)
        xyz.backward(tin["grad"].to(DEV, dtype))
        outs.append((xyz.detach(), raw.grad))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_opcheck_torsion_xyz32(dtype):
    tin = nerf64.make_torsion_inputs(5, 40, seed=2)
    raw = tin["raw"].to(DEV, dtype).requires_grad_(True)
    consts = [float(c) for c in cufk.torsion.torsion_constants(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)]
    torch.library.opcheck(torch.ops.cufk_b200.torsion_reconstruct_xyz32.default, (raw, consts))


def test_compile_fullgraph_traces_through_the_operator():
    inp = inputs(16, 200, torch.float32, seed=11)

    def loss(L, A, D):
        xyz = ops.reconstruct(L, A, D)
        return (xyz[:, 1:] - xyz[:, :-1]).pow(2).sum()

    compiled = torch.compile(loss, backend="aot_eager", fullgraph=True)
    results = []
    for fn in (loss, compiled):
        L, A, D = (inp[k].clone().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
        out = fn(L, A, D)
        out.backward()
        results.append((out.detach(), L.grad, A.grad, D.grad))
    for a, b in zip(*results):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)


def test_cuda_graph_capture_of_forward_and_backward_operators():
    inp = inputs(64, 384, torch.float32, seed=13)
    L, A, D, G = (inp[k] for k in ("lengths", "angles", "dihedrals", "grad"))
    op_f, op_b = torch.ops.cufk_b200.reconstruct, torch.ops.cufk_b200.reconstruct_backward
    eager_xyz = op_f(L, A, D, None, None, None)
    eager_g = op_b(L, A, D, None, None, None, eager_xyz, G)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        op_b(L, A, D, None, None, None, op_f(L, A, D, None, None, None), G)  # warm-up off the capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        xyz = op_f(L, A, D, None, None, None)
        g = op_b(L, A, D, None, None, None, xyz, G)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(xyz, eager_xyz)
    for a, b in zip(g, eager_g):
        assert torch.equal(a, b)
