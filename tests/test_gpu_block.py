"""GPU parity of the block path (cufk_b200.reconstruct) against the float64 oracle.

Tolerances (fp32) are the targets of the port: max-abs xyz error <= 5e-4 nm at N = 2051 and
gradient relative L2 <= 1e-4 against float64; fp64 is held to 1e-10.  16-bit storage types compute
in float32, so the bound is the rounding of the output (and of the gradients) to the 16-bit type.
Sizes cover the single/multi-warp and odd/even plan boundaries, batch sizes 1..4096, anchors and
the 1-D single-chain form.
"""

from __future__ import annotations

import math

import pytest
import torch

import cufk_b200 as cufk
from oracle import nerf64

pytestmark = pytest.mark.gpu

DEV = "cuda"
F64 = torch.float64
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")

# xyz max-abs relative to max |x| and gradient relative L2 for the 16-bit types
LOWP = {torch.float16: (2.0**-10, 2.0**-8), torch.bfloat16: (2.0**-7, 2.0**-5)}


def rel_l2(a, b):
    return float((a.to(F64) - b.to(F64)).norm() / b.to(F64).norm().clamp_min(1e-300))


def run_ours(inp, dtype, anchors):
    L = inp["lengths"].to(DEV, dtype).requires_grad_(True)
    A = inp["angles"].to(DEV, dtype).requires_grad_(True)
    D = inp["dihedrals"].to(DEV, dtype).requires_grad_(True)
    kw = {k: inp[k].to(DEV, dtype) for k in ANCHOR_KEYS} if anchors else {}
    xyz = cufk.reconstruct(L, A, D, **kw)
    xyz.backward(inp["grad"].to(DEV, dtype))
    return xyz.detach().cpu(), L.grad.cpu(), A.grad.cpu(), D.grad.cpu()


def run_oracle(inp, dtype, anchors):
    cast = {k: v.to(dtype).to(F64) for k, v in inp.items()}
    kw = {k: cast[k] for k in ANCHOR_KEYS} if anchors else {}
    return nerf64.reconstruct64_with_grads(cast["lengths"], cast["angles"], cast["dihedrals"], cast["grad"], **kw)


def check(ours, ref, dtype, points):
    xyz, gl, ga, gd = ours
    rxyz, rgl, rga, rgd = ref
    err = float((xyz.to(F64) - rxyz).abs().max())
    scale = float(rxyz.abs().max())
    if dtype == torch.float32:
        assert err <= 5e-4, err
        # far below the 5e-4 target for short chains: catches indexing mistakes at small N
        assert err <= 2e-6 * max(1.0, scale) * math.sqrt(points), err
        gtol = 1e-4
    elif dtype == F64:
        assert err <= 1e-10, err
        gtol = 1e-10
    else:
        assert err <= LOWP[dtype][0] * scale, (err, scale)
        gtol = LOWP[dtype][1]
    for name, a, b in (("lengths", gl, rgl), ("angles", ga, rga), ("dihedrals", gd, rgd)):
        r = rel_l2(a, b)
        assert r <= gtol, (name, r)


FP32_POINTS = [4, 5, 6, 7, 8, 33, 100, 257, 258, 384, 513, 514, 768, 769, 1025, 1026, 1027, 1540, 2050, 2051]


@pytest.mark.parametrize("points", FP32_POINTS)
def test_fp32_matches_oracle(points):
    anchors = points % 2 == 1
    inp = nerf64.make_inputs(3, points, seed=points, anchors=anchors)
    check(run_ours(inp, torch.float32, anchors), run_oracle(inp, torch.float32, anchors), torch.float32, points)


@pytest.mark.parametrize("batch", [1, 2, 64, 333, 4096])
def test_fp32_batch_sizes(batch):
    points = 33 if batch > 64 else 700
    inp = nerf64.make_inputs(batch, points, seed=batch)
    check(run_ours(inp, torch.float32, False), run_oracle(inp, torch.float32, False), torch.float32, points)


def test_fp32_throughput_config_and_long_chain_with_anchors():
    # config 1 (B=4096, N=768) in full, and the config 2 shape with anchors on a batch subset
    inp = nerf64.make_inputs(4096, 768, seed=0)
    check(run_ours(inp, torch.float32, False), run_oracle(inp, torch.float32, False), torch.float32, 768)
    inp = nerf64.make_inputs(16, 2051, seed=0, anchors=True)
    check(run_ours(inp, torch.float32, True), run_oracle(inp, torch.float32, True), torch.float32, 2051)


@pytest.mark.parametrize("points", [4, 7, 257, 1027, 2051])
def test_fp64_matches_oracle(points):
    inp = nerf64.make_inputs(2, points, seed=points + 1, dtype=F64, anchors=True)
    check(run_ours(inp, F64, True), run_oracle(inp, F64, True), F64, points)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("points", [4, 33, 1026, 2051])
def test_16bit_matches_oracle(dtype, points):
    inp = nerf64.make_inputs(4, points, seed=points + 7, anchors=points == 33)
    check(run_ours(inp, dtype, points == 33), run_oracle(inp, dtype, points == 33), dtype, points)


def test_single_chain_and_contiguity():
    inp = nerf64.make_inputs(1, 50, seed=9)
    L = inp["lengths"][0].cuda()
    A = inp["angles"][0].cuda()
    D = inp["dihedrals"][0].cuda()
    one = cufk.reconstruct(L, A, D)
    assert one.shape == (50, 3) and one.dtype == torch.float32
    many = cufk.reconstruct(L[None], A[None], D[None])
    torch.testing.assert_close(one, many[0], rtol=0, atol=0)
    # non-contiguous batched views go through .contiguous() as in the reference
    big = nerf64.make_inputs(6, 50, seed=9)
    Ls = big["lengths"].cuda()[::2]
    As = big["angles"].cuda()[::2]
    Ds = big["dihedrals"].cuda()[::2]
    torch.testing.assert_close(cufk.reconstruct(Ls, As, Ds), cufk.reconstruct(Ls.contiguous(), As.contiguous(), Ds.contiguous()))


def test_default_anchors_equal_explicit_defaults():
    inp = nerf64.make_inputs(5, 300, seed=4)
    L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
    explicit = cufk.reconstruct(
        L, A, D, torch.zeros(3, device=DEV), torch.tensor([1.0, 0, 0], device=DEV), torch.tensor([0, 0, 1.0], device=DEV)
    )
    torch.testing.assert_close(cufk.reconstruct(L, A, D), explicit, rtol=0, atol=0)


def test_degenerate_initial_normal_uses_stable_perpendicular():
    inp = nerf64.make_inputs(2, 20, seed=8, dtype=F64)
    fd = torch.tensor([0.3, -0.2, 0.9], dtype=F64)
    nn = 2.0 * fd  # parallel to the first direction: the reference falls back to stable_perpendicular
    kw = {"p0": torch.zeros(3, dtype=F64), "first_direction": fd, "initial_normal": nn}
    ref = nerf64.reconstruct64_with_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], **kw)
    ours = run_ours(dict(inp, **kw), F64, True)
    check(ours, ref, F64, 20)


def test_empty_batch():
    L = torch.empty(0, 9, device=DEV, requires_grad=True)
    A = torch.empty(0, 8, device=DEV, requires_grad=True)
    D = torch.empty(0, 7, device=DEV, requires_grad=True)
    xyz = cufk.reconstruct(L, A, D)
    assert xyz.shape == (0, 10, 3)
    xyz.sum().backward()
    assert L.grad.shape == (0, 9)


def test_gradcheck_fp64():
    inp = nerf64.make_inputs(2, 8, seed=12, dtype=F64, anchors=True)
    L, A, D = (inp[k].cuda().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    anc = [inp[k].cuda() for k in ANCHOR_KEYS]
    assert torch.autograd.gradcheck(lambda a, b, c: cufk.reconstruct(a, b, c, *anc), (L, A, D), eps=1e-6, atol=1e-7)


def test_repeated_calls_are_deterministic():
    inp = nerf64.make_inputs(64, 768, seed=21)
    a = run_ours(inp, torch.float32, False)
    b = run_ours(inp, torch.float32, False)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_full_size_bond_lengths_property():
    inp = nerf64.make_inputs(2048, 2051, seed=3, anchors=True)
    kw = {k: inp[k].cuda() for k in ANCHOR_KEYS}
    xyz = cufk.reconstruct(inp["lengths"].cuda(), inp["angles"].cuda(), inp["dihedrals"].cuda(), **kw)
    bonds = (xyz[:, 1:] - xyz[:, :-1]).double().norm(dim=-1)
    assert float((bonds - inp["lengths"].cuda().double()).abs().max()) < 5e-5


ERRORS = [
    (lambda L, A, D: cufk.reconstruct(L, A.double(), D), "angles must have the same dtype as reference"),
    (lambda L, A, D: cufk.reconstruct(L, A, D.cpu()), "dihedrals must be CUDA"),
    (lambda L, A, D: cufk.reconstruct(L, A[:, :-1], D), "bad angles shape"),
    (lambda L, A, D: cufk.reconstruct(L, A, D[:, :-1]), "bad dihedrals shape"),
    (lambda L, A, D: cufk.reconstruct(L[:, :2], A[:, :1], D[:, :0]), "point_count must be >= 4"),
    (lambda L, A, D: cufk.reconstruct(L.int(), A, D), "lengths must be float32, float64, float16, or bfloat16"),
    (lambda L, A, D: cufk.reconstruct(L, A, D, torch.zeros(4, device=DEV)), "p0 must have shape (3,)"),
    (lambda L, A, D: cufk.reconstruct(L, A, D, None, torch.ones(3, device=DEV, requires_grad=True)), "first_direction gradients are not supported"),
    (lambda L, A, D: cufk.reconstruct(L, A, D, None, None, torch.ones(3, device=DEV, dtype=F64)), "initial_normal must have the same dtype as reference"),
    (lambda L, A, D: cufk.reconstruct(L, A, D, torch.zeros(3)), "p0 must be CUDA"),
]


@pytest.mark.parametrize("case", range(len(ERRORS)))
def test_errors_match_reference_messages(case):
    fn, msg = ERRORS[case]
    inp = nerf64.make_inputs(2, 10, seed=0)
    L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
    with pytest.raises(RuntimeError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        fn(L, A, D)


def test_too_many_points():
    n = cufk.BLOCK_SCAN_MAX_POINT_COUNT + 1
    with pytest.raises(RuntimeError, match="reconstruct supports at most 2048 local transforms"):
        cufk.reconstruct(torch.ones(1, n - 1, device=DEV), torch.ones(1, n - 2, device=DEV), torch.ones(1, n - 3, device=DEV))


def test_current_stream_is_used():
    inp = nerf64.make_inputs(128, 512, seed=2)
    L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
    expect = cufk.reconstruct(L, A, D)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        got = cufk.reconstruct(L, A, D)
    torch.cuda.current_stream().wait_stream(s)
    torch.testing.assert_close(got, expect, rtol=0, atol=0)


def test_cuda_graph_capture_of_forward_and_backward():
    from cufk_b200 import _native

    inp = nerf64.make_inputs(256, 400, seed=6)
    L, A, D, G = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad"))
    C = _native._C
    eager = (C.block_forward(L, A, D, None, None, None), *C.block_backward(L, A, D, None, None, None, G))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        C.block_forward(L, A, D, None, None, None)
        with torch.cuda.graph(g):
            out = (C.block_forward(L, A, D, None, None, None), *C.block_backward(L, A, D, None, None, None, G))
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(out, eager):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
