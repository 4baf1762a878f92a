"""The backward that reads the forward's xyz (bond directions and plane normals instead of rebuilt
local transforms) against the recompute backward and the float64 oracle, through the raw ops, the
C ABI and autograd, including the chains it hands to the recompute form."""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from cufk_b200 import _native
from oracle import nerf64

pytestmark = pytest.mark.gpu

C = _native._C
F64 = torch.float64
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")


def _run_both(inp, dtype, anchors):
    L, A, D, G = (inp[k].to("cuda", dtype) for k in ("lengths", "angles", "dihedrals", "grad"))
    anc = [inp[k].to("cuda", dtype) for k in ANCHOR_KEYS] if anchors else [None, None, None]
    xyz = C.block_forward(L, A, D, *anc)
    from_xyz = C.block_backward_from_xyz(L, A, D, *anc, xyz, G)
    recomputed = C.block_backward(L, A, D, *anc, G)
    return xyz, from_xyz, recomputed


def _oracle(inp, anchors):
    c = {k: v.double() for k, v in inp.items()}
    return nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"], **({k: c[k] for k in ANCHOR_KEYS} if anchors else {}))


def _rel(a, b):
    return float((a.double().cpu() - b.double().cpu()).norm() / b.double().cpu().norm())


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("batch,points,anchors", [(3, 4, False), (2, 5, True), (5, 97, True), (64, 768, False), (7, 1027, True), (4, 2051, True), (1500, 300, False)])
def test_from_xyz_matches_recompute_and_oracle(dtype, batch, points, anchors):
    inp = nerf64.make_inputs(batch, points, seed=points + batch, dtype=dtype, anchors=anchors)
    _, from_xyz, recomputed = _run_both(inp, dtype, anchors)
    rtol = 1e-4 if dtype == torch.float32 else 1e-10
    ref = _oracle(inp, anchors)
    for got, rec, want in zip(from_xyz, recomputed, ref[1:]):
        assert _rel(got, rec) <= rtol
        assert _rel(got, want) <= rtol


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_16bit_from_xyz_recomputes(dtype):
    inp = nerf64.make_inputs(8, 200, seed=3)
    _, from_xyz, recomputed = _run_both(inp, dtype, False)
    for a, b in zip(from_xyz, recomputed):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_non_orthonormal_frame_falls_back_to_recompute():
    inp = nerf64.make_inputs(6, 120, seed=9, dtype=F64, anchors=True)
    inp["angles"][:, 0] = 0.0  # collinear first angle: the base frame is not orthonormal
    _, from_xyz, recomputed = _run_both(inp, F64, True)
    for a, b in zip(from_xyz, recomputed):
        torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_straight_and_zero_length_steps_fall_back(dtype):
    # chain 0: a bond angle of exactly pi (the plane normal is undefined from positions); chain 1: an
    # angle 2 degrees from pi (below the 1e-2 threshold on sin^2); chain 2: a zero-length bond;
    # chain 3: untouched.  Every chain must match the recompute backward and the oracle.
    inp = nerf64.make_inputs(4, 300, seed=11, dtype=F64)
    inp["angles"][0, 150] = math.pi
    inp["angles"][1, 40] = math.pi - math.radians(2.0)
    inp["lengths"][2, 77] = 0.0
    _, from_xyz, recomputed = _run_both(inp, dtype, False)
    rtol = 1e-4 if dtype == torch.float32 else 1e-10
    ref = _oracle(inp, False)
    for got, rec, want in zip(from_xyz, recomputed, ref[1:]):
        for b in range(4):
            assert _rel(got[b], rec[b]) <= rtol, b
            assert _rel(got[b], want[b]) <= rtol, b


def test_c_abi_matches_raw_op():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_backward_from_xyz.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    inp = nerf64.make_inputs(33, 500, seed=5)
    L, A, D, G = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad"))
    xyz = C.block_forward(L, A, D)
    want = C.block_backward_from_xyz(L, A, D, None, None, None, xyz, G)
    got = [torch.full_like(t, float("nan")) for t in (L, A, D)]
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.cufkb_block_backward_from_xyz(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), G.data_ptr(),
                                           *(t.data_ptr() for t in got), 33, 500, stream)
    assert st == 0
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_autograd_reads_saved_xyz_and_detects_inplace_edits():
    import cufk_b200 as cufk

    inp = nerf64.make_inputs(4, 40, seed=4)
    L = inp["lengths"].cuda().requires_grad_(True)
    xyz = cufk.reconstruct(L, inp["angles"].cuda(), inp["dihedrals"].cuda())
    xyz.add_(1.0)  # the saved output was modified in place
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        xyz.sum().backward()


def test_raw_op_checks_xyz_shape():
    inp = nerf64.make_inputs(8, 60, seed=2)
    L, A, D, G = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad"))
    xyz = C.block_forward(L, A, D)
    with pytest.raises(RuntimeError, match="xyz must have shape"):
        C.block_backward_from_xyz(L, A, D, None, None, None, xyz[:, :-1].contiguous(), G)


@pytest.mark.parametrize("offset", [3.0, 300.0])
def test_chain_far_from_origin(offset):
    # at 3 nm the xyz form runs; at 300 nm float32 positions are too coarse for bond directions
    # (bond / |x| < 1e-3) and the chain goes to the recompute form.  Both stay within tolerance.
    inp = nerf64.make_inputs(5, 400, seed=12, anchors=True)
    inp["p0"] = inp["p0"] + offset
    _, from_xyz, recomputed = _run_both(inp, torch.float32, True)
    ref = _oracle(inp, True)
    for got, rec, want in zip(from_xyz, recomputed, ref[1:]):
        assert _rel(got, want) <= 1e-4
        assert _rel(rec, want) <= 1e-4


def test_full_size_linearity_and_agreement():
    # config 1 size: the backward is linear in grad_xyz, and the xyz form agrees with the recompute
    # form on every chain
    inp = nerf64.make_inputs(4096, 768, seed=0)
    L, A, D, G = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad"))
    G2 = torch.randn(G.shape, generator=torch.Generator().manual_seed(1)).cuda()
    xyz = C.block_forward(L, A, D, None, None, None)
    g1 = C.block_backward_from_xyz(L, A, D, None, None, None, xyz, G)
    g2 = C.block_backward_from_xyz(L, A, D, None, None, None, xyz, G2)
    g12 = C.block_backward_from_xyz(L, A, D, None, None, None, xyz, 2.0 * G - 3.0 * G2)
    for a, b, c in zip(g1, g2, g12):
        assert _rel(c, 2.0 * a - 3.0 * b) <= 1e-5
    rec = C.block_backward(L, A, D, None, None, None, G)
    for a, b in zip(g1, rec):
        per_chain = ((a - b).double().norm(dim=1) / b.double().norm(dim=1)).max()
        assert float(per_chain) <= 1e-4
