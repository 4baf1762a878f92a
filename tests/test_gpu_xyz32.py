"""The float16/bfloat16 path that keeps the forward's float32 positions (cufkb_block_forward_xyz32)
and takes the gradients from them (cufkb_block_backward_from_xyz32): against the float64 oracle on
the 16-bit-rounded inputs, against the recompute backward, through the raw ops, the C ABI and
autograd, including the chains it hands to the recompute form."""

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
LOWP = (torch.float16, torch.bfloat16)
# gradient relative L2 against the oracle, as for the recompute backward of the 16-bit types
GTOL = {torch.float16: 2.0**-8, torch.bfloat16: 2.0**-5}


def _cuda(inp, dtype, anchors):
    L, A, D, G = (inp[k].to("cuda", dtype) for k in ("lengths", "angles", "dihedrals", "grad"))
    anc = [inp[k].to("cuda", dtype) for k in ANCHOR_KEYS] if anchors else [None, None, None]
    return L, A, D, G, anc


def _oracle(inp, dtype, anchors):
    c = {k: v.to(dtype).double() for k, v in inp.items()}
    kw = {k: c[k] for k in ANCHOR_KEYS} if anchors else {}
    return nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"], **kw)


def _rel(a, b):
    return float((a.double().cpu() - b.double().cpu()).norm() / b.double().cpu().norm())


@pytest.mark.parametrize("dtype", LOWP)
@pytest.mark.parametrize(
    "batch,points,anchors",
    [(3, 4, False), (2, 5, True), (4, 6, False), (5, 97, True), (64, 768, False), (7, 1027, True), (4, 2051, True), (1500, 300, False)],
)
def test_xyz32_matches_oracle_and_recompute(dtype, batch, points, anchors):
    inp = nerf64.make_inputs(batch, points, seed=points + batch, anchors=anchors)
    L, A, D, G, anc = _cuda(inp, dtype, anchors)
    xyz, xyz32 = C.block_forward_xyz32(L, A, D, *anc)
    # the 16-bit output is the plain forward's, bit for bit; the float32 positions are its unrounded values
    assert torch.equal(xyz, C.block_forward(L, A, D, *anc))
    assert xyz32.dtype == torch.float32 and xyz32.shape == xyz.shape
    torch.testing.assert_close(xyz32.to(dtype), xyz, rtol=0, atol=0)
    ref = _oracle(inp, dtype, anchors)
    scale = float(ref[0].abs().max())
    assert float((xyz32.double().cpu() - ref[0]).abs().max()) <= 2e-6 * max(1.0, scale) * math.sqrt(points)
    got = C.block_backward_from_xyz32(L, A, D, *anc, xyz32, G)
    rec = C.block_backward(L, A, D, *anc, G)
    for name, a, r, want in zip(("lengths", "angles", "dihedrals"), got, rec, ref[1:]):
        assert a.dtype == dtype
        assert _rel(a, want) <= GTOL[dtype], name
        assert _rel(r, want) <= GTOL[dtype], name


@pytest.mark.parametrize("dtype", LOWP)
def test_degenerate_chains_fall_back(dtype):
    # chain 0: a bond angle of pi; chain 1: 2 degrees from pi; chain 2: a zero-length bond; chains 3
    # and 4 untouched.  The first three take the recompute form inside the kernel.
    inp = nerf64.make_inputs(5, 300, seed=11, dtype=F64, anchors=True)
    inp["angles"][0, 150] = math.pi
    inp["angles"][1, 40] = math.pi - math.radians(2.0)
    inp["lengths"][2, 77] = 0.0
    L, A, D, G, anc = _cuda(inp, dtype, True)
    xyz, xyz32 = C.block_forward_xyz32(L, A, D, *anc)
    got = C.block_backward_from_xyz32(L, A, D, *anc, xyz32, G)
    rec = C.block_backward(L, A, D, *anc, G)
    ref = _oracle(inp, dtype, True)
    for a, r, want in zip(got, rec, ref[1:]):
        for b in range(5):
            assert _rel(a[b], want[b]) <= GTOL[dtype], b
            assert _rel(r[b], want[b]) <= GTOL[dtype], b


@pytest.mark.parametrize("dtype", LOWP)
def test_non_orthonormal_frame_takes_general_form(dtype):
    inp = nerf64.make_inputs(6, 120, seed=9, dtype=F64, anchors=True)
    inp["angles"][:, 0] = 0.0
    L, A, D, G, anc = _cuda(inp, dtype, True)
    _, xyz32 = C.block_forward_xyz32(L, A, D, *anc)
    got = C.block_backward_from_xyz32(L, A, D, *anc, xyz32, G)
    rec = C.block_backward(L, A, D, *anc, G)
    # the same form as the recompute backward, over another split of the steps between threads
    for a, r in zip(got, rec):
        finite = torch.isfinite(r)
        assert torch.equal(torch.isfinite(a), finite)
        if bool(finite.any()):
            assert _rel(a[finite], r[finite]) <= GTOL[dtype]


@pytest.mark.parametrize("dtype", LOWP)
def test_autograd_uses_float32_positions(dtype):
    import cufk_b200 as cufk

    inp = nerf64.make_inputs(9, 400, seed=21, anchors=True)
    L, A, D, G, anc = _cuda(inp, dtype, True)
    leaves = [t.clone().requires_grad_(True) for t in (L, A, D)]
    xyz = cufk.reconstruct(*leaves, *anc)
    xyz.backward(G)
    _, xyz32 = C.block_forward_xyz32(L, A, D, *anc)
    want = C.block_backward_from_xyz32(L, A, D, *anc, xyz32, G)
    for leaf, w in zip(leaves, want):
        torch.testing.assert_close(leaf.grad, w, rtol=0, atol=0)
    # an in-place edit of the returned 16-bit xyz does not touch the saved float32 positions
    leaves2 = [t.clone().requires_grad_(True) for t in (L, A, D)]
    out = cufk.reconstruct(*leaves2, *anc)
    out.data.add_(1.0)
    out.backward(G)
    for leaf, w in zip(leaves2, want):
        torch.testing.assert_close(leaf.grad, w, rtol=0, atol=0)


def test_linearity_at_config_size():
    # config 4 size (B=8192, N=1026, float16): the backward is linear in grad_xyz up to 16-bit rounding
    inp = nerf64.make_inputs(8192, 1026, seed=4)
    L, A, D, G, _ = _cuda(inp, torch.float16, False)
    G2 = torch.randn(G.shape, generator=torch.Generator().manual_seed(1)).to("cuda", torch.float16)
    _, xyz32 = C.block_forward_xyz32(L, A, D)
    g1 = C.block_backward_from_xyz32(L, A, D, None, None, None, xyz32, G)
    g2 = C.block_backward_from_xyz32(L, A, D, None, None, None, xyz32, G2)
    g12 = C.block_backward_from_xyz32(L, A, D, None, None, None, xyz32, (G.float() + G2.float()).half())
    for a, b, c in zip(g1, g2, g12):
        assert _rel(c, a.double() + b.double()) <= 2.0**-9
    rec = C.block_backward(L, A, D, None, None, None, G)
    for a, b in zip(g1, rec):
        per_chain = ((a.double() - b.double()).norm(dim=1) / b.double().norm(dim=1)).max()
        assert float(per_chain) <= 2.0**-8


def test_c_abi_matches_raw_ops():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_backward_from_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    inp = nerf64.make_inputs(33, 500, seed=5)
    L, A, D, G, _ = _cuda(inp, torch.bfloat16, False)
    want_xyz, want_xyz32 = C.block_forward_xyz32(L, A, D)
    want = C.block_backward_from_xyz32(L, A, D, None, None, None, want_xyz32, G)
    xyz = torch.full_like(want_xyz, float("nan"))
    xyz32 = torch.full_like(want_xyz32, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    BF16 = 3
    st = lib.cufkb_block_forward_xyz32(BF16, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), xyz32.data_ptr(), 33, 500, stream)
    assert st == 0
    got = [torch.full_like(t, float("nan")) for t in (L, A, D)]
    st = lib.cufkb_block_backward_from_xyz32(BF16, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz32.data_ptr(), G.data_ptr(),
                                             *(t.data_ptr() for t in got), 33, 500, stream)
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(xyz, want_xyz) and torch.equal(xyz32, want_xyz32)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_raw_op_checks():
    inp = nerf64.make_inputs(8, 60, seed=2)
    L, A, D, G, _ = _cuda(inp, torch.float16, False)
    _, xyz32 = C.block_forward_xyz32(L, A, D)
    with pytest.raises(RuntimeError, match="xyz32 must be float32"):
        C.block_backward_from_xyz32(L, A, D, None, None, None, xyz32.half(), G)
    with pytest.raises(RuntimeError, match="xyz32 must have shape"):
        C.block_backward_from_xyz32(L, A, D, None, None, None, xyz32[:, :-1].contiguous(), G)
    with pytest.raises(RuntimeError, match="supports float16 and bfloat16"):
        C.block_forward_xyz32(L.float(), A.float(), D.float())


@pytest.mark.parametrize("dtype_code,dtype", [(2, torch.float16), (3, torch.bfloat16)])
@pytest.mark.parametrize("xyz_shift,xyz32_shift", [(0, 0), (1, 0), (0, 1), (3, 2)])
def test_c_abi_offset_rows_take_the_element_paths(dtype_code, dtype, xyz_shift, xyz32_shift):
    # xyz and xyz32 rows whose residues mod 16 do not pair up (buffers shifted by whole elements):
    # the 16-bit output row and the grad row then move element by element; results stay within
    # the 16-bit tolerances of the oracle
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_backward_from_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    B, N = 21, 301
    inp = nerf64.make_inputs(B, N, seed=8)
    L, A, D, G, _ = _cuda(inp, dtype, False)
    xyz_buf = torch.zeros(B * N * 3 + 8, device="cuda", dtype=dtype)
    xyz32_buf = torch.zeros(B * N * 3 + 8, device="cuda", dtype=torch.float32)
    xyz = xyz_buf[xyz_shift : xyz_shift + B * N * 3].view(B, N, 3)
    xyz32 = xyz32_buf[xyz32_shift : xyz32_shift + B * N * 3].view(B, N, 3)
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.cufkb_block_forward_xyz32(dtype_code, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), xyz32.data_ptr(), B, N, stream)
    assert st == 0
    got = [torch.full_like(t, float("nan")) for t in (L, A, D)]
    st = lib.cufkb_block_backward_from_xyz32(dtype_code, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz32.data_ptr(), G.data_ptr(),
                                             *(t.data_ptr() for t in got), B, N, stream)
    assert st == 0
    torch.cuda.synchronize()
    # the buffers around the rows are untouched
    assert not xyz_buf[:xyz_shift].any() and not xyz_buf[xyz_shift + B * N * 3 :].any()
    assert not xyz32_buf[:xyz32_shift].any() and not xyz32_buf[xyz32_shift + B * N * 3 :].any()
    assert torch.equal(xyz, xyz32.to(dtype))
    ref = _oracle(inp, dtype, False)
    assert float((xyz32.double().cpu() - ref[0]).abs().max()) <= 2e-6 * max(1.0, float(ref[0].abs().max())) * math.sqrt(N)
    for a, want in zip(got, ref[1:]):
        assert _rel(a, want) <= GTOL[dtype]
