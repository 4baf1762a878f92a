"""The C ABI called directly (ctypes, raw device pointers, an explicit stream) on the GPU gives the
same results as the PyTorch wrapper, which is built on it."""

from __future__ import annotations

import ctypes

import pytest
import torch

from cufk_b200 import _native
from oracle import nerf64

pytestmark = pytest.mark.gpu

vp, i64 = ctypes.c_void_p, ctypes.c_int64


class TorsionConstants(ctypes.Structure):
    _fields_ = [("bond_lengths", ctypes.c_double * 3), ("bond_angle_sin", ctypes.c_double * 3), ("bond_angle_cos", ctypes.c_double * 3)]


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    lib.cufkb_block_forward.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_backward.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_torsion_forward.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, i64, i64, vp]
    lib.cufkb_torsion_backward.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, vp, i64, i64, i64, vp]
    return lib


def test_block_forward_backward_through_cabi(lib):
    B, N = 96, 640
    inp = nerf64.make_inputs(B, N, seed=1, anchors=True)
    L, A, D, G, p0, fd, nn = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad", "p0", "first_direction", "initial_normal"))
    stream = torch.cuda.Stream()
    xyz = torch.empty(B, N, 3, device="cuda")
    gl, ga, gd = torch.empty_like(L), torch.empty_like(A), torch.empty_like(D)
    torch.cuda.synchronize()
    assert lib.cufkb_block_forward(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), p0.data_ptr(), fd.data_ptr(), nn.data_ptr(), xyz.data_ptr(), B, N, stream.cuda_stream) == 0
    assert lib.cufkb_block_backward(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), p0.data_ptr(), fd.data_ptr(), nn.data_ptr(), G.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(), B, N, stream.cuda_stream) == 0
    stream.synchronize()
    C = _native._C
    torch.testing.assert_close(xyz, C.block_forward(L, A, D, p0, fd, nn), rtol=0, atol=0)
    for a, b in zip((gl, ga, gd), C.block_backward(L, A, D, p0, fd, nn, G)):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_torsion_through_cabi(lib):
    import math

    B, N = 40, 300
    inp = nerf64.make_torsion_inputs(B, N, seed=2)
    raw, G = inp["raw"].cuda(), inp["grad"].cuda()
    consts = TorsionConstants((ctypes.c_double * 3)(*nerf64.BACKBONE_LENGTHS), (ctypes.c_double * 3)(*[math.sin(a) for a in nerf64.BACKBONE_ANGLES]), (ctypes.c_double * 3)(*[math.cos(a) for a in nerf64.BACKBONE_ANGLES]))
    xyz = torch.empty(B, N, 3, device="cuda")
    graw = torch.empty_like(raw)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.cufkb_torsion_forward(0, raw.data_ptr(), raw.stride(0), ctypes.byref(consts), xyz.data_ptr(), B, N, s) == 0
    assert lib.cufkb_torsion_backward(0, raw.data_ptr(), raw.stride(0), ctypes.byref(consts), G.data_ptr(), graw.data_ptr(), graw.stride(0), B, N, s) == 0
    import cufk_b200 as cufk

    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)
    torch.testing.assert_close(xyz, _native._C.torsion_forward(raw, f.constants), rtol=0, atol=0)
    torch.testing.assert_close(graw, _native._C.torsion_backward(raw, f.constants, G), rtol=0, atol=0)


def test_unaligned_row_starts_through_cabi(lib):
    # rows start at every residue mod 16 (odd N): the bulk-store head/tail handling is exercised
    for N in (5, 9, 37, 101):
        inp = nerf64.make_inputs(7, N, seed=N)
        L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
        base = torch.full((7 * N * 3 + 1,), float("nan"), device="cuda")
        xyz = base[1:].view(7, N, 3)  # 4-byte aligned, not 16
        assert lib.cufkb_block_forward(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), 7, N, torch.cuda.current_stream().cuda_stream) == 0
        # the threads' ranges follow the row's residue mod 16, so the scan's rounding may differ in
        # the last bits from the aligned call
        torch.testing.assert_close(xyz, _native._C.block_forward(L, A, D, None, None, None), rtol=0, atol=2e-6)
        assert torch.isnan(base[0])  # nothing written before the output
