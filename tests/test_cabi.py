"""CPU checks of the C ABI (include/cufkb.h, cufk_b200/libcufkb.so): loading, exported symbols and
argument validation.  Validation returns before any CUDA call, so no GPU is needed; the fake
pointers passed here are never dereferenced."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "cufkb.h"
LIB = ROOT / "cufk_b200" / "libcufkb.so"

SUCCESS, INVALID_DTYPE, NULL_POINTER, POINT_COUNT, TOO_MANY_STEPS, SHAPE_LIMITS, BAD_STRIDE, MISALIGNED, INVALID_VALUE, CUDA = range(10)
F32, F64, F16, BF16 = range(4)


class TorsionConstants(ctypes.Structure):
    _fields_ = [("bond_lengths", ctypes.c_double * 3), ("bond_angle_sin", ctypes.c_double * 3), ("bond_angle_cos", ctypes.c_double * 3)]


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:CUFKB_API\s+)?(?:const\s+)?\w+\*?\s+\*?(cufkb_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(LIB))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_backward.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_torsion_forward.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, i64, i64, vp]
    lib.cufkb_torsion_backward.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, vp, i64, i64, i64, vp]
    lib.cufkb_status_string.restype = ctypes.c_char_p
    return lib


def test_header_declares_the_boundary():
    names = declared_functions()
    assert {"cufkb_block_forward", "cufkb_block_backward", "cufkb_torsion_forward", "cufkb_torsion_backward"} <= set(names)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_max_point_count(lib):
    assert lib.cufkb_max_point_count() == 2051


def fwd(lib, dtype=F32, L=16, A=32, D=48, xyz=64, batch=2, points=10, anchors=(None, None, None)):
    return lib.cufkb_block_forward(dtype, L, A, D, *anchors, xyz, batch, points, None)


def test_block_forward_validation(lib):
    assert fwd(lib, dtype=9) == INVALID_DTYPE
    assert fwd(lib, points=3) == POINT_COUNT
    assert fwd(lib, points=2052) == TOO_MANY_STEPS
    assert fwd(lib, batch=-1) == SHAPE_LIMITS
    assert fwd(lib, batch=2**31) == SHAPE_LIMITS
    assert fwd(lib, points=2**31 + 5) == SHAPE_LIMITS
    assert fwd(lib, batch=0, L=None, A=None, D=None, xyz=None) == SUCCESS
    assert fwd(lib, L=None) == NULL_POINTER
    assert fwd(lib, xyz=None) == NULL_POINTER
    assert fwd(lib, L=18) == MISALIGNED
    assert fwd(lib, dtype=F64, L=20) == MISALIGNED
    assert fwd(lib, anchors=(17, None, None)) == MISALIGNED


def test_block_backward_validation(lib):
    def bwd(**kw):
        args = dict(dtype=F32, L=16, A=32, D=48, g=64, gl=80, ga=96, gd=112, batch=2, points=10)
        args.update(kw)
        return lib.cufkb_block_backward(
            args["dtype"], args["L"], args["A"], args["D"], None, None, None, args["g"], args["gl"], args["ga"], args["gd"],
            args["batch"], args["points"], None,
        )

    assert bwd(points=3) == POINT_COUNT
    assert bwd(points=2051 + 1) == TOO_MANY_STEPS
    assert bwd(batch=0, L=None, g=None) == SUCCESS
    assert bwd(g=None) == NULL_POINTER
    assert bwd(gd=None) == NULL_POINTER
    assert bwd(gl=82) == MISALIGNED


def test_from_xyz_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_backward_from_xyz.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    args = [16, 32, 48, None, None, None, 64, 80, 96, 112, 128]
    assert lib.cufkb_block_backward_from_xyz(F32, *args[:6], None, *args[7:], 2, 10, None) == NULL_POINTER
    assert lib.cufkb_block_backward_from_xyz(BF16, *args[:6], None, *args[7:], 2, 10, None) == NULL_POINTER
    assert lib.cufkb_block_backward_from_xyz(F32, *args[:6], 66, *args[7:], 2, 10, None) == MISALIGNED
    assert lib.cufkb_block_backward_from_xyz(F64, *args, 2, 2052, None) == TOO_MANY_STEPS
    assert lib.cufkb_block_backward_from_xyz(F32, *args, 2, 3, None) == POINT_COUNT
    assert lib.cufkb_block_backward_from_xyz(F32, *args, 0, 10, None) == SUCCESS
    assert lib.cufkb_block_backward_from_xyz(7, *args, 2, 10, None) == INVALID_DTYPE


def test_torsion_validation(lib):
    c = TorsionConstants()
    assert lib.cufkb_torsion_forward(F32, 16, -1, ctypes.byref(c), 64, 2, 10, None) == BAD_STRIDE
    assert lib.cufkb_torsion_forward(F32, 16, 14, None, 64, 2, 10, None) == INVALID_VALUE
    assert lib.cufkb_torsion_forward(F32, 16, 14, ctypes.byref(c), 64, 2, 3, None) == POINT_COUNT
    assert lib.cufkb_torsion_backward(F32, 16, 14, ctypes.byref(c), 64, 128, 13, 2, 10, None) == BAD_STRIDE
    assert lib.cufkb_torsion_backward(F32, 16, 14, ctypes.byref(c), 64, None, 14, 2, 10, None) == NULL_POINTER
    assert lib.cufkb_torsion_backward(F32, 16, 14, ctypes.byref(c), 64, 128, 14, 0, 10, None) == SUCCESS


def test_torsion_from_xyz_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_torsion_backward_from_xyz.argtypes = [ctypes.c_int, vp, i64, vp, vp, vp, vp, i64, i64, i64, vp]
    c = TorsionConstants()
    assert lib.cufkb_torsion_backward_from_xyz(F32, 16, 14, ctypes.byref(c), None, 64, 128, 14, 2, 10, None) == NULL_POINTER
    assert lib.cufkb_torsion_backward_from_xyz(BF16, 16, 14, ctypes.byref(c), None, 64, 128, 14, 2, 10, None) == NULL_POINTER
    assert lib.cufkb_torsion_backward_from_xyz(F32, 16, 14, None, 32, 64, 128, 14, 2, 10, None) == INVALID_VALUE
    assert lib.cufkb_torsion_backward_from_xyz(F32, 16, 14, ctypes.byref(c), 34, 64, 128, 14, 2, 10, None) == MISALIGNED
    assert lib.cufkb_torsion_backward_from_xyz(F32, 16, 14, ctypes.byref(c), 32, 64, 128, 13, 2, 10, None) == BAD_STRIDE
    assert lib.cufkb_torsion_backward_from_xyz(F32, 16, 14, ctypes.byref(c), 32, 64, 128, 14, 0, 10, None) == SUCCESS
    assert lib.cufkb_torsion_backward_from_xyz(F64, 16, 14, ctypes.byref(c), 32, 64, 128, 14, 2, 2052, None) == TOO_MANY_STEPS


def test_long_path_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_long_static.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_forward_long.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp, ctypes.c_size_t, vp]
    lib.cufkb_block_long_workspace_bytes.argtypes = [ctypes.c_int, i64, i64, ctypes.POINTER(ctypes.c_size_t)]
    size = ctypes.c_size_t()
    assert lib.cufkb_block_long_workspace_bytes(F32, 4, 10000, ctypes.byref(size)) == SUCCESS
    assert size.value == 4 * 5 * 18 * 4  # 9997 steps: 5 segments of at most 2048
    assert lib.cufkb_block_long_workspace_bytes(F16, 4, 10000, ctypes.byref(size)) == 11
    assert lib.cufkb_block_long_workspace_bytes(F32, 4, 3, ctypes.byref(size)) == POINT_COUNT
    assert lib.cufkb_block_forward_long(F32, 16, 32, 48, None, None, None, 64, 2, 5000, None, 0, None) == NULL_POINTER
    assert lib.cufkb_block_forward_long(F32, 16, 32, 48, None, None, None, 64, 2, 5000, 72, 10**6, None) == MISALIGNED
    assert lib.cufkb_block_forward_long(F32, 16, 32, 48, None, None, None, 64, 2, 5000, 80, 16, None) == 10
    assert lib.cufkb_block_forward_long_static(BF16, 16, 32, 48, None, None, None, 64, 2, 5000, None) == 11
    assert lib.cufkb_block_forward_long_static(F32, 16, 32, 48, None, None, None, 64, 100, 10**6, None) == 12
    assert lib.cufkb_block_forward_long_static(F32, 16, 32, 48, None, None, None, 64, 0, 5000, None) == SUCCESS
    assert lib.cufkb_status_string(12).startswith(b"batch x segments exceeds")


def test_status_strings(lib):
    assert lib.cufkb_status_string(SUCCESS) == b"success"
    assert lib.cufkb_status_string(POINT_COUNT) == b"point_count must be >= 4"
    assert b"2048 local transforms" in lib.cufkb_status_string(TOO_MANY_STEPS)
    assert lib.cufkb_status_string(12345) == b"unknown status"
    assert lib.cufkb_last_cuda_error() == 0


def test_packed_entry_points_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_packed.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    lib.cufkb_block_backward_packed_from_xyz.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]

    def fwd_packed(offsets=128, batch=2, max_points=10, dtype=F32, total=20):
        return lib.cufkb_block_forward_packed(dtype, 16, 32, 48, None, None, None, offsets, 64, batch, total, max_points, None)

    assert fwd_packed(offsets=None) == NULL_POINTER
    assert fwd_packed(offsets=132) == MISALIGNED  # int64 offsets need 8-byte alignment
    assert fwd_packed(max_points=3) == POINT_COUNT
    assert fwd_packed(max_points=2052) == TOO_MANY_STEPS
    assert fwd_packed(dtype=7) == INVALID_DTYPE
    assert fwd_packed(batch=0, offsets=None, total=0) == SUCCESS  # nothing to launch
    assert fwd_packed(total=7) == SHAPE_LIMITS  # fewer than 4 points per chain
    assert fwd_packed(total=-1) == SHAPE_LIMITS
    bwd = lib.cufkb_block_backward_packed_from_xyz
    assert bwd(F32, 16, 32, 48, None, None, None, None, 64, 80, 96, 112, 128, 2, 20, 10, None) == NULL_POINTER
    assert bwd(F32, 16, 32, 48, None, None, None, 136, 64, 80, 96, 112, 128, 2, 20, 2052, None) == TOO_MANY_STEPS
    assert bwd(F32, 16, 32, 48, None, None, None, 136, 64, 80, 96, 112, 128, 2, 7, 10, None) == SHAPE_LIMITS
    assert bwd(F16, 16, 32, 48, None, None, None, 136, 64, 80, 96, 112, 128, 0, 0, 10, None) == SUCCESS


def test_fused_mse_entry_point_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_mse.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    mse = lib.cufkb_block_mse
    assert mse(F16, 16, 32, 48, None, None, None, 64, 80, None, None, None, 2, 10, None) == 11  # float32/float64 only
    assert mse(F32, 16, 32, 48, None, None, None, 64, 80, 96, None, None, 2, 10, None) == NULL_POINTER  # all three grads or none
    assert mse(F32, 16, 32, 48, None, None, None, None, 80, None, None, None, 2, 10, None) == NULL_POINTER  # target required
    assert mse(F32, 16, 32, 48, None, None, None, 64, 80, None, None, None, 2, 3, None) == POINT_COUNT
    assert mse(F64, 16, 32, 48, None, None, None, 64, 80, None, None, None, 0, 10, None) == SUCCESS


def test_xyz32_entry_points_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_backward_from_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    fwd32 = lib.cufkb_block_forward_xyz32
    bwd32 = lib.cufkb_block_backward_from_xyz32
    assert fwd32(F32, 16, 32, 48, None, None, None, 64, 128, 2, 10, None) == 11  # float16/bfloat16 only
    assert fwd32(F64, 16, 32, 48, None, None, None, 64, 128, 2, 10, None) == 11
    assert fwd32(F16, 16, 32, 48, None, None, None, 64, None, 2, 10, None) == NULL_POINTER
    assert fwd32(BF16, 16, 32, 48, None, None, None, 64, 130, 2, 10, None) == MISALIGNED  # float32 positions: 4-byte alignment
    assert fwd32(F16, 16, 32, 48, None, None, None, 64, 128, 2, 3, None) == POINT_COUNT
    assert fwd32(F16, 16, 32, 48, None, None, None, 64, 128, 2, 2052, None) == TOO_MANY_STEPS
    assert fwd32(7, 16, 32, 48, None, None, None, 64, 128, 2, 10, None) == INVALID_DTYPE
    assert fwd32(BF16, None, None, None, None, None, None, None, None, 0, 10, None) == SUCCESS  # nothing to launch
    args = [16, 32, 48, None, None, None, 128, 64, 80, 96, 112]
    assert bwd32(F32, *args, 2, 10, None) == 11
    assert bwd32(F16, *args[:6], None, *args[7:], 2, 10, None) == NULL_POINTER
    assert bwd32(F16, *args[:6], 130, *args[7:], 2, 10, None) == MISALIGNED
    assert bwd32(BF16, *args[:7], 65, *args[8:], 2, 10, None) == MISALIGNED  # grad_xyz: 2-byte alignment
    assert bwd32(BF16, *args, 2, 2052, None) == TOO_MANY_STEPS
    assert bwd32(F16, *args, 0, 10, None) == SUCCESS
    assert b"float16 and bfloat16 only" in lib.cufkb_status_string(11)
    lib.cufkb_block_forward_packed_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    lib.cufkb_block_backward_packed_from_xyz32.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    fwdp = lib.cufkb_block_forward_packed_xyz32
    bwdp = lib.cufkb_block_backward_packed_from_xyz32
    assert fwdp(F32, 16, 32, 48, None, None, None, 136, 64, 128, 2, 20, 10, None) == 11
    assert fwdp(F16, 16, 32, 48, None, None, None, None, 64, 128, 2, 20, 10, None) == NULL_POINTER  # offsets required
    assert fwdp(F16, 16, 32, 48, None, None, None, 132, 64, 128, 2, 20, 10, None) == MISALIGNED
    assert fwdp(BF16, 16, 32, 48, None, None, None, 136, 64, 128, 2, 7, 10, None) == SHAPE_LIMITS
    assert fwdp(BF16, 16, 32, 48, None, None, None, 136, 64, 128, 2, 20, 2052, None) == TOO_MANY_STEPS
    assert fwdp(BF16, 16, 32, 48, None, None, None, None, 64, 128, 0, 0, 10, None) == SUCCESS
    assert bwdp(F64, 16, 32, 48, None, None, None, 136, 128, 64, 80, 96, 112, 2, 20, 10, None) == 11
    assert bwdp(F16, 16, 32, 48, None, None, None, 136, None, 64, 80, 96, 112, 2, 20, 10, None) == NULL_POINTER
    assert bwdp(F16, 16, 32, 48, None, None, None, 136, 130, 64, 80, 96, 112, 2, 20, 10, None) == MISALIGNED
    assert bwdp(F16, 16, 32, 48, None, None, None, 136, 128, 64, 80, 96, 112, 2, -1, 10, None) == SHAPE_LIMITS
    assert bwdp(F16, 16, 32, 48, None, None, None, 136, 128, 64, 80, 96, 112, 0, 0, 10, None) == SUCCESS


def test_torsion_xyz32_entry_points_validation(lib):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_torsion_forward_xyz32.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, vp, i64, i64, vp]
    lib.cufkb_torsion_backward_from_xyz32.argtypes = [ctypes.c_int, vp, i64, ctypes.POINTER(TorsionConstants), vp, vp, vp, i64, i64, i64, vp]
    c = TorsionConstants()
    f = lib.cufkb_torsion_forward_xyz32
    b = lib.cufkb_torsion_backward_from_xyz32
    assert f(F32, 16, 14, ctypes.byref(c), 64, 128, 2, 10, None) == 11  # float16/bfloat16 only
    assert f(F16, 16, 14, ctypes.byref(c), 64, None, 2, 10, None) == NULL_POINTER
    assert f(F16, 16, 14, None, 64, 128, 2, 10, None) == INVALID_VALUE
    assert f(BF16, 16, -1, ctypes.byref(c), 64, 128, 2, 10, None) == BAD_STRIDE
    assert f(BF16, 16, 14, ctypes.byref(c), 64, 130, 2, 10, None) == MISALIGNED
    assert f(F16, 16, 14, ctypes.byref(c), 64, 128, 0, 10, None) == SUCCESS
    assert b(F64, 16, 14, ctypes.byref(c), 128, 64, 80, 14, 2, 10, None) == 11
    assert b(F16, 16, 14, ctypes.byref(c), None, 64, 80, 14, 2, 10, None) == NULL_POINTER
    assert b(F16, 16, 14, ctypes.byref(c), 128, 64, 80, 13, 2, 10, None) == BAD_STRIDE  # rows of 14 values would overlap
    assert b(BF16, 16, 14, ctypes.byref(c), 130, 64, 80, 14, 2, 10, None) == MISALIGNED
    assert b(BF16, 16, 14, ctypes.byref(c), 128, 64, 80, 14, 2, 2052, None) == TOO_MANY_STEPS
