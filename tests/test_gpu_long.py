"""Chains longer than BLOCK_SCAN_MAX_POINT_COUNT (reconstruct_long; the reference has none): the
segmented forward and backward against the float64 oracle, against the one-CTA kernels where
both apply, through the C ABI with a caller workspace, and their argument checks."""

from __future__ import annotations

import ctypes

import pytest
import torch

import cufk_b200 as cufk
from cufk_b200 import _native
from oracle import nerf64

pytestmark = pytest.mark.gpu

F64 = torch.float64
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")


def _grads(fn, inp, dtype, anchors):
    L, A, D = (inp[k].to("cuda", dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: inp[k].to("cuda", dtype) for k in ANCHOR_KEYS} if anchors else {}
    xyz = fn(L, A, D, **kw)
    xyz.backward(inp["grad"].to("cuda", dtype))
    return [t.detach().double().cpu() for t in (xyz, L.grad, A.grad, D.grad)]


def _oracle(inp, anchors):
    c = {k: v.double() for k, v in inp.items()}
    return nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"], **({k: c[k] for k in ANCHOR_KEYS} if anchors else {}))


def _check(got, want, xtol, gtol):
    assert float((got[0] - want[0]).abs().max()) <= xtol
    for a, b in zip(got[1:], want[1:]):
        assert float((a - b).norm() / b.norm()) <= gtol


@pytest.mark.parametrize("dtype", [torch.float32, F64])
@pytest.mark.parametrize("batch,points,anchors", [(3, 2052, False), (2, 2500, True), (2, 4099, False), (2, 6150, True), (1, 20000, False)])
def test_long_chains_match_oracle(dtype, batch, points, anchors):
    inp = nerf64.make_inputs(batch, points, seed=points, dtype=dtype, anchors=anchors)
    got = _grads(cufk.reconstruct_long, inp, dtype, anchors)
    want = _oracle(inp, anchors)
    # float32 error grows with the chain: 5e-4 nm is the stated bound at N = 2051
    xtol = (5e-4 * max(1.0, points / 2051.0)) if dtype == torch.float32 else 1e-9
    gtol = 1e-4 if dtype == torch.float32 else 1e-9
    _check(got, want, xtol, gtol)


@pytest.mark.parametrize("points", [4, 5, 300, 2051])
def test_short_chains_agree_with_one_cta_path(points):
    inp = nerf64.make_inputs(5, points, seed=points, anchors=True)
    a = _grads(cufk.reconstruct_long, inp, torch.float32, True)
    b = _grads(cufk.reconstruct, inp, torch.float32, True)
    # two float32 scans of the same chain with different thread layouts: each is within ~3e-5 nm of
    # float64 at N = 2051, so they agree to the sum
    _check(a, b, 6e-5, 1e-5)


def test_single_chain_and_empty_batch():
    inp = nerf64.make_inputs(1, 3000, seed=1)
    L, A, D = (inp[k][0].cuda() for k in ("lengths", "angles", "dihedrals"))
    assert cufk.reconstruct_long(L, A, D).shape == (3000, 3)
    empty = cufk.reconstruct_long(torch.empty(0, 2999, device="cuda"), torch.empty(0, 2998, device="cuda"), torch.empty(0, 2997, device="cuda"))
    assert empty.shape == (0, 3000, 3)


def test_16bit_is_rejected():
    inp = nerf64.make_inputs(1, 3000, seed=1)
    L, A, D = (inp[k].cuda().half() for k in ("lengths", "angles", "dihedrals"))
    with pytest.raises(RuntimeError, match="take float32 and float64 only"):
        cufk.reconstruct_long(L, A, D)


def test_degenerate_first_frame_gives_nan_gradients():
    inp = nerf64.make_inputs(2, 2600, seed=4, dtype=F64)
    inp["angles"][0, 0] = 0.0  # collinear first angle: the base frame is not orthonormal
    got = _grads(cufk.reconstruct_long, inp, F64, False)
    assert torch.isnan(got[1][0]).all() and torch.isfinite(got[1][1]).all()
    want = _oracle({k: v[1:] for k, v in inp.items()}, False)
    _check([t[1:] for t in got], want, 1e-9, 1e-9)


def test_c_abi_workspace():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_long_workspace_bytes.argtypes = [ctypes.c_int, i64, i64, ctypes.POINTER(ctypes.c_size_t)]
    lib.cufkb_block_forward_long.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp, ctypes.c_size_t, vp]
    B, N = 3, 5000
    size = ctypes.c_size_t()
    assert lib.cufkb_block_long_workspace_bytes(0, B, N, ctypes.byref(size)) == 0
    assert size.value == B * 3 * 18 * 4  # 3 segments of at most 2048 steps, 12 + 6 words each
    inp = nerf64.make_inputs(B, N, seed=2)
    L, A, D = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals"))
    ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    xyz = torch.empty(B, N, 3, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.cufkb_block_forward_long(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), B, N, ws.data_ptr(), 16, s) == 10
    assert lib.cufkb_block_forward_long(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), B, N, ws.data_ptr(), size.value, s) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(xyz, cufk.reconstruct_long(L, A, D), rtol=0, atol=0)
