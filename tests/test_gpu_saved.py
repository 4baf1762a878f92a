"""The saved-state backward (forward writes per-segment frames; backward reads them and the forward's
xyz) against the recompute backward and the float64 oracle, through the raw ops and the C ABI."""

from __future__ import annotations

import ctypes

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
    xyz, state = C.block_forward_save(L, A, D, *anc)
    plain = C.block_forward(L, A, D, *anc)
    saved = C.block_backward_saved(L, A, D, *anc, xyz, state, G)
    recomputed = C.block_backward(L, A, D, *anc, G)
    return xyz, plain, state, saved, recomputed


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("batch,points,anchors", [(3, 4, False), (5, 97, True), (64, 768, False), (7, 1027, True), (4, 2051, True), (1500, 300, False)])
def test_saved_matches_recompute_and_oracle(dtype, batch, points, anchors):
    inp = nerf64.make_inputs(batch, points, seed=points + batch, dtype=dtype, anchors=anchors)
    xyz, plain, state, saved, recomputed = _run_both(inp, dtype, anchors)
    torch.testing.assert_close(xyz, plain, rtol=0, atol=0)  # writing the state changes nothing else
    rtol = 1e-4 if dtype == torch.float32 else 1e-10
    for a, b in zip(saved, recomputed):
        assert float((a.double() - b.double()).norm() / b.double().norm()) <= rtol
    c = {k: v.double() for k, v in inp.items()}
    ref = nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"], **({k: c[k] for k in ANCHOR_KEYS} if anchors else {}))
    for got, want in zip(saved, ref[1:]):
        assert float((got.double().cpu() - want).norm() / want.norm()) <= rtol


def test_state_size():
    size = ctypes.c_size_t()
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    assert lib.cufkb_block_state_bytes(0, 4096, 768, ctypes.byref(size)) == 0
    assert size.value > 0 and size.value % (12 * 4) == 0
    assert lib.cufkb_block_state_bytes(3, 4096, 768, ctypes.byref(size)) == 0 and size.value == 0  # bf16 recomputes
    inp = nerf64.make_inputs(16, 50, seed=1)
    _, state = C.block_forward_save(*(inp[k].cuda() for k in ("lengths", "angles", "dihedrals")))
    assert lib.cufkb_block_state_bytes(0, 16, 50, ctypes.byref(size)) == 0 and state.numel() == size.value


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_16bit_saved_path_recomputes(dtype):
    inp = nerf64.make_inputs(8, 200, seed=3)
    xyz, plain, state, saved, recomputed = _run_both(inp, dtype, False)
    assert state.numel() == 0
    for a, b in zip(saved, recomputed):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


def test_degenerate_frame_falls_back_to_recompute():
    inp = nerf64.make_inputs(6, 120, seed=9, dtype=F64, anchors=True)
    inp["angles"][:, 0] = 0.0  # collinear first angle: the base frame is not orthonormal
    xyz, plain, state, saved, recomputed = _run_both(inp, F64, True)
    for a, b in zip(saved, recomputed):
        torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-12)


def test_state_mismatch_is_rejected():
    inp = nerf64.make_inputs(8, 60, seed=2)
    L, A, D, G = (inp[k].cuda() for k in ("lengths", "angles", "dihedrals", "grad"))
    xyz, state = C.block_forward_save(L, A, D)
    with pytest.raises(RuntimeError, match="state does not match"):
        C.block_backward_saved(L, A, D, None, None, None, xyz, state[:-48], G)


def test_autograd_uses_saved_state_and_detects_inplace_edits():
    import cufk_b200 as cufk

    inp = nerf64.make_inputs(4, 40, seed=4)
    L = inp["lengths"].cuda().requires_grad_(True)
    xyz = cufk.reconstruct(L, inp["angles"].cuda(), inp["dihedrals"].cuda())
    xyz.add_(1.0)  # the saved output was modified in place
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        xyz.sum().backward()
