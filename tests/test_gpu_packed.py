"""Packed (ragged) batches on the GPU: reconstruct_packed against the float64 oracle for chains of
different lengths (4 to 2051 points, all dtypes, with anchors), bit-identical to reconstruct when
every chain has the same length, the no-sync form with max_points, and chains outside
[4, max_points] left untouched through the C ABI."""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

import cufk_b200 as cufk
from cufk_b200 import _native
from oracle import nerf64

pytestmark = pytest.mark.gpu

DEV = "cuda"
F64 = torch.float64
KEYS = ("p0", "first_direction", "initial_normal")
LOWP = {torch.float16: (2.0**-10, 2.0**-8), torch.bfloat16: (2.0**-7, 2.0**-5)}


def ragged_inputs(counts, seed, anchors=False):
    """Padded rows of the longest chain (the oracle's input) and their packed forms."""
    maxn = max(counts)
    inp = nerf64.make_inputs(len(counts), maxn, seed=seed, anchors=anchors)
    for b, n in enumerate(counts):
        inp["grad"][b, n:] = 0.0  # padded atoms do not enter the loss
    packed = {
        "lengths": torch.cat([inp["lengths"][b, : n - 1] for b, n in enumerate(counts)]),
        "angles": torch.cat([inp["angles"][b, : n - 2] for b, n in enumerate(counts)]),
        "dihedrals": torch.cat([inp["dihedrals"][b, : n - 3] for b, n in enumerate(counts)]),
        "grad": torch.cat([inp["grad"][b, :n] for b, n in enumerate(counts)]),
    }
    offsets = torch.tensor([0] + torch.tensor(counts).cumsum(0).tolist(), dtype=torch.int64)
    return inp, packed, offsets


def run_packed(packed, offsets, dtype, anchors, max_points=None):
    L, A, D = (packed[k].to(DEV, dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    xyz = cufk.reconstruct_packed(L, A, D, offsets.to(DEV), *anchors, max_points=max_points)
    xyz.backward(packed["grad"].to(DEV, dtype))
    return xyz.detach().cpu(), L.grad.cpu(), A.grad.cpu(), D.grad.cpu()


@pytest.mark.parametrize("dtype", [torch.float32, F64, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("with_anchors", [False, True])
def test_ragged_batch_matches_float64(dtype, with_anchors):
    g = torch.Generator().manual_seed(31)
    counts = [4, 5, 7, 2051] + torch.randint(4, 700, (41,), generator=g).tolist()
    inp, packed, offsets = ragged_inputs(counts, seed=32, anchors=with_anchors)
    anchors = [inp[k].to(DEV, dtype) for k in KEYS] if with_anchors else []
    xyz, gl, ga, gd = run_packed(packed, offsets, dtype, anchors)
    cast = {k: v.to(dtype).to(F64) for k, v in inp.items()}
    kw = {k: cast[k] for k in KEYS} if with_anchors else {}
    rx, rgl, rga, rgd = nerf64.reconstruct64_with_grads(cast["lengths"], cast["angles"], cast["dihedrals"], cast["grad"], **kw)
    p = 0
    ref_g = [torch.cat([r[b, : n - k] for b, n in enumerate(counts)]) for r, k in ((rgl, 1), (rga, 2), (rgd, 3))]
    for b, n in enumerate(counts):
        err = float((xyz[p : p + n].double() - rx[b, :n]).abs().max())
        scale = float(rx[b, :n].abs().max())
        if dtype == torch.float32:
            assert err <= 2e-6 * max(1.0, scale) * math.sqrt(n), (b, n, err)
        elif dtype == F64:
            assert err <= 1e-10 * max(1.0, scale), (b, n, err)
        else:
            assert err <= LOWP[dtype][0] * max(scale, 0.5), (b, n, err, scale)
        p += n
    gtol = {torch.float32: 1e-4, F64: 1e-9}.get(dtype, LOWP.get(dtype, (0, 0))[1])
    for got, ref in zip((gl, ga, gd), ref_g):
        rel = float((got.double() - ref).norm() / ref.norm())
        assert rel <= gtol, (dtype, rel)
    assert xyz.shape == (sum(counts), 3)


@pytest.mark.parametrize("dtype", [torch.float32, F64, torch.float16, torch.bfloat16])
def test_equal_lengths_match_the_batched_entry_point_bit_for_bit(dtype):
    B, N = 96, 513
    inp, packed, offsets = ragged_inputs([N] * B, seed=33)
    got = run_packed(packed, offsets, dtype, [])
    L, A, D = (inp[k].to(DEV, dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    xyz = cufk.reconstruct(L, A, D)
    xyz.backward(inp["grad"].to(DEV, dtype))
    assert torch.equal(got[0], xyz.detach().cpu().reshape(-1, 3))
    for a, b in zip(got[1:], (L.grad, A.grad, D.grad)):
        assert torch.equal(a, b.cpu().reshape(-1))


def test_max_points_given_needs_no_readback():
    counts = [300, 17, 250, 4]
    _, packed, offsets = ragged_inputs(counts, seed=34)
    a = run_packed(packed, offsets, torch.float32, [])
    b = run_packed(packed, offsets, torch.float32, [], max_points=300)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_single_chain_and_empty_batch():
    _, packed, offsets = ragged_inputs([2051], seed=35)
    xyz, *_ = run_packed(packed, offsets, torch.float32, [])
    ref = cufk.reconstruct(packed["lengths"].to(DEV), packed["angles"].to(DEV), packed["dihedrals"].to(DEV))
    assert torch.equal(xyz, ref.cpu())
    empty = torch.zeros(0, device=DEV)
    out = cufk.reconstruct_packed(empty, empty, empty, torch.zeros(1, dtype=torch.int64, device=DEV))
    assert out.shape == (0, 3)


def test_chain_beyond_max_points_is_left_untouched_through_the_c_abi():
    counts = [12, 40, 9]
    _, packed, offsets = ragged_inputs(counts, seed=36)
    L, A, D = (packed[k].to(DEV) for k in ("lengths", "angles", "dihedrals"))
    off = offsets.to(DEV)
    xyz = torch.full((sum(counts), 3), float("nan"), device=DEV)
    lib = _native._LIB
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_packed.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.cufkb_block_forward_packed(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, off.data_ptr(), xyz.data_ptr(), 3, sum(counts), 16, stream)
    torch.cuda.synchronize()
    assert st == 0
    x = xyz.cpu()
    assert torch.isnan(x[12:52]).all()  # the 40-point chain exceeds max_points = 16
    assert torch.isfinite(x[:12]).all() and torch.isfinite(x[52:]).all()
    ref = cufk.reconstruct_packed(L, A, D, off).cpu()
    torch.testing.assert_close(x[:12], ref[:12], rtol=0, atol=1e-5)
    torch.testing.assert_close(x[52:], ref[52:], rtol=0, atol=1e-5)


def test_offsets_outside_the_packed_arrays_skip_only_those_chains():
    # Four 10-point chains.  Chain 1's start is made negative (so chain 0 gets a negative count) and
    # chain 3's end lies far past the packed total: chains 0, 1 and 3 are skipped, chain 2 is
    # reconstructed, and nothing is written outside the output (guard rows around it stay NaN).
    counts = [10, 10, 10, 10]
    total = sum(counts)
    _, packed, offsets = ragged_inputs(counts, seed=37)
    L, A, D, G = (packed[k].to(DEV) for k in ("lengths", "angles", "dihedrals", "grad"))
    bad = offsets.clone()
    bad[1] = -20
    bad[4] = 100
    off = bad.to(DEV)
    guard = 32
    base = torch.full((total + 2 * guard, 3), float("nan"), device=DEV)
    xyz = base[guard : guard + total]
    lib = _native._LIB
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.cufkb_block_forward_packed.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    lib.cufkb_block_backward_packed_from_xyz.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.cufkb_block_forward_packed(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, off.data_ptr(), xyz.data_ptr(), 4, total, 2051, stream)
    assert st == 0
    gbase = [torch.full((n + 2 * guard,), float("nan"), device=DEV) for n in (L.numel(), A.numel(), D.numel())]
    gl, ga, gd = (g[guard:-guard] for g in gbase)
    st = lib.cufkb_block_backward_packed_from_xyz(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, off.data_ptr(), xyz.data_ptr(),
                                                  G.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(), 4, total, 2051, stream)
    assert st == 0
    torch.cuda.synchronize()
    b = base.cpu()
    assert torch.isnan(b[:guard]).all() and torch.isnan(b[guard + total :]).all()
    x = xyz.cpu()
    assert torch.isnan(x[:20]).all() and torch.isnan(x[30:]).all()
    ref = cufk.reconstruct_packed(L, A, D, offsets.to(DEV)).cpu()
    torch.testing.assert_close(x[20:30], ref[20:30], rtol=0, atol=1e-5)
    # chain 2's gradients (lengths from 20 - 2, angles from 20 - 4, dihedrals from 20 - 6), the rest NaN
    for g, start, n in ((gbase[0], 18, 9), (gbase[1], 16, 8), (gbase[2], 14, 7)):
        h = g.cpu()
        assert torch.isfinite(h[guard + start : guard + start + n]).all()
        assert torch.isnan(h[: guard + start]).all() and torch.isnan(h[guard + start + n :]).all()
