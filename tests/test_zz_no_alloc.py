"""cufkb_block_forward_long_static: the long-chain forward that allocates nothing (its scratch is
a static device array inside libcufkb.so).  Collected last, so that it also runs after every other
test has used the library; it must pass alone as well.  Two calls on different inputs must give
exactly what cufkb_block_forward_long gives with a caller workspace."""

from __future__ import annotations

import ctypes

import pytest
import torch

from cufk_b200 import _native
from oracle import nerf64

pytestmark = pytest.mark.gpu

vp, i64 = ctypes.c_void_p, ctypes.c_int64
SCRATCH_CAPACITY = 12


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    lib.cufkb_block_forward_long_static.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
    lib.cufkb_block_forward_long.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp, ctypes.c_size_t, vp]
    lib.cufkb_block_long_workspace_bytes.argtypes = [ctypes.c_int, i64, i64, ctypes.POINTER(ctypes.c_size_t)]
    return lib


def _run(lib, dtype_code, inp, dtype, anchors, static):
    B, N = inp["lengths"].shape[0], inp["lengths"].shape[1] + 1
    L, A, D = (inp[k].to("cuda", dtype) for k in ("lengths", "angles", "dihedrals"))
    anc = [inp[k].to("cuda", dtype) for k in ("p0", "first_direction", "initial_normal")] if anchors else [None, None, None]
    ptrs = [t.data_ptr() if t is not None else None for t in anc]
    xyz = torch.full((B, N, 3), float("nan"), device="cuda", dtype=dtype)
    s = torch.cuda.current_stream().cuda_stream
    if static:
        st = lib.cufkb_block_forward_long_static(dtype_code, L.data_ptr(), A.data_ptr(), D.data_ptr(), *ptrs, xyz.data_ptr(), B, N, s)
    else:
        size = ctypes.c_size_t()
        assert lib.cufkb_block_long_workspace_bytes(dtype_code, B, N, ctypes.byref(size)) == 0
        ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
        st = lib.cufkb_block_forward_long(dtype_code, L.data_ptr(), A.data_ptr(), D.data_ptr(), *ptrs, xyz.data_ptr(), B, N, ws.data_ptr(), size.value, s)
    assert st == 0
    torch.cuda.synchronize()
    return xyz


@pytest.mark.parametrize("dtype_code,dtype", [(0, torch.float32), (1, torch.float64)])
def test_two_calls_match_the_workspace_entry_point(lib, dtype_code, dtype):
    first = nerf64.make_inputs(7, 5000, seed=1, dtype=dtype, anchors=True)
    second = nerf64.make_inputs(3, 2600, seed=2, dtype=dtype)
    for inp, anchors in ((first, True), (second, False)):
        got = _run(lib, dtype_code, inp, dtype, anchors, static=True)
        want = _run(lib, dtype_code, inp, dtype, anchors, static=False)
        assert torch.equal(got, want)


def test_short_chains_and_capacity(lib):
    inp = nerf64.make_inputs(5, 300, seed=3)
    assert torch.equal(_run(lib, 0, inp, torch.float32, False, static=True), _run(lib, 0, inp, torch.float32, False, static=False))
    # 100 chains of 1e6 points need 100 x 489 segments x 48 B > 2 MiB: rejected before any launch
    assert lib.cufkb_block_forward_long_static(0, 16, 32, 48, None, None, None, 64, 100, 1_000_000, None) == SCRATCH_CAPACITY


def test_capacity_boundary_float64(lib):
    # one segment per chain, 96 B of scratch per chain in float64: 21845 chains fill 2,097,120 of the
    # 2,097,152 bytes (accepted, twice in a row); one chain more does not fit
    inp = nerf64.make_inputs(21845, 40, seed=4, dtype=torch.float64)
    for _ in range(2):
        got = _run(lib, 1, inp, torch.float64, False, static=True)
        assert torch.equal(got, _run(lib, 1, inp, torch.float64, False, static=False))
    assert lib.cufkb_block_forward_long_static(1, 16, 32, 48, None, None, None, 64, 21846, 40, None) == SCRATCH_CAPACITY


def test_call_allocates_no_device_memory(lib):
    # after a warm-up call (module loading is done), a call changes neither torch's allocator
    # statistics nor the device's free memory
    inp = nerf64.make_inputs(16, 3000, seed=5)
    L, A, D = (inp[k].to("cuda") for k in ("lengths", "angles", "dihedrals"))
    xyz = torch.empty(16, 3000, 3, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def call():
        assert lib.cufkb_block_forward_long_static(0, L.data_ptr(), A.data_ptr(), D.data_ptr(), None, None, None, xyz.data_ptr(), 16, 3000, s) == 0
        torch.cuda.synchronize()

    call()
    stats = torch.cuda.memory_stats()
    free_before, _ = torch.cuda.mem_get_info()
    call()
    free_after, _ = torch.cuda.mem_get_info()
    after = torch.cuda.memory_stats()
    assert free_after == free_before
    for key in ("allocated_bytes.all.current", "reserved_bytes.all.current", "allocation.all.allocated"):
        assert after.get(key, 0) == stats.get(key, 0), key
