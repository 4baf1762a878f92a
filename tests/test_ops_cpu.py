"""The torch.library operators (cufk_b200/ops.py) without a GPU: registration, schemas, the fake
(shape-inference) implementations under FakeTensorMode with CUDA fake tensors, and the anchor
gradient error.  The operators' real kernels are tested in test_gpu_ops.py."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import cufk_b200 as cufk
from cufk_b200 import ops

OPS = ("reconstruct", "reconstruct_xyz32", "reconstruct_backward", "torsion_reconstruct", "torsion_reconstruct_xyz32", "torsion_backward")


def test_operators_registered():
    for name in OPS:
        op = getattr(torch.ops.cufk_b200, name)
        assert "cufk_b200::" + name in str(op.default._schema)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16, torch.bfloat16])
def test_fake_reconstruct_shapes(dtype):
    with FakeTensorMode():
        L = torch.empty(5, 99, device="cuda", dtype=dtype)
        A = torch.empty(5, 98, device="cuda", dtype=dtype)
        D = torch.empty(5, 97, device="cuda", dtype=dtype)
        xyz = torch.ops.cufk_b200.reconstruct(L, A, D, None, None, None)
        assert xyz.shape == (5, 100, 3) and xyz.dtype == dtype and xyz.device.type == "cuda"
        g = torch.ops.cufk_b200.reconstruct_backward(L, A, D, None, None, None, xyz, torch.empty_like(xyz))
        assert [t.shape for t in g] == [L.shape, A.shape, D.shape]
        assert all(t.dtype == dtype for t in g)
        # the single-chain helper adds and removes the batch dimension
        single = ops.reconstruct(L[0], A[0], D[0])
        assert single.shape == (100, 3) and single.dtype == dtype
        if dtype in (torch.float16, torch.bfloat16):
            xyz16, xyz32 = torch.ops.cufk_b200.reconstruct_xyz32(L, A, D, None, None, None)
            assert xyz16.shape == xyz32.shape == (5, 100, 3) and xyz16.dtype == dtype and xyz32.dtype == torch.float32
            g = torch.ops.cufk_b200.reconstruct_backward(L, A, D, None, None, None, xyz32, torch.empty_like(xyz16))
            assert [t.shape for t in g] == [L.shape, A.shape, D.shape] and all(t.dtype == dtype for t in g)
        else:
            with pytest.raises(Exception, match="supports float16 and bfloat16"):
                torch.ops.cufk_b200.reconstruct_xyz32(L, A, D, None, None, None)


def test_fake_rejects_inconsistent_shapes():
    with FakeTensorMode():
        L = torch.empty(2, 10, device="cuda")
        A = torch.empty(2, 8, device="cuda")  # should be (2, 9)
        D = torch.empty(2, 8, device="cuda")
        with pytest.raises(Exception, match="bad angles shape"):
            torch.ops.cufk_b200.reconstruct(L, A, D, None, None, None)


def test_fake_torsion_shapes_and_strides():
    with FakeTensorMode():
        base = torch.empty(4, 2 * 61 + 6, device="cuda")
        raw = base[:, : 2 * 61]  # row stride 128, 122 columns
        consts = [0.1] * 9
        xyz = torch.ops.cufk_b200.torsion_reconstruct(raw, consts)
        assert xyz.shape == (4, 64, 3)
        g = torch.ops.cufk_b200.torsion_backward(raw, consts, xyz, torch.empty_like(xyz))
        assert g.shape == raw.shape and g.stride() == raw.stride()


def test_anchor_gradients_rejected_before_launch():
    L, A, D = torch.zeros(1, 5), torch.zeros(1, 4), torch.zeros(1, 3)
    p0 = torch.zeros(3, requires_grad=True)
    with pytest.raises(RuntimeError, match="p0 gradients are not supported"):
        ops.reconstruct(L, A, D, p0=p0)


def test_public_module_exposes_ops():
    assert cufk.ops is ops
    assert callable(ops.reconstruct) and callable(ops.torsion)
