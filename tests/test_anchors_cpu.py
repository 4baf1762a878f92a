"""Anchor gradients (cufk_b200/anchors.py) without a GPU: the first frame restated for autograd
matches the oracle's (block.cu:113-148), and the anchor gradients computed from a chain's xyz and
incoming gradient match float64 autograd through the whole oracle forward, for general anchors,
the default anchors and the stable-perpendicular branch (normal parallel to the first direction)."""

from __future__ import annotations

import pytest
import torch

from cufk_b200 import anchors
from oracle import nerf64

F64 = torch.float64


def _anchor_set(kind, g):
    if kind == "random":
        q, _ = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=F64))
        return torch.randn(3, generator=g, dtype=F64), 2.5 * q[:, 0], 0.7 * q[:, 1] + 0.3 * q[:, 0]
    if kind == "default":
        return torch.zeros(3, dtype=F64), torch.tensor([1.0, 0, 0], dtype=F64), torch.tensor([0, 0, 1.0], dtype=F64)
    # initial normal parallel to the first direction: the stable perpendicular branch
    d = torch.tensor([0.95, 0.2, -0.1], dtype=F64)
    return torch.tensor([1.0, -2.0, 0.5], dtype=F64), d, 3.0 * d


@pytest.mark.parametrize("kind", ["random", "default", "parallel"])
def test_first_frame_matches_oracle(kind):
    g = torch.Generator().manual_seed(1)
    p0, fd, nn = _anchor_set(kind, g)
    inp = nerf64.make_inputs(5, 20, seed=2, dtype=F64)
    l0, l1, a0 = inp["lengths"][:, 0], inp["lengths"][:, 1], inp["angles"][:, 0]
    p1, p2, F = anchors.first_frame(l0, l1, a0, p0, fd, nn)
    ref = nerf64.first_frame64(l0, l1, a0, p0, fd, nn)
    torch.testing.assert_close(p1, ref["p1"], rtol=0, atol=1e-14)
    torch.testing.assert_close(p2, ref["p2"], rtol=0, atol=1e-14)
    torch.testing.assert_close(F, ref["frame"], rtol=0, atol=1e-14)


@pytest.mark.parametrize("kind", ["random", "default", "parallel"])
def test_anchor_gradients_match_float64_autograd(kind):
    g = torch.Generator().manual_seed(3)
    p0, fd, nn = _anchor_set(kind, g)
    inp = nerf64.make_inputs(7, 64, seed=4, dtype=F64)
    xyz, gp, gf, gn = nerf64.reconstruct64_anchor_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], p0, fd, nn)
    got = anchors.anchor_gradients(inp["lengths"], inp["angles"], (p0, fd, nn), xyz, inp["grad"], (True, True, True))
    for a, b in zip(got, (gp, gf, gn)):
        torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-10)


def test_only_requested_anchor_gradients_are_returned():
    g = torch.Generator().manual_seed(5)
    p0, fd, nn = _anchor_set("random", g)
    inp = nerf64.make_inputs(3, 30, seed=6, dtype=F64)
    xyz, gp, _, gn = nerf64.reconstruct64_anchor_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"], p0, fd, nn)
    got = anchors.anchor_gradients(inp["lengths"], inp["angles"], (p0, None, nn), xyz, inp["grad"], (True, False, True))
    assert got[1] is None
    torch.testing.assert_close(got[0], gp, rtol=1e-10, atol=1e-10)
    # first_direction None means the default (1, 0, 0); the oracle above used fd, so only p0's
    # gradient (which does not depend on the direction) is comparable across the two
    assert got[2].shape == (3,)
