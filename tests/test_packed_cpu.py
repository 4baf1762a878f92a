"""Host-side checks of reconstruct_packed (ragged batches) without a GPU: the validation of the
point offsets that the wrapper performs when it reads them back, and the shape checks of the
packed rows."""

from __future__ import annotations

import pytest
import torch

import cufk_b200 as cufk


def packed_rows(counts):
    b, total = len(counts), sum(counts)
    offsets = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int64)
    return torch.zeros(total - b), torch.zeros(total - 2 * b), torch.zeros(total - 3 * b), offsets


def test_offsets_must_start_at_zero():
    L, A, D, off = packed_rows([5, 6])
    with pytest.raises(RuntimeError, match="must start at 0"):
        cufk.reconstruct_packed(L, A, D, off + 1)


@pytest.mark.parametrize("counts", [[5, 3], [2052, 10]])
def test_chain_sizes_are_bounded(counts):
    L, A, D, off = packed_rows(counts)
    with pytest.raises(RuntimeError, match="needs 4 to 2051 points"):
        cufk.reconstruct_packed(L, A, D, off)


def test_total_must_match_the_rows():
    L, A, D, off = packed_rows([5, 6])
    with pytest.raises(RuntimeError, match="packed point count"):
        cufk.reconstruct_packed(L[:-1], A, D, off)


def test_host_tensors_rejected_with_reference_text():
    L, A, D, off = packed_rows([5, 6, 7])
    with pytest.raises(RuntimeError, match="lengths must be CUDA"):
        cufk.reconstruct_packed(L, A, D, off)
