"""CPU checks of the Python surface: names, caching, error text for host tensors, and that the
product never imports the oracle (the checker) or falls back to a CPU path."""

from __future__ import annotations

import ast
from pathlib import Path

import pytest
import torch

import cufk_b200 as cufk

PKG = Path(cufk.__file__).resolve().parent


def test_public_surface_matches_reference():
    # the reference's surface, plus reconstruct_long for chains the reference cannot reconstruct and
    # ops, the same path as torch.library operators
    assert set(cufk.__all__) == {"BLOCK_SCAN_MAX_POINT_COUNT", "__version__", "compile_torsion", "ops", "reconstruct", "reconstruct_long", "reconstruct_mse", "reconstruct_packed"}
    assert cufk.BLOCK_SCAN_MAX_POINT_COUNT == 2051
    assert cufk.__version__ == "0.1.0"


def test_host_tensors_are_rejected_with_reference_text():
    with pytest.raises(RuntimeError, match="lengths must be CUDA"):
        cufk.reconstruct(torch.ones(2, 9), torch.ones(2, 8), torch.ones(2, 7))
    with pytest.raises(RuntimeError, match="lengths must be CUDA"):
        cufk.reconstruct(torch.ones(9), torch.ones(8), torch.ones(7))
    with pytest.raises(RuntimeError, match="raw_pairs must be CUDA"):
        cufk.compile_torsion((1.0, 1.0, 1.0), (2.0, 2.0, 2.0))(torch.ones(2, 8))
    with pytest.raises(RuntimeError, match="lengths must be CUDA"):
        cufk.reconstruct_long(torch.ones(2, 9), torch.ones(2, 8), torch.ones(2, 7))


def test_compile_torsion_is_cached_per_constants():
    a = cufk.compile_torsion((0.1, 0.2, 0.3), (1.0, 2.0, 3.0))
    b = cufk.compile_torsion((0.1, 0.2, 0.3), (1.0, 2.0, 3.0))
    c = cufk.compile_torsion((0.1, 0.2, 0.3), (1.0, 2.0, 3.5))
    assert a is b and a is not c
    with pytest.raises(AssertionError, match="bond_angles must have 3 elements"):
        cufk.compile_torsion((0.1, 0.2, 0.3), (1.0, 2.0))


def test_product_never_imports_the_oracle():
    for path in PKG.rglob("*.py"):
        tree = ast.parse(path.read_text())
        for node in ast.walk(tree):
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            else:
                continue
            assert not any(n.split(".")[0] in ("oracle", "tests", "_work") for n in names), (path, names)


def test_native_extension_is_loaded():
    from cufk_b200 import _native

    assert _native.LIB_PATH.exists()
    assert hasattr(_native._C, "apply") and hasattr(_native._C, "torsion_apply")


def test_bench_and_oracle_generate_the_same_inputs():
    import bench
    from oracle import nerf64

    a = bench.make_inputs(5, 40, seed=3)
    b = nerf64.make_inputs(5, 40, seed=3)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_shards_cover_the_batch():
    import bench

    for world in (1, 2, 3, 4, 8):
        ranges = [bench.shard(4096, world, r) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == 4096
        assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
        sizes = [hi - lo for lo, hi in ranges]
        assert max(sizes) - min(sizes) <= 1


def test_rank_inputs_weak_and_strong():
    import bench

    make = lambda b, seed: bench.make_inputs(b, 20, seed=seed)  # noqa: E731
    # weak: every rank a whole batch of its own chains; the job is world x batch
    w0, total = bench.rank_inputs(make, 6, "weak", 2, 0)
    w1, _ = bench.rank_inputs(make, 6, "weak", 2, 1)
    assert total == 12 and w0["lengths"].shape[0] == 6 and w1["lengths"].shape[0] == 6
    assert not torch.equal(w0["dihedrals"], w1["dihedrals"])
    # strong: the ranks' slices of one batch
    whole = make(7, 0)
    parts = [bench.rank_inputs(make, 7, "strong", 2, r) for r in range(2)]
    assert all(t == 7 for _, t in parts)
    for k in whole:
        assert torch.equal(torch.cat([p[k] for p, _ in parts]), whole[k])
    # one rank: the same either way
    assert torch.equal(bench.rank_inputs(make, 5, "weak", 1, 0)[0]["grad"], bench.rank_inputs(make, 5, "strong", 1, 0)[0]["grad"])


def test_e2e_rank_summary_two_ranks():
    # the per-rank part of bench.py's e2e record, as rank 0 builds it from two ranks' gathered values
    import bench

    ranks = [[0.0, 54.8, 55.7, 1.70], [1.0, 50.2, 51.0, 1.80]]
    s = bench.e2e_rank_summary(ranks, 1.9)
    assert [p["rank"] for p in s["per_rank"]] == [0, 1]
    assert [p["numa_node"] for p in s["per_rank"]] == [0, 1]
    assert s["per_rank"][1]["h2d_gbs"] == 50.2 and s["per_rank"][1]["copy_floor_ms"] == 1.8
    assert s["copy_floor_ms"] == 1.8
    assert s["of_copy_floor"] == round(1.8 / 1.9, 3)
