"""Accuracy of the kernels' own float sine/cosine (nerf_math.cuh), built for the host with g++ and
its correctly rounded fmaf, against double precision: below 1.25 ulp(1) of absolute error on the
whole fast range and below 1.15 ulp(1) on [-pi, pi] (the angles of real chains).  The bound is
absolute: the reduction by pi leaves |r| <= pi/2, where sin r reaches 1."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
ULP1 = 2.0**-23


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_sincos_fast_accuracy(tmp_path):
    exe = tmp_path / "sincos_accuracy"
    subprocess.run(
        ["g++", "-O2", "-mfma", "-std=c++17", f"-I{ROOT / 'cufk_b200' / 'csrc'}", str(ROOT / "tests" / "sincos_accuracy.cpp"), "-o", str(exe)],
        check=True,
    )
    near_s, near_c, wide_s, wide_c = map(float, subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split())
    assert near_s < 1.15 * ULP1 and near_c < 1.15 * ULP1, (near_s, near_c)
    assert wide_s < 1.25 * ULP1 and wide_c < 1.25 * ULP1, (wide_s, wide_c)
