"""The tensor-core prefilter's error bound allows the fp16 MMA's f32
accumulation an error of 2^-12 of sum |a_i b_i| (csrc/tcscan.cu).  This
builds a one-CTA tcgen05 probe against the library's own wrappers and
checks, over 32,768 fp16 dots of K = 128 in each of seven scenarios --
random mixed magnitudes and adversarial ones (one dominant product among
tiny ones, alternating-sign cancellation, partial sums that change exponent
between K slices, fp16 subnormal operands, operands near the fp16 maximum,
slices of their own scale) -- that the largest observed error stays far
below that allowance."""
from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def test_accumulation_error_far_below_the_allowance(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "tc_acc"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-I", str(REPO / "ultravec-ann_b200" / "csrc"), "-o", str(exe),
                    str(REPO / "tests" / "cuda" / "tc_accumulation_probe.cu")], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=120).stdout
    worst = [float(x) for x in re.findall(r"max \|tc-exact\|/sum\|ab\| = ([0-9.e+-]+)", out)]
    above = [int(x) for x in re.findall(r"above 2\^-12: (\d+) of", out)]
    assert out.count("scenario ") == 7 and len(worst) == 8 and len(above) == 8, out
    assert "timeout 0" in out and max(above) == 0, out
    assert max(worst) < 2.0 ** -16, out  # 16x inside the 2^-12 allowance at least
