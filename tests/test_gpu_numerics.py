"""Exhaustive bit-for-bit checks of the exact arithmetic shortcuts the kernels use (tests/cuda/numerics_check.cu):
the quantizer's a / 127 and 1 / d and its half-away rounding, each against the CUDA operation it replaces over its
whole input range (about 2^32 inputs, a few milliseconds on the GPU)."""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_exact_shortcuts_over_every_input(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "numerics_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    f"-I{ROOT / 'quanta.cpp_b200' / 'csrc'}", str(ROOT / "tests" / "cuda" / "numerics_check.cu"),
                    "-o", str(exe)], check=True, capture_output=True, text=True, timeout=600)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    m = re.search(r"div127=(\d+) frcp=(\d+) round=(\d+)", r.stdout)
    assert m, r.stdout
    assert [int(g) for g in m.groups()] == [0, 0, 0], r.stdout
