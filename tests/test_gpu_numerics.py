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


def test_exp_ref_equals_host_expf_over_every_input(tmp_path):
    """exp_ref (the device e^x of softmax, SwiGLU and the sampler) against the host libm's expf for every float in
    (-104, 89), about 2.2e9 inputs: zero mismatches.  Checks the device's own double exp rounding too, which is not
    correctly rounded and could fall on the other side of a float midpoint than the host's."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "exp_check"
    csrc = ROOT / "quanta.cpp_b200" / "csrc"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", f"-I{csrc}",
                    str(ROOT / "tests" / "cuda" / "exp_check.cu"), str(csrc / "exp_table.cpp"), "-o", str(exe)],
                   check=True, capture_output=True, text=True, timeout=600)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    m = re.search(r"exp_ref checked=(\d+) mismatches=(\d+)", r.stdout)
    assert m, r.stdout
    print(r.stdout)
    assert int(m.group(1)) > 2_000_000_000
    assert int(m.group(2)) == 0, r.stdout
