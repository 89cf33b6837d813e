"""The drop-in at the ops level, proved with the reference's own code: oracle/_ref/cuda/quanta is the reference CLI
linked with a kernel registry (oracle/cuda_dispatch.cpp, the interface of engine/src/ops_dispatch.cpp:53-77) that
lists the B200 kernels as the families `cuda` (CUDA-core matmul) and `cuda_tc` (tcgen05 matmul), through
qnt_matvec_host / qnt_matmul_host.

- `quanta selftest` (engine/src/checks.cpp:64-146) checks each family's matvec against matvec_q_ref on the 4864 x 896
  Q8_0 and Q4_0 fixtures and each family's matmul (x32 and a ragged x7) against its own matvec, bit for bit.
- `QUANTA_KERNEL=cuda quanta gen` runs the reference's Model::forward with every linear layer on the device kernels,
  called from its thread pool on disjoint row ranges at once, and must give the ids of the scalar family.
"""
import os
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "oracle" / "_ref" / "cuda" / "quanta"


def _cli():
    if not CLI.exists():
        pytest.skip("oracle/_ref/cuda/quanta not built (make -C oracle cuda)")
    return str(CLI)


def test_reference_selftest_passes_on_device_families():
    r = subprocess.run([_cli(), "selftest"], capture_output=True, text=True, timeout=600, env=dict(os.environ))
    out = r.stdout + r.stderr
    print(out)
    assert r.returncode == 0, out
    for dt in ("q8_0", "q4_0"):
        for fam in ("cuda", "cuda_tc"):
            mv = re.search(rf"^{dt}\s+{fam}\s+matvec max err (\S+) .* (PASS|FAIL)\s+([\d.]+) us", out, re.M)
            assert mv and mv.group(2) == "PASS", (dt, fam, out)
            assert float(mv.group(1)) == 0.0  # the device matvec equals matvec_q_ref bit for bit
            mm = re.search(rf"^{dt}\s+{fam}\s+matmul x32: bit-exact (PASS|FAIL)", out, re.M)
            assert mm and mm.group(1) == "PASS", (dt, fam, out)


def test_reference_model_runs_on_device_kernels(models):
    path = models("tiny_q8")
    ids = ",".join(str(i) for i in np.random.default_rng(3).integers(0, 4900, 20))
    got = {}
    for fam in ("ref", "cuda", "cuda_tc"):
        env = dict(os.environ, QUANTA_KERNEL=fam)
        r = subprocess.run([_cli(), "gen", "-m", str(path), "--ids", ids, "-n", "16", "-t", "4"], capture_output=True,
                           text=True, timeout=600, env=env)
        assert r.returncode == 0, r.stdout + r.stderr
        got[fam] = r.stdout.strip().splitlines()[-1]
    assert got["cuda"] == got["ref"] == got["cuda_tc"], got
