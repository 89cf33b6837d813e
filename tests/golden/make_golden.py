"""Writes tests/golden/golden.{npz,json}: outputs of the reference engine built from its own sources
(oracle/_ref/libquanta_ref.so) on small seeded inputs.  Run here, where the reference exists:

    make -C oracle && python tests/golden/make_golden.py

The fixtures pin the C restatement (oracle/qnt_oracle.c) on machines without the reference.
"""
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
sys.path.insert(0, str(HERE.parent))
import ref as R  # noqa: E402
from test_gpu_ops import q4_gptq_weights, q8_weights  # noqa: E402


def xorshift_fixture(dt, rows, cols):
    """engine/src/checks.cpp:64-89 generator at a reduced row count."""
    state = 0x9E3779B97F4A7C15
    M = (1 << 64) - 1

    def nxt():
        nonlocal state
        state ^= (state << 13) & M
        state ^= state >> 7
        state ^= (state << 17) & M
        return state

    qbytes = rows * cols if dt == 2 else rows * cols // 2
    q = np.array([nxt() & 0xFF for _ in range(qbytes)], np.uint8)
    s = np.array([0x2000 + nxt() % 0x800 for _ in range(rows * cols // 32)], np.uint16)
    x = np.array([float(int(nxt() % 2001) - 1000) / 1000.0 for _ in range(cols)], np.float32)
    return np.concatenate([q, s.view(np.uint8)]), x


def main():
    arrays, meta = {}, {"matvec": [], "quantize": [], "sampler": []}
    rng = np.random.default_rng(20261201)
    cases = [("selftest_q8", 2, 64, 896, *xorshift_fixture(2, 64, 896)),
             ("selftest_q4", 3, 64, 896, *xorshift_fixture(3, 64, 896)),
             ("normal_q8", 2, 96, 896, q8_weights(rng, 96, 896), rng.standard_normal(896).astype(np.float32)),
             ("gptq_q4_down", 3, 16, 4864, q4_gptq_weights(rng, 16, 4864), rng.standard_normal(4864).astype(np.float32))]
    for name, dt, rows, cols, raw, x in cases:
        q, d = R.quantize_q8(x)
        arrays[name + "_raw"], arrays[name + "_q"], arrays[name + "_d"] = raw, q, d
        arrays[name + "_out"] = R.matvec_q(dt, rows, cols, raw, q, d)
        meta["matvec"].append(dict(name=name, dtype=dt, rows=rows, cols=cols, raw=name + "_raw", q=name + "_q",
                                   d=name + "_d", out=name + "_out"))
    for i, scale in enumerate((0.0, 1e-3, 1.0, 300.0)):
        x = (rng.standard_normal(256) * scale).astype(np.float32)
        x[5] = 0.5 * scale  # ties of the form k + 0.5 after scaling are rare; keep a spread of magnitudes
        q, d = R.quantize_q8(x)
        arrays[f"qx{i}"], arrays[f"qq{i}"], arrays[f"qd{i}"] = x, q, d
        meta["quantize"].append(dict(name=f"quantize_{i}", x=f"qx{i}", q=f"qq{i}", d=f"qd{i}"))
    hist = rng.integers(0, 400, 40).astype(np.int32)
    arrays["hist"] = hist
    for j, params in enumerate([dict(temperature=0.0, repeat_penalty=1.0), dict(seed=1234), dict(seed=7, top_k=8, min_p=0.1),
                                dict(seed=5, repeat_penalty=1.3, repeat_window=10, top_p=0.9)]):
        lg = (rng.standard_normal((12, 400)) * 2.5).astype(np.float32)
        s = R.Sampler(**params)
        picks = [int(s.sample(lg[i], 390, hist)) for i in range(12)]
        arrays[f"lg{j}"] = lg
        meta["sampler"].append(dict(name=f"sampler_{j}", params=params, logits=f"lg{j}", history="hist", n_valid=390,
                                    picks=picks))
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", HERE / "golden.npz", (HERE / "golden.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
