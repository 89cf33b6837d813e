"""Pins the C restatement (oracle/qnt_oracle.c) to the reference built from its own sources (oracle/_ref) and to
the committed golden vectors (tests/golden, made by tests/golden/make_golden.py from the reference).  CPU only."""
import json
from pathlib import Path

import numpy as np
import pytest

import ref as R

GOLDEN = Path(__file__).resolve().parent / "golden"
need_ref = pytest.mark.skipif(not R.have_ref(), reason="reference not built (oracle/_ref)")


def _rng_q8(rng, rows, cols):
    from test_gpu_ops import q8_weights
    return q8_weights(rng, rows, cols)


def _rng_q4(rng, rows, cols):
    from test_gpu_ops import q4_gptq_weights
    return q4_gptq_weights(rng, rows, cols)


def test_f16_conversion_all_patterns():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([R.orc().orc_f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    w = want[::97]
    nan = np.isnan(w)
    assert np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan], w[~nan])


@need_ref
def test_restated_ops_bit_identical_to_reference():
    rng = np.random.default_rng(3)
    for n in (32, 896, 4864):
        x = rng.standard_normal(n).astype(np.float32) * rng.uniform(0.01, 100)
        assert all(np.array_equal(a, b) for a, b in zip(R.Oracle.quantize_q8(x), R.quantize_q8(x)))
    for dt, mk in ((2, _rng_q8), (3, _rng_q4)):
        rows, cols = 300, 896
        raw = mk(rng, rows, cols)
        X = rng.standard_normal((7, cols)).astype(np.float32)
        Q, D = zip(*(R.quantize_q8(x) for x in X))
        Q, D = np.stack(Q), np.stack(D)
        assert np.array_equal(R.Oracle.matvec_q(dt, rows, cols, raw, Q[0], D[0]), R.matvec_q(dt, rows, cols, raw, Q[0], D[0]))
        assert np.array_equal(R.Oracle.matmul_q(dt, rows, cols, raw, Q, D), R.matmul_q(dt, rows, cols, raw, Q, D))


@need_ref
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl", "tiny_had"])
def test_restated_model_bit_identical_to_reference(models, name):
    path = models(name)
    o = R.OracleModel(path)
    r = R.RefModel(path, threads=2)
    ids = np.random.default_rng(1).integers(0, o.vocab, 40)
    for p, t in enumerate(ids):
        assert np.array_equal(o.forward(t, p), r.forward(t, p)), p
    if name == "tiny_q4sl":
        nv = o.n_tokens
        for k in (1, 20):
            must = ids[-30:]
            a, ca, ua, ra = o.head(top_k=k, n_valid=nv, must=must, want_bounds=True)
            b, cb, ub, rb = r.head(top_k=k, n_valid=nv, must=must, want_bounds=True)
            assert np.array_equal(a, b) and np.array_equal(ca, cb) and np.array_equal(ua, ub) and ra == rb


@need_ref
def test_restated_sampler_matches_reference():
    rng = np.random.default_rng(4)
    hist = rng.integers(0, 500, 60)
    for params in (dict(temperature=0.0, repeat_penalty=1.0), dict(), dict(top_k=5, top_p=0.95, min_p=0.05),
                   dict(repeat_penalty=1.3, repeat_window=16)):
        a = R.OracleSampler(seed=99, **params)
        b = R.Sampler(seed=99, **params)
        for _ in range(50):
            lg = rng.standard_normal(500).astype(np.float32) * 3
            assert a.sample(lg, 480, hist) == b.sample(lg, 480, hist)


def test_golden_vectors():
    """The restatement reproduces the reference outputs committed under tests/golden."""
    meta = json.loads((GOLDEN / "golden.json").read_text())
    z = np.load(GOLDEN / "golden.npz")
    for case in meta["matvec"]:
        raw = z[case["raw"]]
        got = R.Oracle.matvec_q(case["dtype"], case["rows"], case["cols"], raw, z[case["q"]], z[case["d"]])
        assert np.array_equal(got, z[case["out"]]), case["name"]
    for case in meta["quantize"]:
        q, d = R.Oracle.quantize_q8(z[case["x"]])
        assert np.array_equal(q, z[case["q"]]) and np.array_equal(d, z[case["d"]]), case["name"]
    for case in meta["sampler"]:
        s = R.OracleSampler(**case["params"])
        got = [s.sample(z[case["logits"]][i], case["n_valid"], z[case["history"]]) for i in range(len(case["picks"]))]
        assert got == case["picks"], case["name"]


@need_ref
def test_hadamard_flag_needs_ffn_multiple_of_256(qb, tmp_path):
    """FLAG_HADAMARD_DOWN with ffn_dim % 256 != 0 is refused at load by the reference (engine/src/model.cpp:39-42) and
    by the restated oracle alike; with ffn_dim % 256 == 0 both load it."""
    bad = qb.synth_model(tmp_path / "had_bad.qnt", shape=dict(qb.TINY, ffn_dim=384), mlp_q4=False, shortlist=False,
                         seed=5, flags=1)
    with pytest.raises(RuntimeError):
        R.RefModel(bad, threads=1)
    with pytest.raises(RuntimeError):
        R.OracleModel(bad)
    good = qb.synth_model(tmp_path / "had_ok.qnt", shape=qb.TINY, mlp_q4=False, shortlist=False, seed=5, flags=1)
    R.RefModel(good, threads=1).close()
    R.OracleModel(good).close()
