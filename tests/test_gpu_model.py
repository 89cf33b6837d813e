"""Model-level parity on the GPU against the reference engine on the same synthetic .qnt files.

Bars: logits within 1e-3 relative (max |diff| / max |ref logit|, as checks.cpp:97-102 scales
errors), greedy ids identical, batched prefill equal to token-by-token (on the device: bit-identical), shortlist
head exact rows bit-identical to the full head and its bound never violated (check_head, checks.cpp:178-239).
"""
import numpy as np
import pytest

import ref as R

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(got, want):
    return float(np.max(np.abs(got - want)) / np.max(np.abs(want)))


@pytest.fixture(scope="module")
def tiny(qb, models):
    out = {}
    for name in ("tiny_q8", "tiny_q4sl", "tiny_had"):
        out[name] = (qb.Model(models(name)), R.RefModel(models(name), threads=4))
    yield out
    for m, r in out.values():
        m.close()
        r.close()


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl", "tiny_had"])
def test_forward_logits_match_reference(tiny, name):
    m, r = tiny[name]
    rng = np.random.default_rng(5)
    ids = rng.integers(0, m.vocab, 70)
    worst = 0.0
    for p, t in enumerate(ids):
        got = m.forward(t, p)
        want = r.forward(t, p)
        worst = max(worst, rel_err(got, want))
        assert worst < TOL, (p, worst)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl", "tiny_had"])
def test_batched_prefill_equals_token_by_token(tiny, name):
    """check_batch (checks.cpp:148-176) on the device: maxdiff must be 0, incl. a second turn at pos0 > 0."""
    m, r = tiny[name]
    rng = np.random.default_rng(6)
    ids = rng.integers(0, m.vocab, 140)
    for pos0, n in [(0, 1), (0, 31), (0, 32), (0, 33), (0, 100), (40, 45), (0, 140)]:
        for p in range(pos0 + n):
            lg = m.forward(ids[p], p)
        want = lg
        if pos0 > 0:
            m.forward_batch(ids[:pos0], 0)
        got = m.forward_batch(ids[pos0:pos0 + n], pos0)
        assert np.array_equal(got, want), (pos0, n, np.abs(got - want).max())
        ref_lg = r.forward_batch(ids[:pos0 + n], 0)
        assert rel_err(got, ref_lg) < TOL


def test_long_prompt_batched_windows(qb, models):
    """Prompts past 512 positions: the batched attention streams its scores in windows (the single-token path keeps
    them resident), and both must give the same bits; the reference bounds the logits."""
    m = qb.Model(models("tiny_long"), ctx_len=2048)
    r = R.RefModel(models("tiny_long"), ctx=2048, threads=4)
    try:
        ids = np.random.default_rng(8).integers(0, m.vocab, 1200)
        by_token = {}
        for p in range(1200):
            lg = m.forward(ids[p], p)
            if p in (599, 1199):
                by_token[p] = lg
        got = m.forward_batch(ids[:1200], 0)
        assert np.array_equal(got, by_token[1199])
        m.forward_batch(ids[:600], 0)
        got2 = m.forward_batch(ids[600:1200], 600)
        assert np.array_equal(got2, by_token[1199])
        assert rel_err(got, r.forward_batch(ids[:1200], 0)) < TOL
    finally:
        m.close()
        r.close()


@pytest.mark.parametrize("k", [1, 20])
def test_shortlist_head_exact(tiny, k):
    """check_head: bound holds for every row; exact rows bit-identical to the full head; top-k and must included."""
    m, r = tiny["tiny_q4sl"]
    assert m.has_shortlist
    rng = np.random.default_rng(7)
    ids = rng.integers(0, m.vocab, 30)
    nv = m.hp.n_tokens
    for p, t in enumerate(ids):
        full = m.forward(t, p)
        must = ids[max(0, p - 63):p + 1]
        sl, coarse, upper = m.head(dict(top_k=k, n_valid=nv, must=must), want_bounds=True)
        bound = upper - coarse
        assert np.all(np.abs(full - coarse) <= bound)
        exact = sl != -np.inf
        assert np.array_equal(sl[exact], full[exact])
        top = np.argsort(-full[:nv], kind="stable")[:k]
        assert np.all(exact[top]) and np.all(exact[must[must < nv]])
        assert m.last_head_rows == int(exact.sum())
        # the reference's shortlist on the same token agrees on the chosen token and its coarse scores' bound
        rfull = r.forward(t, p)
        rsl, rco, rup, rows = r.head(top_k=k, n_valid=nv, must=must, want_bounds=True)
        assert int(np.argmax(sl[:nv])) == int(np.argmax(full[:nv]))
        assert rel_err(coarse, rco) < TOL


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl", "tiny_had"])
def test_greedy_ids_match_reference(tiny, name):
    m, r = tiny[name]
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, m.hp.n_tokens, 40)
    sp = __import__("quanta_b200").SamplerParams(temperature=0.0, repeat_penalty=1.0)
    got, st = m.generate(prompt, sp, 64, shortlist=True, batch_prefill=True)
    want, _ = r.generate(prompt, 64, temperature=0.0, repeat_penalty=1.0, batch_prefill=True, shortlist=True)
    assert len(got) == 64
    assert np.array_equal(got, want)


@pytest.mark.parametrize("top_k", [0, 40, 24, 28])
def test_sampled_ids_match_reference_any_top_k(tiny, qb, top_k):
    """Session::generate with sampling, against the reference, for top_k values around the device's limits: 0
    (disabled) and 40 run the sorting sampler; 24 keeps the shortlist (k + 8 seeds = 32); 28 uses the full head."""
    m, r = tiny["tiny_q4sl"]
    prompt = np.random.default_rng(12).integers(0, m.hp.n_tokens, 30)
    sp = qb.SamplerParams(temperature=0.9, top_k=top_k, top_p=0.9, repeat_penalty=1.1, seed=321)
    got, _ = m.generate(prompt, sp, 40, shortlist=True, batch_prefill=True)
    want, _ = r.generate(prompt, 40, temperature=0.9, top_k=top_k, top_p=0.9, repeat_penalty=1.1, seed=321,
                         batch_prefill=True, shortlist=True)
    assert np.array_equal(got, want)


def test_sampled_shortlist_equals_full_head(tiny, qb):
    """bench's `decode output identical (full vs shortlist)` (checks.cpp:371-373) with Qwen defaults, seed 1234."""
    m, _ = tiny["tiny_q4sl"]
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, m.hp.n_tokens, 50)
    sp = qb.SamplerParams(seed=1234)
    a, sa = m.generate(prompt, sp, 48, shortlist=True)
    b, sb = m.generate(prompt, sp, 48, shortlist=False)
    assert np.array_equal(a, b)
    assert sa["head_rows"] < sb["head_rows"]


def test_bad_position_and_token(tiny):
    m, _ = tiny["tiny_q8"]
    with pytest.raises(Exception):
        m.forward(1, m.hp.ctx_len)
    with pytest.raises(Exception):
        m.forward(m.vocab + 5, 0)
    m.forward(1, 0)  # the handle stays usable


def test_hadamard_flag_needs_ffn_multiple_of_256(qb, tmp_path):
    """The device refuses FLAG_HADAMARD_DOWN files whose ffn_dim is not a multiple of 256, with the reference's
    condition (engine/src/model.cpp:39-42), and loads the same shape without the flag."""
    bad = qb.synth_model(tmp_path / "had_bad.qnt", shape=dict(qb.TINY, ffn_dim=384), mlp_q4=False, shortlist=False,
                         seed=5, flags=1)
    with pytest.raises(qb.QntError, match="256"):
        qb.Model(bad)
    plain = qb.synth_model(tmp_path / "had_plain.qnt", shape=dict(qb.TINY, ffn_dim=384), mlp_q4=False, shortlist=False,
                           seed=5, flags=0)
    qb.Model(plain).close()
