"""The Exact Shortlist Head screened with the high nibble plane of the Q8 output head (QNT_OPEN_NIBBLE_SCREEN).

The screen is this build's own (the reference's research notes, docs/PROGRESS.md:121-130, describe it; its engine
screens with quanta.head_q4).  What must hold is what makes a shortlist exact: every row's exact logit lies within
its bound of the screen score, the rows scored exactly carry the full head's logits bit for bit, the top k rows are
among them, and so the sampled ids equal the full head's and the reference-screen shortlist's."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def check_head(m, tok, pos, hist, nv, ks=(1, 20)):
    full = m.forward(tok, pos)
    rows = []
    for k in ks:
        sl, coarse, upper = m.head(dict(top_k=k, n_valid=nv, must=hist), want_bounds=True)
        ex = sl != -np.inf
        assert np.array_equal(sl[ex], full[ex])
        assert np.all(np.abs(full[:nv] - coarse[:nv]) <= upper[:nv] - coarse[:nv])  # the bound holds for every row
        top = np.argsort(-full[:nv], kind="stable")[:k]
        assert np.all(ex[top])
        rows.append(m.last_head_rows)
    return full, rows


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_text", "q4mix_sl"])
def test_nibble_screen_bound_and_exact_rows(qb, models, name):
    """tiny_text has no quanta.head_q4: the nibble screen gives it a shortlist head."""
    m = qb.Model(models(name), ctx_len=1024, nibble_screen=True)
    try:
        assert m.has_shortlist
        nv = m.hp.n_tokens
        prompt = np.random.default_rng(31).integers(0, nv, 64)
        logits = m.forward_batch(prompt, 0)
        tok = int(np.argmax(logits[:nv]))
        seen = []
        for p in range(64, 72):
            hist = np.concatenate([prompt, [tok]])
            full, rows = check_head(m, tok, p, hist, nv)
            seen.append(rows)
            tok = int(np.argmax(full[:nv]))
            prompt = hist
        print(name, "exact rows per head pass (k=1, k=20):", seen)
    finally:
        m.close()


@pytest.mark.parametrize("top_k,penalty", [(20, 1.1), (1, 1.0), (40, 1.1)])
def test_nibble_screen_sampled_ids_equal_reference_screen(qb, models, top_k, penalty):
    """Config-4 sampling (T 0.7, top-p 0.8) on the full-size q4mix shortlist file: the nibble screen, the file's Q4
    screen and the full head sample the same ids (the Q4 screen is pinned to the reference elsewhere)."""
    path = models("q4mix_sl")
    prompt = np.random.default_rng(5).integers(0, 4000, 256)
    sp = qb.SamplerParams(temperature=0.7, top_k=top_k, top_p=0.8, repeat_penalty=penalty, seed=99)
    got = {}
    for key, nib, sl in (("nibble", True, True), ("q4", False, True), ("full", False, False)):
        m = qb.Model(path, ctx_len=1024, nibble_screen=nib)
        try:
            ids, st = m.generate(prompt, sp, 48, shortlist=sl)
            got[key] = (list(ids), st["head_rows"] / max(st["head_calls"], 1))
        finally:
            m.close()
    print("exact rows per step:", {k: round(v[1]) for k, v in got.items()})
    assert got["nibble"][0] == got["full"][0] == got["q4"][0]


def test_open_rejects_unknown_flags(qb, models):
    import ctypes as C
    h = C.c_void_p()
    rc = qb.lib().qnt_model_open(str(models("tiny_q8")).encode(), 256, 8, C.byref(h))
    assert rc == -1
