"""The standalone device sampler (qnt_sampler_*, Sampler::sample of engine/src/sampler.cpp:22-85) against the
reference's own Sampler (oracle/_ref) on the same logits, history and seed: identical ids over consecutive calls (the
xorshift64* state carries over), and the in-place edit of the logits (the penalised ids) bit-identical.  Exact ties
among the top logits are avoided: the reference orders equal logits by std::nth_element/std::sort, which are not
stable, while the device breaks ties toward the lower id."""
import numpy as np
import pytest

import ref as R

pytestmark = pytest.mark.gpu

PARAMS = [
    dict(temperature=0.0, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=5),
    dict(temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=1234),
    dict(temperature=1.0, top_k=32, top_p=1.0, min_p=0.05, repeat_penalty=1.3, repeat_window=16, seed=77),
    dict(temperature=0.5, top_k=5, top_p=0.9, min_p=0.0, repeat_penalty=1.0, repeat_window=0, seed=3),
    dict(temperature=1.5, top_k=1, top_p=1.0, min_p=0.0, repeat_penalty=1.2, repeat_window=4, seed=9),
    # top_k 0 (disabled) and above 32: the sorting sampler over every id below n_valid
    dict(temperature=0.7, top_k=0, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=1234),
    dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.0, repeat_window=0, seed=11),
    dict(temperature=0.8, top_k=0, top_p=0.95, min_p=0.01, repeat_penalty=1.2, repeat_window=8, seed=12),
    dict(temperature=0.7, top_k=40, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=13),
    dict(temperature=1.3, top_k=100, top_p=0.9, min_p=0.02, repeat_penalty=1.05, repeat_window=0, seed=14),
    dict(temperature=2.0, top_k=5000, top_p=1.0, min_p=0.0, repeat_penalty=1.0, repeat_window=0, seed=15),
]


def distinct(logits):
    """Nudges repeated values to neighbouring floats: the reference orders equal logits by an unstable sort."""
    while True:
        _, first, counts = np.unique(logits, return_index=True, return_counts=True)
        dup = np.setdiff1d(np.arange(logits.size), first)
        if dup.size == 0:
            return logits
        logits[dup] = np.nextafter(logits[dup], np.float32(np.inf))


@pytest.mark.parametrize("pi", range(len(PARAMS)))
def test_sampler_matches_reference(qb, pi):
    import torch
    if not R.have_ref():
        pytest.skip("oracle/_ref not built")
    p = PARAMS[pi]
    rng = np.random.default_rng(100 + pi)
    V, n_valid = 151936, 151665
    dev = qb.Sampler(qb.SamplerParams(**p))
    ref = R.Sampler(**p)
    history = list(rng.integers(0, V, 40))  # ids >= n_valid are skipped by the penalty, as in the reference
    history += [history[3], history[7], -1]
    for step in range(8):
        logits = (rng.standard_normal(V) * 3.0).astype(np.float32)
        # a few close contenders (distinct values: the reference orders equal logits by an unstable sort)
        logits[rng.choice(n_valid, 3, replace=False)] = logits.max() + np.float32([0.5, 0.5002, 0.4998])
        if p["top_k"] == 0 or p["top_k"] > 32:
            logits = distinct(logits)
        t = torch.from_numpy(logits).cuda()
        got = dev.sample(t, n_valid, history)
        want = ref.sample(logits, n_valid, history)
        assert got == want, (step, got, want)
        edited = t.cpu().numpy()
        assert np.array_equal(edited[:n_valid].view(np.uint32), ref.last_logits[:n_valid].view(np.uint32))
        history.append(got)
    dev.close()


def test_sampler_small_vocab_keeps_every_id(qb):
    """top_k >= n_valid keeps every id (sampler.cpp:45-50)."""
    import torch
    if not R.have_ref():
        pytest.skip("oracle/_ref not built")
    for top_k in (20, 0, 64):
        p = dict(temperature=0.9, top_k=top_k, top_p=1.0, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=42)
        dev = qb.Sampler(qb.SamplerParams(**p))
        ref = R.Sampler(**p)
        rng = np.random.default_rng(1)
        for _ in range(16):
            logits = rng.standard_normal(12).astype(np.float32)
            t = torch.from_numpy(logits).cuda()
            assert dev.sample(t, 12, [1, 2, 2]) == ref.sample(logits, 12, [1, 2, 2]), top_k
        dev.close()


def test_sort_sampler_ties_and_long_tails(qb):
    """The sorting sampler's early-stopped chains on inputs built to stress them: many equal logits (ties sort by id,
    and every tied candidate has the same exp, so the sums do not depend on their order) and a flat distribution
    whose nucleus runs deep into the sorted order.  With equal top logits the draw's pick among tied ids is the one
    place the reference's unstable sort can differ, so the check there is on the sampled logit's value."""
    import torch
    if not R.have_ref():
        pytest.skip("oracle/_ref not built")
    V = 151936
    rng = np.random.default_rng(7)
    for case in range(4):
        p = dict(temperature=[0.7, 1.0, 3.0, 0.2][case], top_k=0, top_p=[0.8, 0.99, 0.999, 0.5][case], min_p=0.0,
                 repeat_penalty=1.0, repeat_window=0, seed=100 + case)
        dev = qb.Sampler(qb.SamplerParams(**p))
        ref = R.Sampler(**p)
        for step in range(4):
            if case % 2 == 0:
                logits = rng.integers(-40, 40, V).astype(np.float32) * np.float32(0.25)  # 320 distinct values
            else:
                logits = (rng.standard_normal(V) * 0.05).astype(np.float32)  # nearly flat
                logits = distinct(logits)
            t = torch.from_numpy(logits).cuda()
            got = dev.sample(t, V, [])
            want = ref.sample(logits, V, [])
            assert logits[got] == logits[want], (case, step, got, want)
            if case % 2 == 1:
                assert got == want, (case, step)
        dev.close()
