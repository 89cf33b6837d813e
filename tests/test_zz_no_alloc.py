"""qnt_sampler_sample_noalloc (static device scratch, no allocation) against the sampler object's entry point
qnt_sampler_sample: the same ids and the same in-place edit of the logits on two calls in a row, with the xorshift64*
state carried from the first call to the second.  Collected last so that it also runs after every other test."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    dict(temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=1234),
    dict(temperature=0.0, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.3, repeat_window=8, seed=7),
    dict(temperature=1.2, top_k=32, top_p=0.95, min_p=0.02, repeat_penalty=1.0, repeat_window=0, seed=99),
]


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_noalloc_matches_sampler_object(qb, ci):
    import torch
    p = CASES[ci]
    sp = qb.SamplerParams(**p)
    obj = qb.Sampler(sp)
    state = (p["seed"] or 1) | 1
    rng = np.random.default_rng(500 + ci)
    V, n_valid = 151936, 151665
    history = list(rng.integers(0, n_valid, 64))
    for call in range(2):
        logits = (rng.standard_normal(V) * 2.5).astype(np.float32)
        a = torch.from_numpy(logits).cuda()
        b = a.clone()
        want = obj.sample(a, n_valid, history)
        got, state = qb.sample_noalloc(sp, state, b, n_valid, history)
        assert got == want, (call, got, want)
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
        history.append(got)
    obj.close()


def test_noalloc_rejects_sizes_beyond_its_limits(qb):
    import torch
    sp = qb.SamplerParams(temperature=0.7, top_k=20, seed=1)
    big = torch.zeros(262145, device="cuda")
    with pytest.raises(qb.QntError, match="262144"):
        qb.sample_noalloc(sp, 3, big)
    small = torch.zeros(1000, device="cuda")
    with pytest.raises(qb.QntError, match="32768"):
        qb.sample_noalloc(sp, 3, small, 1000, np.zeros(32769, np.int32))
    with pytest.raises(qb.QntError):
        qb.sample_noalloc(qb.SamplerParams(temperature=0.7, top_k=33), 3, small)
