"""A sampled session's repetition window (`repeat_window`) with the shortlist head.

Inside a decode step the sampler marks the next head's must ids (the penalised window of the history after its own
draw); this checks those marks against an independent route: the full head token by token and the standalone
sampler (pinned to the reference's Sampler in test_gpu_sampler.py) given the same history.  21 steps run as two
8-step graphs and five single steps."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("window,penalty", [(8, 1.3), (3, 1.5), (0, 1.2), (8, 1.0)])
def test_session_window_matches_full_head_and_sampler(qb, models, window, penalty):
    import torch
    path = models("tiny_q4sl")
    sp = qb.SamplerParams(temperature=0.8, top_k=20, top_p=0.9, repeat_penalty=penalty, repeat_window=window, seed=7)
    m = qb.Model(path, ctx_len=256)
    nv = m.hp.n_tokens
    rng = np.random.default_rng(window * 10 + int(penalty * 10))
    prompt = rng.integers(0, nv, 40).astype(np.int32)
    prompt[20:30] = prompt[:10]  # repeated ids inside and outside the window
    try:
        m.session_begin(prompt, sp)
        m.session_step(21)
        got, _ = m.session_read()
    finally:
        m.close()
    ref = qb.Model(path, ctx_len=256)
    smp = qb.Sampler(sp)
    try:
        hist = list(prompt)
        logits = ref.forward_batch(prompt, 0)
        want = []
        for step in range(21):
            t = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
            tok = smp.sample(t, nv, hist)
            want.append(tok)
            hist.append(tok)
            if step < 20:
                logits = ref.forward(tok, len(hist) - 1)
    finally:
        smp.close()
        ref.close()
    assert list(got) == want
