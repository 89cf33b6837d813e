"""Generated streams against the reference, id for id, on the full-size random-init Qwen2.5-0.5B files.

Config 4 (the benchmarked workload): q4mix + Exact Shortlist Head, a 512-token prompt, then 256 sampled steps at
temperature 0.7, top-k 20, top-p 0.8, fixed seed -- once with the repetition penalty 1.1 over the whole history (the
reference CLI's default, which makes every history id a must row of the shortlist) and once with 1.0.  On the device
the sampler's first stage is fused into the head kernels; the reference runs Session::generate
(engine/src/session.cpp:33-52) with Sampler::sample (engine/src/sampler.cpp:22-85).

Config 5: a batch of 256 sequences with 512-token prompts advanced together for 128 greedy tokens through
qnt_prefill_batch / qnt_decode_batch; 16 of them, picked at random, are replayed alone through the reference.
"""
import concurrent.futures as cf
import multiprocessing as mp
import os

import numpy as np
import pytest

import ref as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("penalty,top_k,steps", [(1.1, 20, 256), (1.0, 20, 256), (1.1, 0, 64), (1.1, 40, 64)])
def test_config4_sampled_stream_equals_reference(qb, models, penalty, top_k, steps):
    """top_k 0 and 40 run the device's sorting sampler after the full head (the reference: the full head for top_k 0,
    its shortlist with k = 40, whose exact rows are the full head's)."""
    path = models("q4mix_sl")
    m = qb.Model(path, ctx_len=1024)
    r = R.RefModel(path, ctx=1024)
    try:
        prompt = np.random.default_rng(41).integers(0, m.hp.n_tokens, 512).astype(np.int32)
        sp = qb.SamplerParams(temperature=0.7, top_k=top_k, top_p=0.8, repeat_penalty=penalty, seed=1234)
        got, st = m.generate(prompt, sp, steps, shortlist=True, batch_prefill=True)
        want, rst = r.generate(prompt, steps, temperature=0.7, top_k=top_k, top_p=0.8, repeat_penalty=penalty, seed=1234,
                               batch_prefill=True, shortlist=True)
        assert len(got) == len(want) == steps
        first = next((i for i in range(steps) if got[i] != want[i]), None)
        assert first is None, f"first differing step {first}: device {got[first]} reference {want[first]}"
        # both heads read about the same share of exact rows (the device counts the rows it rescored)
        print(f"rp {penalty}: {len(set(got.tolist()))} distinct ids; exact-row fraction device "
              f"{st['head_rows'] / max(st['head_calls'], 1) / m.vocab:.4f} reference {rst['head_fraction']:.4f}")
    finally:
        m.close()
        r.close()


def _replay(args):
    """One sequence alone through the reference (runs in a spawned worker process)."""
    path, prompt, n_gen, threads = args
    import ref as RR
    rm = RR.RefModel(path, ctx=1024, threads=threads)
    ids, _ = rm.generate(np.asarray(prompt, np.int32), n_gen, temperature=0.0, repeat_penalty=1.0, batch_prefill=True,
                         shortlist=True)
    rm.close()
    return ids.tolist()


def test_config5_batch_sequences_replayed_through_reference(qb, models):
    path = models("q4mix_sl")
    n_seq, prompt_len, n_gen, n_check = 256, 512, 128, 16
    rng = np.random.default_rng(55)
    m = qb.Model(path, ctx_len=1024)
    prompts = rng.integers(0, m.hp.n_tokens, (n_seq, prompt_len)).astype(np.int32)
    check = sorted(rng.choice(n_seq, n_check, replace=False).tolist())
    # the reference replays run on the host cores while the device serves the batch
    workers = 4
    threads = max(1, (os.cpu_count() or 8) // workers)
    pool = cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn"))
    futs = [pool.submit(_replay, (str(path), prompts[s], n_gen, threads)) for s in check]
    try:
        m.batch_init(n_seq, prompt_len + n_gen + 8)
        got = [[m.prefill_batch(s, prompts[s])] for s in range(n_seq)]
        seqs = np.arange(n_seq, dtype=np.int32)
        for _ in range(n_gen - 1):
            nxt = m.decode_batch(seqs, [g[-1] for g in got])
            for s in range(n_seq):
                got[s].append(int(nxt[s]))
        wants = [f.result(timeout=1200) for f in futs]
    finally:
        pool.shutdown(cancel_futures=True)
        m.close()
    for s, want in zip(check, wants):
        assert len(want) == n_gen
        assert got[s] == want, (s, next(i for i in range(n_gen) if got[s][i] != want[i]))
