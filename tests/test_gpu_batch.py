"""Batched serving (qnt_prefill_batch / qnt_decode_batch): several sequences with their own KV caches advanced
together through the tensor-core matmul and the fused greedy head must produce exactly the ids each sequence gets
alone from the single-stream path (Session::generate at temperature 0, which is itself checked against the
reference), whatever the mix of sequences in a step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def greedy_alone(qb, m, prompt, n):
    sp = qb.SamplerParams(temperature=0.0, top_k=1, repeat_penalty=1.0, seed=1)
    ids, _ = m.generate(np.asarray(prompt, np.int32), sp, n, shortlist=False, batch_prefill=True)
    return list(ids)


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl"])
def test_batch_decode_equals_single_stream(qb, models, name):
    m = qb.Model(models(name), ctx_len=512)
    try:
        rng = np.random.default_rng(21)
        lens = [10, 25, 40, 60, 3]
        prompts = [rng.integers(0, m.hp.n_tokens, n) for n in lens]
        steps = 16
        want = [greedy_alone(qb, m, p, steps + 1) for p in prompts]
        m.batch_init(len(prompts), 256)
        got = [[m.prefill_batch(s, p)] for s, p in enumerate(prompts)]
        for k in range(steps):
            # a different mix and order of sequences in each step (every sequence advances once per step)
            order = rng.permutation(len(prompts))
            nxt = m.decode_batch(order, [got[s][-1] for s in order])
            for s, t in zip(order, nxt):
                got[s].append(int(t))
        for s in range(len(prompts)):
            assert got[s] == want[s], (s, got[s], want[s])
    finally:
        m.close()


def test_batch_full_size_64_sequences(qb, models):
    """The q4mix shortlist file at Qwen2.5-0.5B shapes: 64 sequences, 48-token prompts, 8 greedy steps."""
    m = qb.Model(models("q4mix_sl"), ctx_len=1024)
    try:
        rng = np.random.default_rng(5)
        n_seq, steps = 64, 8
        prompts = [rng.integers(0, m.hp.n_tokens, 48) for _ in range(n_seq)]
        m.batch_init(n_seq, 128)
        got = [[m.prefill_batch(s, p)] for s, p in enumerate(prompts)]
        for _ in range(steps):
            nxt = m.decode_batch(np.arange(n_seq), [g[-1] for g in got])
            for s in range(n_seq):
                got[s].append(int(nxt[s]))
        for s in (0, 17, 63):
            assert got[s] == greedy_alone(qb, m, prompts[s], steps + 1), s
    finally:
        m.close()


def test_batch_rejects_duplicates_and_overflow(qb, models):
    m = qb.Model(models("tiny_q8"), ctx_len=512)
    try:
        m.batch_init(2, 8)
        m.prefill_batch(0, [1, 2, 3])
        with pytest.raises(qb.QntError):
            m.decode_batch([0, 0], [4, 5])
        with pytest.raises(qb.QntError):
            m.prefill_batch(1, list(range(9)))
    finally:
        m.close()


def test_matmul_epilogue_fusions_give_the_same_ids(qb, models, monkeypatch):
    """QNT_TC_SWIGLU=1 / QNT_TC_QKV=1 move the SwiGLU + quantize and the q|k|v bias / RoPE / K-V stores into the
    tensor-core matmul's epilogue: the batched ids (64 sequences at Qwen2.5-0.5B shapes) equal the default kernels'."""
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 4000, 48) for _ in range(64)]

    def run():
        m = qb.Model(models("q4mix_sl"), ctx_len=1024)
        try:
            m.batch_init(64, 128)
            got = [[m.prefill_batch(s, p)] for s, p in enumerate(prompts)]
            for _ in range(6):
                nxt = m.decode_batch(np.arange(64), [g[-1] for g in got])
                for s in range(64):
                    got[s].append(int(nxt[s]))
            return got
        finally:
            m.close()

    want = run()
    monkeypatch.setenv("QNT_TC_SWIGLU", "1")
    monkeypatch.setenv("QNT_TC_QKV", "1")
    assert run() == want
