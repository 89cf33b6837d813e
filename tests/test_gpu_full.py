"""Full-size parity on the GPU: random-init Qwen2.5-0.5B (BASELINE configs 3 and 4) against the reference engine on the
same .qnt files and ids.

Config 3 (Q8_0 file): 128 uniform-random prompt ids prefilled in one batched call, then 64 greedy steps; at every step
the device logits are compared with the reference's (max |diff| / max |ref logit|) and the greedy ids must agree.
Config 4 (q4mix + shortlist file): 512-token prompt, decode steps with the shortlist head: the exact rows equal the
device's full head bit for bit and the chosen token is the full head's.
"""
import numpy as np
import pytest

import ref as R

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel_err(got, want):
    return float(np.max(np.abs(got - want)) / np.max(np.abs(want)))


def test_config3_prefill_and_64_greedy_steps(qb, models):
    path = models("q8_0")
    m = qb.Model(path, ctx_len=4096)
    r = R.RefModel(path, ctx=4096)
    prompt = np.random.default_rng(3).integers(0, m.hp.n_tokens, 128)
    got = m.forward_batch(prompt, 0)
    want = r.forward_batch(prompt, 0)
    errs = [rel_err(got, want)]
    agree = [int(np.argmax(got[:m.hp.n_tokens])) == int(np.argmax(want[:m.hp.n_tokens]))]
    tok = int(np.argmax(want[:m.hp.n_tokens]))
    for p in range(128, 128 + 64):
        got = m.forward(tok, p)
        want = r.forward(tok, p)
        errs.append(rel_err(got, want))
        agree.append(int(np.argmax(got[:m.hp.n_tokens])) == int(np.argmax(want[:m.hp.n_tokens])))
        tok = int(np.argmax(want[:m.hp.n_tokens]))
    print("config3 rel errors: max %.3e median %.3e; argmax agree %d/%d" % (max(errs), np.median(errs), sum(agree), len(agree)))
    assert all(agree)
    assert max(errs) < TOL, errs


def test_config4_shortlist_matches_full_head(qb, models):
    path = models("q4mix_sl")
    m = qb.Model(path, ctx_len=4096)
    r = R.RefModel(path, ctx=4096)
    nv = m.hp.n_tokens
    prompt = np.random.default_rng(4).integers(0, nv, 512)
    full = m.forward_batch(prompt, 0)
    want = r.forward_batch(prompt, 0)
    errs = [rel_err(full, want)]
    tok = int(np.argmax(want[:nv]))
    for p in range(512, 512 + 8):
        full = m.forward(tok, p)
        hist = np.concatenate([prompt, [tok]])
        for k in (1, 20):
            sl, coarse, upper = m.head(dict(top_k=k, n_valid=nv, must=hist), want_bounds=True)
            ex = sl != -np.inf
            assert np.array_equal(sl[ex], full[ex])
            assert np.all(np.abs(full - coarse) <= upper - coarse)
            assert int(np.argmax(sl[:nv])) == int(np.argmax(full[:nv]))
            top = np.argsort(-full[:nv], kind="stable")[:k]
            assert np.all(ex[top])
        want = r.forward(tok, p)
        errs.append(rel_err(full, want))
        tok = int(np.argmax(want[:nv]))
        prompt = hist
    print("config4 rel errors:", ["%.2e" % e for e in errs])
    assert max(errs) < TOL, errs


_FUSE_SCRIPT = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import quanta_b200 as qb
m = qb.Model(sys.argv[2], ctx_len=4096)
prompt = np.random.default_rng(21).integers(0, m.hp.n_tokens, 300)
ids, st = m.generate(prompt, qb.SamplerParams(seed=99), 48, shortlist=True, batch_prefill=True)
print(json.dumps({"ids": [int(i) for i in ids], "kps": st["kernels_per_step"], "layers": m.hp.n_layers}))
"""


def test_fused_qkv_attention_decode_equals_two_kernels(qb, models):
    """Decode with the q|k|v matvec fused into the attention kernel (the default where the shape allows) against the
    two-kernel path (QNT_FUSE_QKV=0): the same sampled ids on the full-size q4mix model, and one launch fewer per
    layer, so the fused kernel is the one that ran."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path

    path = models("q4mix_sl")
    pkg = str(Path(qb.__file__).resolve().parent)
    out = {}
    for fuse in ("1", "0"):
        env = dict(os.environ, QNT_FUSE_QKV=fuse)
        r = subprocess.run([sys.executable, "-c", _FUSE_SCRIPT, pkg, str(path)], env=env, capture_output=True,
                           text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        out[fuse] = json.loads(r.stdout.strip().splitlines()[-1])
    assert len(out["1"]["ids"]) == 48
    assert out["1"]["ids"] == out["0"]["ids"]
    assert out["0"]["kps"] - out["1"]["kps"] == out["1"]["layers"], (out["0"]["kps"], out["1"]["kps"])
