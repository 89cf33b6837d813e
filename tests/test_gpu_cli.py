"""The command-line driver (tools/cli/main.cpp's commands over the C ABI): selftest, checkbatch and checkhead print
the reference's PASS lines and exit 0; gen prints the same greedy ids as the library."""
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def cli(qb, *args):
    exe = qb.PKG / "lib" / "quanta_b200"
    return subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=600)


def test_cli_selftest(qb):
    r = cli(qb, "selftest")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and r.stdout.count("PASS") >= 7


def test_cli_checkbatch_and_checkhead(qb, models):
    ids = ",".join(map(str, np.random.default_rng(2).integers(0, 4000, 140)))
    r = cli(qb, "checkbatch", "-m", models("tiny_q4sl"), "--ctx", "512", "--ids", ids)
    assert r.returncode == 0 and r.stdout.count("PASS") == 7, r.stdout + r.stderr
    r = cli(qb, "checkhead", "-m", models("tiny_q4sl"), "--ctx", "512", "--ids", ids[:200])
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr


def test_cli_gen_matches_library(qb, models):
    prompt = np.random.default_rng(3).integers(0, 4000, 20)
    r = cli(qb, "gen", "-m", models("tiny_q8"), "--ctx", "512", "-n", "12", "--ids", ",".join(map(str, prompt)))
    assert r.returncode == 0, r.stderr
    m = qb.Model(models("tiny_q8"), ctx_len=512)
    try:
        want, _ = m.generate(prompt, qb.SamplerParams(temperature=0.0, repeat_penalty=1.0), 12, shortlist=True)
    finally:
        m.close()
    assert [int(x) for x in r.stdout.strip().split(",")] == list(want)


def test_cli_text_commands_explain(qb, models):
    r = cli(qb, "run", "-m", models("tiny_q8"))
    assert r.returncode == 2 and "tokenizer" in r.stderr
