"""The command-line driver (tools/cli/main.cpp's commands over the C ABI): selftest, checkbatch and checkhead print
the reference's PASS lines and exit 0; gen prints the same greedy ids as the library; the text commands (tokenize,
run, chat, ppl) print what the reference CLI (oracle/_ref/quanta) prints for the same model, text, flags and seed;
bench, batchcurve and compare produce their reports."""
import random
import re
import subprocess
from pathlib import Path

import tokenizer_vocab as TV

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def cli(qb, *args, stdin=None):
    exe = qb.PKG / "lib" / "quanta_b200"
    return subprocess.run([str(exe), *map(str, args)], capture_output=True, timeout=600, input=stdin, encoding="utf-8",
                          errors="surrogateescape")


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


REF_CLI = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "quanta"


def ref_cli(*args, stdin=None):
    if not REF_CLI.exists():
        pytest.skip("oracle/_ref/quanta not built")
    return subprocess.run([str(REF_CLI), *map(str, args)], capture_output=True, timeout=600, input=stdin, encoding="utf-8",
                          errors="surrogateescape")


def test_cli_tokenize_run_chat_match_reference(qb, models):
    path = models("tiny_text")
    text = TV.sample_text(random.Random(11), 60)
    a, b = cli(qb, "tokenize", "-m", path, "-p", text), ref_cli("tokenize", "-m", path, "-p", text)
    assert a.returncode == 0 and a.stdout == b.stdout
    for flags in (["--seed", "5"], ["--greedy"], ["--seed", "9", "--top-k", "0", "--temp", "1.1", "--no-batch"]):
        a = cli(qb, "run", "-m", path, "-p", text, "-n", "40", *flags)
        b = ref_cli("run", "-m", path, "-p", text, "-n", "40", *flags)
        assert a.returncode == 0, a.stderr
        assert a.stdout == b.stdout, flags
    turns = "hello there\nwhat comes next?\n/reset\nonce more, from the start\nand again\n/exit\n"
    a = cli(qb, "chat", "-m", path, "-n", "24", "--seed", "7", stdin=turns)
    b = ref_cli("chat", "-m", path, "-n", "24", "--seed", "7", stdin=turns)
    assert a.returncode == 0, a.stderr
    assert a.stdout == b.stdout and len(a.stdout) > 0


def test_cli_ppl_matches_reference(qb, models, tmp_path):
    path = models("tiny_text")
    f = tmp_path / "text.txt"
    f.write_text(TV.sample_text(random.Random(12), 400))
    pat = re.compile(r"ppl ([\d.]+) over (\d+) tokens")
    a = pat.search(cli(qb, "ppl", "-m", path, "-f", f, "-n", "300").stdout)
    b = pat.search(ref_cli("ppl", "-m", path, "-f", f, "-n", "300").stdout)
    assert a and b and a.group(2) == b.group(2) == "299"
    print("ppl device", a.group(1), "reference", b.group(1))
    assert abs(float(a.group(1)) / float(b.group(1)) - 1) < 1e-6


def test_cli_reports(qb, models):
    r = cli(qb, "bench", "-m", models("tiny_q4sl"))
    assert r.returncode == 0 and "ALL PASS" in r.stdout, r.stdout + r.stderr
    assert "decode output identical (full vs shortlist): PASS" in r.stdout
    r = cli(qb, "batchcurve", "-m", models("tiny_q8"))
    assert r.returncode == 0 and len(re.findall(r"^\s+\d+\s+[\d.]+\s+[\d.]+x", r.stdout, re.M)) == 6, r.stdout
    r = cli(qb, "compare", "-m", models("tiny_q4sl"))
    assert r.returncode == 0 and r.stdout.count("RESULT engine=quanta_b200") == 2, r.stdout
