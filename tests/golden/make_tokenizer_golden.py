"""Writes tests/golden/tokenizer_golden.json: the reference tokenizer's ids (oracle/_ref, engine/src/tokenizer.cpp) for
the tokenizer tests' strings on the generated BPE vocabulary of tests/tokenizer_vocab.py.  Run here, where the
reference exists:

    make -C oracle && python quanta.cpp_b200/build.py && python tests/golden/make_tokenizer_golden.py

The fixture pins the device build's tokenizer on machines without the reference.
"""
import json
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (ROOT / "oracle", ROOT / "quanta.cpp_b200", HERE.parent):
    sys.path.insert(0, str(p))
import quanta_b200 as qb  # noqa: E402  (the synthetic model writer)
import ref as R  # noqa: E402
import tokenizer_vocab as TV  # noqa: E402


def main():
    path = qb.synth_model(Path("/tmp/qnt_models/tiny_text.qnt"), shape=qb.TINY, mlp_q4=False, shortlist=False, seed=19,
                          tokenizer=TV.tokenizer_section(qb.TINY["n_tokens"]), overwrite=True)
    r = R.RefModel(path, threads=1)
    cases = [dict(text_hex=t.hex(), ids=r.tokenize(t).tolist()) for t in TV.test_strings(random.Random(7), 120)]
    specials = {s: r.token_id(s) for s in TV.SPECIALS}
    r.close()
    (HERE / "tokenizer_golden.json").write_text(json.dumps(dict(specials=specials, cases=cases)) + "\n")
    print(f"{len(cases)} cases")


if __name__ == "__main__":
    main()
