"""The host tokenizer (quanta.cpp_b200/csrc/tokenizer.cpp, C ABI qnt_tokenize / qnt_token_piece / qnt_token_id) against
the reference's Tokenizer (engine/src/tokenizer.cpp, built in oracle/_ref) on a byte-level BPE vocabulary with real
merges and code-point classes (tests/tokenizer_vocab.py): every rule of the split pattern, special tokens, invalid
UTF-8 and generated strings; plus the committed golden ids (tests/golden/tokenizer_golden.json) and round trips.
CPU only: the tokenizer needs no GPU."""
import json
import random
from pathlib import Path

import pytest

import ref as R
import tokenizer_vocab as TV

GOLDEN = Path(__file__).resolve().parent / "golden" / "tokenizer_golden.json"


@pytest.fixture(scope="module")
def text_model(models):
    return models("tiny_text")


@pytest.fixture(scope="module")
def tok(qb, text_model):
    t = qb.Tokenizer(text_model)
    yield t
    t.close()


def test_matches_golden_ids(tok):
    g = json.loads(GOLDEN.read_text())
    for s, i in g["specials"].items():
        assert tok.token_id(s) == i
    for c in g["cases"]:
        text = bytes.fromhex(c["text_hex"])
        assert tok.encode(text).tolist() == c["ids"], text


@pytest.mark.skipif(not R.have_ref(), reason="reference not built (oracle/_ref)")
def test_matches_reference_tokenizer(tok, text_model):
    r = R.RefModel(text_model, threads=1)
    try:
        for text in TV.test_strings(random.Random(99), 400):
            assert tok.encode(text).tolist() == r.tokenize(text).tolist(), text
    finally:
        r.close()


def test_round_trip_and_merges(tok):
    rng = random.Random(5)
    text = TV.sample_text(rng, 400).encode()
    ids = tok.encode(text)
    assert tok.decode(ids) == text
    assert len(ids) < len(text) / 2  # the merges do shorten generated prose
    assert tok.decode(tok.encode("<|im_start|>user\n")) == b"<|im_start|>user\n"
    assert tok.decode(10 ** 9) == b""


def test_vocabulary_without_byte_tokens_is_rejected(qb, tmp_path):
    import struct
    blob = struct.pack("<I", 3) + b"".join(struct.pack("<I", 1) + bytes([c]) for c in b"abc") + struct.pack("<IIIII", 0, 0, 0, 0, 0)
    path = qb.synth_model(tmp_path / "bad_vocab.qnt", shape=dict(qb.TINY, n_tokens=3), mlp_q4=False, shortlist=False,
                          seed=1, tokenizer=blob)
    with pytest.raises(qb.QntError, match="single-byte token"):
        qb.Tokenizer(path)
