"""Shared fixtures.  `-m gpu` tests need a B200 and the built libraries; the rest run on CPU.

Synthetic .qnt files are written once per session into $QNT_MODEL_DIR (default /tmp/qnt_models): tiny models for
the fast checks and, on demand, the full Qwen2.5-0.5B shapes of the BASELINE configs.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "quanta.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

MODEL_DIR = Path(os.environ.get("QNT_MODEL_DIR", "/tmp/qnt_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu)")
    config.addinivalue_line("markers", "slow: full-size (Qwen2.5-0.5B) model; minutes on CPU")


def _ensure_built():
    import quanta_b200 as qb
    if not (qb.LIB_DIR / "libqnt_synth.so").exists() or not qb.lib_path().exists():
        from build import build  # quanta.cpp_b200/build.py
        build()
    return qb


@pytest.fixture(scope="session")
def qb():
    return _ensure_built()


@pytest.fixture(scope="session")
def models(qb):
    """name -> path of seeded synthetic models (written lazily)."""
    made = {}

    def get(name: str) -> Path:
        if name in made:
            return made[name]
        specs = {
            "tiny_q8": dict(shape=qb.TINY, mlp_q4=False, shortlist=True, seed=7),
            "tiny_q4sl": dict(shape=qb.TINY, mlp_q4=True, shortlist=True, seed=11),
            "tiny_long": dict(shape=dict(qb.TINY, max_seq=2048), mlp_q4=True, shortlist=True, seed=13),
            "tiny_had": dict(shape=qb.TINY, mlp_q4=True, shortlist=True, seed=17, flags=1),  # FLAG_HADAMARD_DOWN
            "tiny_text": dict(shape=qb.TINY, mlp_q4=False, shortlist=False, seed=19),  # + a trained BPE vocabulary
            "q8_0": dict(shape=qb.QWEN05B, mlp_q4=False, shortlist=False, seed=1234),
            "q4mix_sl": dict(shape=qb.QWEN05B, mlp_q4=True, shortlist=True, seed=1234),
        }
        spec = specs[name]
        if name == "tiny_text":
            import tokenizer_vocab
            spec = dict(spec, tokenizer=tokenizer_vocab.tokenizer_section(qb.TINY["n_tokens"]))
        p = qb.synth_model(MODEL_DIR / f"{name}.qnt", **spec)
        made[name] = p
        return p

    return get
