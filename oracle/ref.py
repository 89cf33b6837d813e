"""ctypes binding of the reference engine built from its own sources (oracle/_ref/libquanta_ref.so, see
oracle/Makefile) and of the C restatement (oracle/_build/libqnt_oracle.so, see oracle/qnt_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
as the checker or the timed CPU path, never by the product.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_SO = HERE / "_ref" / "libquanta_ref.so"            # the checker: no FMA contraction
STOCK_SO = HERE / "_ref" / "stock" / "libquanta_ref.so"  # the reference's own Release flags (the timed CPU baseline)
ORACLE_SO = HERE / "_build" / "libqnt_oracle.so"
QK = 32

_refs = {}
_orc = None


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def have_ref(stock: bool = False) -> bool:
    return (STOCK_SO if stock else REF_SO).exists()


def ref(stock: bool = False) -> C.CDLL:
    """The reference engine (raises if oracle/_ref was not built).  stock: the build with the reference's own Release
    flags (FMA contraction on) instead of the contraction-free checker."""
    so = STOCK_SO if stock else REF_SO
    if so not in _refs:
        if not so.exists():
            raise RuntimeError(f"{so} missing: `make -C oracle` (needs the reference sources)")
        L = C.CDLL(str(so))
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.ref_model_open.argtypes = [C.c_char_p, I, I, I, C.c_char_p, I]
        L.ref_model_open.restype = P
        L.ref_model_close.argtypes = [P]
        for n in ("ref_vocab", "ref_n_tokens", "ref_ctx_len", "ref_n_threads", "ref_has_shortlist", "ref_last_head_rows"):
            getattr(L, n).argtypes = [P]
        L.ref_forward.argtypes = [P, I, I, I, I, P, I, P]
        L.ref_forward_batch.argtypes = [P, P, I, I, I, I, P, I, P]
        L.ref_head.argtypes = [P, I, I, P, I, P, P, P]
        L.ref_quantize_q8.argtypes = [P, I, P, P]
        L.ref_quantize_q8.restype = None
        L.ref_matvec_q.argtypes = [I, I, I, P, P, P, I, I, P]
        L.ref_matvec_q.restype = None
        L.ref_matmul_q.argtypes = [I, I, I, P, P, P, I, I, I, P, I]
        L.ref_matmul_q.restype = None
        L.ref_sampler_new.argtypes = [F, I, F, F, F, I, C.c_ulonglong]
        L.ref_sampler_new.restype = P
        L.ref_sampler_free.argtypes = [P]
        L.ref_sample.argtypes = [P, P, I, P, I]
        L.ref_generate.argtypes = [P, P, I, I, I, F, I, F, F, F, C.c_ulonglong, I, P, C.POINTER(C.c_double),
                                   C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.ref_tokenize.argtypes = [P, C.c_char_p, I, P, I]
        L.ref_token_id.argtypes = [P, C.c_char_p]
        L.ref_check_batch.argtypes = [P, P, I, I]
        L.ref_check_head.argtypes = [P, P, I]
        _refs[so] = L
    return _refs[so]


def quantize_q8(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // QK, np.float32)
    ref().ref_quantize_q8(_p(x), x.size, _p(q), _p(d))
    return q, d


def matvec_q(dtype: int, rows: int, cols: int, raw: np.ndarray, q: np.ndarray, d: np.ndarray, r0=0, r1=None):
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    raw = np.ascontiguousarray(raw).view(np.uint8)
    ref().ref_matvec_q(dtype, rows, cols, _p(raw), _p(np.ascontiguousarray(q, np.int8)), _p(np.ascontiguousarray(d, np.float32)),
                       r0, r1, _p(out))
    return out


def matmul_q(dtype: int, rows: int, cols: int, raw: np.ndarray, q: np.ndarray, d: np.ndarray):
    q = np.ascontiguousarray(q, np.int8)
    n = q.shape[0]
    out = np.zeros((n, rows), np.float32)
    raw = np.ascontiguousarray(raw).view(np.uint8)
    ref().ref_matmul_q(dtype, rows, cols, _p(raw), _p(q), _p(np.ascontiguousarray(d, np.float32)), n, 0, rows, _p(out), rows)
    return out


class RefModel:
    """quanta::Model of the reference (CPU).  stock=True: the build with the reference's Release flags."""

    def __init__(self, path, ctx: int = 0, threads: int = 0, kv_f16: bool = True, stock: bool = False):
        self.L = ref(stock)
        err = C.create_string_buffer(512)
        h = self.L.ref_model_open(str(path).encode(), ctx, threads, int(kv_f16), err, 512)
        if not h:
            raise RuntimeError("reference load failed: " + err.value.decode())
        self.h = h
        self.vocab = self.L.ref_vocab(h)
        self.n_tokens = self.L.ref_n_tokens(h)
        self.threads = self.L.ref_n_threads(h)
        self.out = np.zeros(self.vocab, np.float32)

    def close(self):
        if getattr(self, "h", None):
            self.L.ref_model_close(self.h)
            self.h = None

    __del__ = close

    def forward(self, token, pos, top_k=0, n_valid=0, must=None):
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        if self.L.ref_forward(self.h, int(token), int(pos), top_k, n_valid, _p(m), m.size, _p(self.out)) != 0:
            raise IndexError("reference forward failed")
        return self.out.copy()

    def forward_batch(self, tokens, pos0, top_k=0, n_valid=0, must=None):
        t = np.ascontiguousarray(tokens, np.int32)
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        if self.L.ref_forward_batch(self.h, _p(t), t.size, int(pos0), top_k, n_valid, _p(m), m.size, _p(self.out)) != 0:
            raise IndexError("reference forward_batch failed")
        return self.out.copy()

    def head(self, top_k=0, n_valid=0, must=None, want_bounds=False):
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        coarse = np.zeros(self.vocab, np.float32) if want_bounds else None
        upper = np.zeros(self.vocab, np.float32) if want_bounds else None
        rows = self.L.ref_head(self.h, top_k, n_valid, _p(m), m.size, _p(self.out), _p(coarse), _p(upper))
        if want_bounds:
            return self.out.copy(), coarse, upper, rows
        return self.out.copy()

    @property
    def last_head_rows(self):
        return self.L.ref_last_head_rows(self.h)

    def tokenize(self, text) -> np.ndarray:
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = self.L.ref_tokenize(self.h, b, len(b), None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.L.ref_tokenize(self.h, b, len(b), _p(out), n)
        return out[:n]

    def token_id(self, literal: str) -> int:
        return self.L.ref_token_id(self.h, literal.encode())

    def generate(self, prompt, n_gen, temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, seed=1234,
                 batch_prefill=True, shortlist=True):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_gen, 1), np.int32)
        tp, td, hf = C.c_double(), C.c_double(), C.c_double()
        n = self.L.ref_generate(self.h, _p(p), p.size, int(batch_prefill), int(shortlist), temperature, top_k, top_p, min_p,
                               repeat_penalty, seed, n_gen, _p(out), C.byref(tp), C.byref(td), C.byref(hf))
        if n < 0:
            raise RuntimeError("reference generate failed")
        return out[:n].copy(), dict(prefill_s=tp.value, decode_s=td.value, head_fraction=hf.value)


def have_oracle() -> bool:
    return ORACLE_SO.exists()


def orc() -> C.CDLL:
    """The C restatement (raises if oracle/_build was not built: `make -C oracle -f oracle.mk`)."""
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            raise RuntimeError(f"{ORACLE_SO} missing: `make -C oracle -f oracle.mk`")
        L = C.CDLL(str(ORACLE_SO))
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.orc_quantize_q8.argtypes = [P, I, P, P]
        L.orc_quantize_q8.restype = None
        L.orc_matvec_q.argtypes = [I, I, I, P, P, P, I, I, P]
        L.orc_matvec_q.restype = None
        L.orc_matmul_q.argtypes = [I, I, I, P, P, P, I, I, I, P, I]
        L.orc_matmul_q.restype = None
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_model_open.argtypes = [C.c_char_p, I, C.c_char_p, I]
        L.orc_model_open.restype = P
        L.orc_model_close.argtypes = [P]
        L.orc_model_close.restype = None
        for n in ("orc_vocab", "orc_n_tokens", "orc_last_head_rows"):
            getattr(L, n).argtypes = [P]
        L.orc_forward.argtypes = [P, I, I, I, I, P, I, P]
        L.orc_forward_batch.argtypes = [P, P, I, I, I, I, P, I, P]
        L.orc_head.argtypes = [P, I, I, P, I, P, P, P]
        L.orc_sampler_new.argtypes = [F, I, F, F, F, I, C.c_ulonglong]
        L.orc_sampler_new.restype = P
        L.orc_sampler_free.argtypes = [P]
        L.orc_sampler_free.restype = None
        L.orc_sample.argtypes = [P, P, I, P, I]
        _orc = L
    return _orc


class Oracle:
    """Ops of the C restatement, same signatures as the module-level reference wrappers."""

    @staticmethod
    def quantize_q8(x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(x.size, np.int8)
        d = np.empty(x.size // QK, np.float32)
        orc().orc_quantize_q8(_p(x), x.size, _p(q), _p(d))
        return q, d

    @staticmethod
    def matvec_q(dtype, rows, cols, raw, q, d, r0=0, r1=None):
        r1 = rows if r1 is None else r1
        out = np.zeros(rows, np.float32)
        raw = np.ascontiguousarray(raw).view(np.uint8)
        orc().orc_matvec_q(dtype, rows, cols, _p(raw), _p(np.ascontiguousarray(q, np.int8)),
                           _p(np.ascontiguousarray(d, np.float32)), r0, r1, _p(out))
        return out

    @staticmethod
    def matmul_q(dtype, rows, cols, raw, q, d):
        q = np.ascontiguousarray(q, np.int8)
        n = q.shape[0]
        out = np.zeros((n, rows), np.float32)
        raw = np.ascontiguousarray(raw).view(np.uint8)
        orc().orc_matmul_q(dtype, rows, cols, _p(raw), _p(q), _p(np.ascontiguousarray(d, np.float32)), n, 0, rows, _p(out),
                           rows)
        return out


class OracleModel:
    """The C restatement's model (same interface as RefModel; single-threaded)."""

    def __init__(self, path, ctx: int = 0):
        err = C.create_string_buffer(512)
        h = orc().orc_model_open(str(path).encode(), ctx, err, 512)
        if not h:
            raise RuntimeError("oracle load failed: " + err.value.decode())
        self.h = h
        self.vocab = orc().orc_vocab(h)
        self.n_tokens = orc().orc_n_tokens(h)
        self.out = np.zeros(self.vocab, np.float32)

    def close(self):
        if getattr(self, "h", None):
            orc().orc_model_close(self.h)
            self.h = None

    __del__ = close

    def forward(self, token, pos, top_k=0, n_valid=0, must=None):
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        if orc().orc_forward(self.h, int(token), int(pos), top_k, n_valid, _p(m), m.size, _p(self.out)) != 0:
            raise IndexError("oracle forward failed")
        return self.out.copy()

    def forward_batch(self, tokens, pos0, top_k=0, n_valid=0, must=None):
        t = np.ascontiguousarray(tokens, np.int32)
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        if orc().orc_forward_batch(self.h, _p(t), t.size, int(pos0), top_k, n_valid, _p(m), m.size, _p(self.out)) != 0:
            raise IndexError("oracle forward_batch failed")
        return self.out.copy()

    def head(self, top_k=0, n_valid=0, must=None, want_bounds=False):
        m = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
        coarse = np.zeros(self.vocab, np.float32) if want_bounds else None
        upper = np.zeros(self.vocab, np.float32) if want_bounds else None
        rows = orc().orc_head(self.h, top_k, n_valid, _p(m), m.size, _p(self.out), _p(coarse), _p(upper))
        if want_bounds:
            return self.out.copy(), coarse, upper, rows
        return self.out.copy()

    @property
    def last_head_rows(self):
        return orc().orc_last_head_rows(self.h)


class OracleSampler:
    def __init__(self, temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=1234):
        self.h = orc().orc_sampler_new(temperature, top_k, top_p, min_p, repeat_penalty, repeat_window, seed)

    def sample(self, logits, n_valid, history) -> int:
        lg = np.ascontiguousarray(logits, np.float32).copy()
        h = np.ascontiguousarray(history, np.int32)
        return orc().orc_sample(self.h, _p(lg), n_valid, _p(h), h.size)

    def __del__(self):
        if getattr(self, "h", None):
            orc().orc_sampler_free(self.h)
            self.h = None


class Sampler:
    def __init__(self, temperature=0.7, top_k=20, top_p=0.8, min_p=0.0, repeat_penalty=1.1, repeat_window=0, seed=1234):
        self.h = ref().ref_sampler_new(temperature, top_k, top_p, min_p, repeat_penalty, repeat_window, seed)

    def sample(self, logits: np.ndarray, n_valid: int, history) -> int:
        lg = np.ascontiguousarray(logits, np.float32).copy()
        h = np.ascontiguousarray(history, np.int32)
        tok = ref().ref_sample(self.h, _p(lg), n_valid, _p(h), h.size)
        self.last_logits = lg  # the reference edits its logits in place (the penalised ids)
        return tok

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_sampler_free(self.h)
            self.h = None
