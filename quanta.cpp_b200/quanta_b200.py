"""Python host mirror of the engine's C ABI (include/quanta_b200.h), via ctypes.

The names follow the reference's C++ interface (engine/src/model.h, ops.h, sampler.h, session.h):
    Model(path, ctx).forward(token, pos, hq) / forward_batch(tokens, pos0, hq) / head(hq) / last_head_rows
    quantize_q8(x) ; DeviceTensor(dtype, rows, cols, raw).matvec(q, d, r0, r1) / .matmul(...)
    Model.generate(prompt, SamplerParams(...), shortlist=True, batch_prefill=True, n_gen=64)
    synth_model(path, ...)  seeded random-init .qnt writer
There is no CPU fallback: importing works anywhere, but every call needs libquanta_b200.so and a GPU, and fails
loudly when either is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_DIR = Path(os.environ["QNT_LIB_DIR"]) if os.environ.get("QNT_LIB_DIR") else PKG / "lib"  # timeline.py: lib_stamps

F32, F16, Q8_0, Q4_0 = 0, 1, 2, 3
QK = 32
GEN_SHORTLIST, GEN_BATCH_PREFILL = 1, 2


class QntError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"quanta_b200 error {code}: {msg}")
        self.code = code


class HeadQuery(C.Structure):
    _fields_ = [("top_k", C.c_int), ("n_valid", C.c_int), ("must", C.POINTER(C.c_int)), ("n_must", C.c_int)]


class HParams(C.Structure):
    _fields_ = [(n, C.c_int) for n in "vocab_size dim n_layers n_heads n_kv_heads head_dim ffn_dim max_seq".split()] + [
        ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("tied_embeddings", C.c_int), ("qkv_bias", C.c_int),
        ("flags", C.c_uint32), ("n_tokens", C.c_int), ("ctx_len", C.c_int), ("has_shortlist", C.c_int)]


class SamplerParamsC(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_window", C.c_int), ("seed", C.c_uint64)]


class GenStatsC(C.Structure):
    _fields_ = [("prefill_ms", C.c_double), ("decode_ms", C.c_double), ("head_rows", C.c_longlong),
                ("head_calls", C.c_longlong), ("kernels_per_step", C.c_int)]


class SynthCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in "vocab_size dim n_layers n_heads n_kv_heads head_dim ffn_dim max_seq".split()] + [
        ("rope_theta", C.c_float), ("norm_eps", C.c_float)] + [(n, C.c_int) for n in "mlp_q4 q4_group shortlist n_tokens".split()] + [
        ("w_std", C.c_float), ("seed", C.c_uint64), ("n_threads", C.c_int), ("flags", C.c_uint32),
        ("tok_blob", C.c_char_p), ("tok_len", C.c_uint64)]


@dataclass
class SamplerParams:
    """engine/src/sampler.h:9-18 defaults (Qwen2.5-Instruct generation config)."""
    temperature: float = 0.7
    top_k: int = 20
    top_p: float = 0.8
    min_p: float = 0.0
    repeat_penalty: float = 1.1
    repeat_window: int = 0
    seed: int = 0


_lib = None
_synth = None


def lib_path() -> Path:
    return LIB_DIR / "libquanta_b200.so"


def lib() -> C.CDLL:
    """Loads libquanta_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        p = lib_path()
        if not p.exists():
            raise RuntimeError(f"{p} is missing: run `python quanta.cpp_b200/build.py` (nvcc, sm_100a)")
        L = C.CDLL(str(p))
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.qnt_last_error.restype = C.c_char_p
        L.qnt_tensor_upload.argtypes = [I, I, I, P, C.POINTER(P)]
        L.qnt_tensor_free.argtypes = [P]
        L.qnt_quantize_q8.argtypes = [P, I, I, P, P, P]
        L.qnt_matvec.argtypes = [P, P, P, I, I, P, P]
        L.qnt_matmul.argtypes = [P, P, P, I, I, I, P, I, I, P]
        L.qnt_ops_check.argtypes = [P]
        L.qnt_quantize_q8_host.argtypes = [P, I, P, P]
        L.qnt_matvec_host.argtypes = [P, P, P, I, I, P]
        L.qnt_matmul_host.argtypes = [P, P, P, I, I, I, P, I, I]
        L.qnt_model_open.argtypes = [C.c_char_p, I, I, C.POINTER(P)]
        L.qnt_model_close.argtypes = [P]
        L.qnt_model_close.restype = None
        L.qnt_model_hparams.argtypes = [P, C.POINTER(HParams)]
        L.qnt_model_forward.argtypes = [P, I, I, C.POINTER(HeadQuery), P]
        L.qnt_model_forward_batch.argtypes = [P, P, I, I, C.POINTER(HeadQuery), P]
        L.qnt_model_head.argtypes = [P, C.POINTER(HeadQuery), P, P, P]
        L.qnt_model_last_head_rows.argtypes = [P]
        L.qnt_model_has_shortlist.argtypes = [P]
        L.qnt_model_kv_cache_bytes.argtypes = [P]
        L.qnt_model_kv_cache_bytes.restype = C.c_size_t
        L.qnt_model_weight_bytes.argtypes = [P]
        L.qnt_model_weight_bytes.restype = C.c_size_t
        L.qnt_export_device_layout.argtypes = [C.c_char_p, C.c_char_p]
        L.qnt_model_packed_tensors.argtypes = [P]
        L.qnt_generate.argtypes = [P, P, I, C.POINTER(SamplerParamsC), I, I, P, C.POINTER(GenStatsC)]
        L.qnt_set_device.argtypes = [I]
        L.qnt_session_begin.argtypes = [P, P, I, C.POINTER(SamplerParamsC), I]
        L.qnt_session_step.argtypes = [P, I]
        L.qnt_session_read.argtypes = [P, P, I, C.POINTER(GenStatsC)]
        L.qnt_model_stream.argtypes = [P]
        L.qnt_model_stream.restype = P
        L.qnt_batch_init.argtypes = [P, I, I]
        L.qnt_prefill_batch.argtypes = [P, I, P, I, C.POINTER(I)]
        L.qnt_decode_batch.argtypes = [P, P, P, I, P]
        L.qnt_batch_reset.argtypes = [P, I]
        L.qnt_sampler_create.argtypes = [C.POINTER(SamplerParamsC), C.POINTER(P)]
        L.qnt_sampler_sample.argtypes = [P, P, I, P, I, C.POINTER(I), P]
        L.qnt_sampler_free.argtypes = [P]
        L.qnt_sampler_free.restype = None
        L.qnt_bench_mma_i8.argtypes = [I, C.POINTER(C.c_double)]
        L.qnt_wait_probe.argtypes = [C.c_uint, P]
        L.qnt_session_feed.argtypes = [P, P, I]
        L.qnt_model_nll.argtypes = [P, P, I, C.POINTER(C.c_double)]
        L.qnt_session_rewind.argtypes = [P, I]
        L.qnt_session_last.argtypes = [P, C.POINTER(I), C.POINTER(I)]
        L.qnt_tokenizer_open.argtypes = [C.c_char_p, C.POINTER(P)]
        L.qnt_tokenizer_free.argtypes = [P]
        L.qnt_tokenizer_free.restype = None
        L.qnt_tokenizer_n_tokens.argtypes = [P]
        L.qnt_tokenize.argtypes = [P, C.c_char_p, C.c_size_t, P, I]
        L.qnt_token_piece.argtypes = [P, I, C.c_char_p, I]
        L.qnt_token_id.argtypes = [P, C.c_char_p]
        L.qnt_sampler_sample_noalloc.argtypes = [C.POINTER(SamplerParamsC), C.POINTER(C.c_uint64), P, I, P, I,
                                                 C.POINTER(I), P]
        _lib = L
    return _lib


def _check(rc: int) -> int:
    if rc < 0:
        raise QntError(rc, lib().qnt_last_error().decode(errors="replace"))
    return rc


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def exported_symbols() -> list[str]:
    """Every function declared in include/quanta_b200.h."""
    import re
    hdr = (PKG.parent / "include" / "quanta_b200.h").read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(qnt_\w+)\s*\(", hdr, re.M)))


def device_count() -> int:
    return lib().qnt_device_count()


def set_device(d: int) -> None:
    _check(lib().qnt_set_device(d))


# ---------------------------------------------------------------- ops level

def quantize_q8(x: np.ndarray):
    """quantize_q8 (engine/src/ops_ref.cpp:69-83) on the device: returns (q int8[n], d f32[n/32])."""
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // QK, np.float32)
    _check(lib().qnt_quantize_q8_host(_ptr(x), x.size, _ptr(q), _ptr(d)))
    return q, d


class DeviceTensor:
    """A quantized matrix in HBM (the .qnt byte layout in, device copy inside)."""

    def __init__(self, dtype: int, rows: int, cols: int, raw: np.ndarray | bytes):
        buf = np.frombuffer(raw, np.uint8) if isinstance(raw, (bytes, bytearray)) else np.ascontiguousarray(raw).view(np.uint8)
        self.dtype, self.rows, self.cols = dtype, rows, cols
        self._buf = buf
        h = C.c_void_p()
        _check(lib().qnt_tensor_upload(dtype, rows, cols, _ptr(buf), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.qnt_tensor_free(self.h)
        self.h = None

    __del__ = close

    def matvec(self, q: np.ndarray, d: np.ndarray, r0: int = 0, r1: int | None = None) -> np.ndarray:
        r1 = self.rows if r1 is None else r1
        out = np.zeros(self.rows, np.float32)
        _check(lib().qnt_matvec_host(self.h, _ptr(np.ascontiguousarray(q, np.int8)), _ptr(np.ascontiguousarray(d, np.float32)),
                                     r0, r1, _ptr(out)))
        return out

    def matmul(self, q: np.ndarray, d: np.ndarray, r0: int = 0, r1: int | None = None, impl: int = 0) -> np.ndarray:
        """q [n][cols] int8, d [n][cols/32] -> out [n][rows] (rows outside [r0, r1) are 0)."""
        r1 = self.rows if r1 is None else r1
        q = np.ascontiguousarray(q, np.int8)
        n = q.shape[0]
        out = np.zeros((n, self.rows), np.float32)
        _check(lib().qnt_matmul_host(self.h, _ptr(q), _ptr(np.ascontiguousarray(d, np.float32)), n, r0, r1, _ptr(out),
                                     self.rows, impl))
        return out



class Sampler:
    """Sampler (engine/src/sampler.h:20-38) on the device: sample(logits, n_valid, history) -> id, as
    Sampler::sample (sampler.cpp:22-85).  `logits` is a float32 CUDA tensor (torch) on the current device and is edited
    in place like the reference's array; `history` is a sequence of ids."""

    def __init__(self, sp: SamplerParams):
        spc = SamplerParamsC(sp.temperature, sp.top_k, sp.top_p, sp.min_p, sp.repeat_penalty, sp.repeat_window, sp.seed)
        h = C.c_void_p()
        _check(lib().qnt_sampler_create(C.byref(spc), C.byref(h)))
        self.h = h
        self.params = sp

    def sample(self, logits, n_valid: int | None = None, history=(), stream=None) -> int:
        if not (getattr(logits, "is_cuda", False) and str(logits.dtype) == "torch.float32" and logits.is_contiguous()):
            raise TypeError("logits must be a contiguous float32 CUDA tensor")
        n_valid = logits.numel() if n_valid is None else n_valid
        hist = np.ascontiguousarray(np.asarray(history, np.int32).ravel())
        tok = C.c_int(-1)
        st = None if stream is None else C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))
        _check(lib().qnt_sampler_sample(self.h, C.c_void_p(logits.data_ptr()), n_valid, _ptr(hist) if hist.size else None,
                                        hist.size, C.byref(tok), st))
        return tok.value

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.qnt_sampler_free(self.h)
        self.h = None

    __del__ = close


def sample_noalloc(sp: SamplerParams, rng_state: int, logits, n_valid: int | None = None, history=(), stream=None):
    """qnt_sampler_sample_noalloc: the Sampler without an object and without allocating (static device scratch).
    rng_state is the xorshift64* state ((seed or any nonzero) | 1 to start); returns (id, next rng_state)."""
    if not (getattr(logits, "is_cuda", False) and str(logits.dtype) == "torch.float32" and logits.is_contiguous()):
        raise TypeError("logits must be a contiguous float32 CUDA tensor")
    n_valid = logits.numel() if n_valid is None else n_valid
    spc = SamplerParamsC(sp.temperature, sp.top_k, sp.top_p, sp.min_p, sp.repeat_penalty, sp.repeat_window, sp.seed)
    hist = np.ascontiguousarray(np.asarray(history, np.int32).ravel())
    state = C.c_uint64(rng_state)
    tok = C.c_int(-1)
    st = None if stream is None else C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))
    _check(lib().qnt_sampler_sample_noalloc(C.byref(spc), C.byref(state), C.c_void_p(logits.data_ptr()), n_valid,
                                            _ptr(hist) if hist.size else None, hist.size, C.byref(tok), st))
    return tok.value, state.value

def bench_mma_i8(iters: int = 4096) -> float:
    """Measured dense int8 tensor-core TOP/s of the current GPU (qnt_bench_mma_i8)."""
    v = C.c_double(0)
    _check(lib().qnt_bench_mma_i8(iters, C.byref(v)))
    return v.value

class Tokenizer:
    """Tokenizer (engine/src/tokenizer.h:15-39) of a .qnt file, on the host: encode(text) -> ids, decode(id) -> bytes,
    token_id(literal) -> special id or -1."""

    def __init__(self, path):
        h = C.c_void_p()
        _check(lib().qnt_tokenizer_open(str(path).encode(), C.byref(h)))
        self.h = h
        self.n_tokens = lib().qnt_tokenizer_n_tokens(h)

    def encode(self, text) -> np.ndarray:
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = _check(lib().qnt_tokenize(self.h, b, len(b), None, 0))
        out = np.zeros(max(n, 1), np.int32)
        _check(lib().qnt_tokenize(self.h, b, len(b), _ptr(out), n))
        return out[:n]

    def decode(self, ids) -> bytes:
        if np.isscalar(ids):
            ids = [ids]
        parts = []
        for i in ids:
            n = _check(lib().qnt_token_piece(self.h, int(i), None, 0))
            buf = C.create_string_buffer(max(n, 1))
            lib().qnt_token_piece(self.h, int(i), buf, n)
            parts.append(buf.raw[:n])
        return b"".join(parts)

    def token_id(self, literal: str) -> int:
        return lib().qnt_token_id(self.h, literal.encode())

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.qnt_tokenizer_free(self.h)
        self.h = None

    __del__ = close

# ---------------------------------------------------------------- model level

def head_query(top_k=0, n_valid=0, must=None):
    must_arr = np.ascontiguousarray(must if must is not None else np.zeros(0), np.int32)
    hq = HeadQuery(top_k, n_valid, must_arr.ctypes.data_as(C.POINTER(C.c_int)), must_arr.size)
    hq._keep = must_arr
    return hq


class Model:
    """quanta::Model on the device (engine/src/model.h)."""

    def __init__(self, path: str | os.PathLike, ctx_len: int = 0, nibble_screen: bool = False):
        """nibble_screen: QNT_OPEN_NIBBLE_SCREEN (the shortlist head screens with the Q8 head's high nibble plane)."""
        h = C.c_void_p()
        _check(lib().qnt_model_open(str(path).encode(), ctx_len, 1 if nibble_screen else 0, C.byref(h)))
        self.h = h
        hp = HParams()
        _check(lib().qnt_model_hparams(h, C.byref(hp)))
        self.hp = hp
        self.vocab = hp.vocab_size
        self._logits = np.zeros(self.vocab, np.float32)

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.qnt_model_close(self.h)
        self.h = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @staticmethod
    def _hq(hq):
        if hq is None:
            return None
        if isinstance(hq, HeadQuery):
            return C.byref(hq)
        return C.byref(head_query(**hq)) if isinstance(hq, dict) else hq

    def forward(self, token: int, pos: int, hq=None, copy: bool = True) -> np.ndarray | None:
        hqs = head_query(**hq) if isinstance(hq, dict) else hq
        _check(lib().qnt_model_forward(self.h, int(token), int(pos), C.byref(hqs) if hqs is not None else None,
                                       _ptr(self._logits) if copy else None))
        return self._logits.copy() if copy else None

    def forward_batch(self, tokens, pos0: int, hq=None, copy: bool = True) -> np.ndarray | None:
        t = np.ascontiguousarray(tokens, np.int32)
        hqs = head_query(**hq) if isinstance(hq, dict) else hq
        _check(lib().qnt_model_forward_batch(self.h, _ptr(t), t.size, int(pos0), C.byref(hqs) if hqs is not None else None,
                                             _ptr(self._logits) if copy else None))
        return self._logits.copy() if copy else None

    def head(self, hq=None, want_bounds: bool = False):
        hqs = head_query(**hq) if isinstance(hq, dict) else hq
        coarse = np.zeros(self.vocab, np.float32) if want_bounds else None
        upper = np.zeros(self.vocab, np.float32) if want_bounds else None
        _check(lib().qnt_model_head(self.h, C.byref(hqs) if hqs is not None else None, _ptr(self._logits), _ptr(coarse),
                                    _ptr(upper)))
        if want_bounds:
            return self._logits.copy(), coarse, upper
        return self._logits.copy()

    def nll(self, ids) -> float:
        """Sum over p of -log softmax(logits after ids[:p+1])[ids[p+1]] (the CLI's ppl); perplexity = exp(nll/(n-1))."""
        t = np.ascontiguousarray(ids, np.int32)
        v = C.c_double(0)
        _check(lib().qnt_model_nll(self.h, _ptr(t), t.size, C.byref(v)))
        return v.value

    @property
    def last_head_rows(self) -> int:
        return lib().qnt_model_last_head_rows(self.h)

    @property
    def has_shortlist(self) -> bool:
        return bool(lib().qnt_model_has_shortlist(self.h))

    @property
    def weight_bytes(self) -> int:
        return int(lib().qnt_model_weight_bytes(self.h))

    @property
    def packed_tensors(self) -> int:
        """Fused tensors this load took pre-packed from the file (export_device_layout); 0 for a plain .qnt."""
        return int(lib().qnt_model_packed_tensors(self.h))

    def generate(self, prompt, sp: SamplerParams, n_gen: int, shortlist: bool = True, batch_prefill: bool = True):
        """Session::feed + generate with the device sampler; returns (ids, stats dict)."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(n_gen, 1), np.int32)
        spc = SamplerParamsC(sp.temperature, sp.top_k, sp.top_p, sp.min_p, sp.repeat_penalty, sp.repeat_window, sp.seed)
        st = GenStatsC()
        flags = (GEN_SHORTLIST if shortlist else 0) | (GEN_BATCH_PREFILL if batch_prefill else 0)
        n = _check(lib().qnt_generate(self.h, _ptr(p), p.size, C.byref(spc), flags, n_gen, _ptr(out), C.byref(st)))
        return out[:n].copy(), dict(prefill_ms=st.prefill_ms, decode_ms=st.decode_ms, head_rows=st.head_rows,
                                    head_calls=st.head_calls, kernels_per_step=st.kernels_per_step)


    # Session in pieces (qnt_session_begin / step / read)
    # ---- batched serving (greedy): many sequences with their own KV caches
    def batch_init(self, max_seqs: int, ctx_len: int):
        _check(lib().qnt_batch_init(self.h, max_seqs, ctx_len))

    def prefill_batch(self, seq: int, tokens) -> int:
        """Feeds the prompt of one sequence; returns its greedy next token."""
        t = np.ascontiguousarray(tokens, np.int32)
        nxt = C.c_int(-1)
        _check(lib().qnt_prefill_batch(self.h, seq, _ptr(t), t.size, C.byref(nxt)))
        return nxt.value

    def decode_batch(self, seq_ids, tokens) -> np.ndarray:
        """One greedy step of several distinct sequences; returns their next tokens."""
        s = np.ascontiguousarray(seq_ids, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(s.size, np.int32)
        _check(lib().qnt_decode_batch(self.h, _ptr(s), _ptr(t), s.size, _ptr(out)))
        return out

    def batch_reset(self, seq: int):
        _check(lib().qnt_batch_reset(self.h, seq))

    def session_begin(self, prompt, sp: SamplerParams, shortlist: bool = True, batch_prefill: bool = True):
        p = np.ascontiguousarray(prompt, np.int32)
        spc = SamplerParamsC(sp.temperature, sp.top_k, sp.top_p, sp.min_p, sp.repeat_penalty, sp.repeat_window, sp.seed)
        flags = (GEN_SHORTLIST if shortlist else 0) | (GEN_BATCH_PREFILL if batch_prefill else 0)
        _check(lib().qnt_session_begin(self.h, _ptr(p), p.size, C.byref(spc), flags))

    def session_step(self, n: int) -> int:
        return _check(lib().qnt_session_step(self.h, n))

    def session_feed(self, ids):
        t = np.ascontiguousarray(ids, np.int32)
        _check(lib().qnt_session_feed(self.h, _ptr(t), t.size))

    def session_rewind(self, n_drop: int):
        _check(lib().qnt_session_rewind(self.h, n_drop))

    def session_last(self):
        """(last sampled id, history length) after the queued steps."""
        tok, n = C.c_int(-1), C.c_int(0)
        _check(lib().qnt_session_last(self.h, C.byref(tok), C.byref(n)))
        return tok.value, n.value

    def session_read(self, max_ids: int = 1 << 16):
        out = np.zeros(max(max_ids, 1), np.int32)
        st = GenStatsC()
        n = _check(lib().qnt_session_read(self.h, _ptr(out), max_ids, C.byref(st)))
        return out[:n].copy(), dict(head_rows=st.head_rows, head_calls=st.head_calls, kernels_per_step=st.kernels_per_step)

    @property
    def stream(self) -> int:
        return int(lib().qnt_model_stream(self.h) or 0)


# ---------------------------------------------------------------- synthetic models

QWEN05B = dict(vocab_size=151936, dim=896, n_layers=24, n_heads=14, n_kv_heads=2, head_dim=64, ffn_dim=4864, max_seq=4096,
               rope_theta=1e6, norm_eps=1e-6, n_tokens=151665)
TINY = dict(vocab_size=5000, dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, max_seq=512,
            rope_theta=1e6, norm_eps=1e-6, n_tokens=4900)


def export_device_layout(src, dst) -> Path:
    """A copy of the .qnt at src, written to dst, with the device's fused q|k|v, gate|up and q|k|v-bias tensors stored
    pre-packed beside the original ones (which stay byte for byte, so the reference reads the copy unchanged).  No
    GPU needed."""
    _check(lib().qnt_export_device_layout(str(src).encode(), str(dst).encode()))
    return Path(dst)


def synth_model(path, *, shape: dict = QWEN05B, mlp_q4: bool = True, shortlist: bool = True, q4_group: int = 128,
                seed: int = 1234, w_std: float = 0.02, threads: int = 0, overwrite: bool = False, flags: int = 0,
                tokenizer: bytes | None = None) -> Path:
    """Writes a seeded random-init .qnt (q4mix = attention Q8_0 + MLP GPTQ-sym int4; or all Q8_0); flags = the header
    flags (1: FLAG_HADAMARD_DOWN); tokenizer = a complete tokenizer section (its token count must be shape's n_tokens)
    instead of the synthetic byte vocabulary."""
    global _synth
    path = Path(path)
    if path.exists() and not overwrite:
        return path
    if _synth is None:
        p = PKG / "lib" / "libqnt_synth.so"  # the model writer is not part of the phase-timed build
        if not p.exists():
            raise RuntimeError(f"{p} is missing: run `python quanta.cpp_b200/build.py`")
        _synth = C.CDLL(str(p))
        _synth.qnt_synth_write.argtypes = [C.c_char_p, C.POINTER(SynthCfg)]
        _synth.qnt_synth_last_error.restype = C.c_char_p
    cfg = SynthCfg(**{k: shape[k] for k in ("vocab_size", "dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim",
                                             "max_seq", "rope_theta", "norm_eps", "n_tokens")},
                   mlp_q4=int(mlp_q4), q4_group=q4_group, shortlist=int(shortlist), w_std=w_std, seed=seed,
                   n_threads=threads, flags=flags, tok_blob=tokenizer, tok_len=len(tokenizer) if tokenizer else 0)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + f".tmp{os.getpid()}")
    if _synth.qnt_synth_write(str(tmp).encode(), C.byref(cfg)) != 0:
        raise RuntimeError(_synth.qnt_synth_last_error().decode())
    os.replace(tmp, path)
    return path
