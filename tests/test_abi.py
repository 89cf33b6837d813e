"""CPU checks of the drop-in boundary: the C-ABI library loads and exports every symbol the header declares, and
its errors come back as status codes (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def test_library_exports_every_header_symbol(qb):
    lib = qb.lib()
    names = qb.exported_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_header_cites_reference_interfaces():
    hdr = (ROOT / "include" / "quanta_b200.h").read_text()
    # every function block comment names the reference file it replaces (engine/src/...)
    decls = re.findall(r"^\w[\w\s\*]*?\b(qnt_\w+)\s*\(", hdr, re.M)
    assert "engine/src/ops.h" in hdr and "engine/src/model.h" in hdr and "engine/src/session" in hdr
    assert len(decls) == len(set(decls))


def test_errors_are_status_codes_not_crashes(qb):
    lib = qb.lib()
    h = C.c_void_p()
    rc = lib.qnt_model_open(b"/nonexistent/model.qnt", 0, 0, C.byref(h))
    assert rc < 0
    assert lib.qnt_last_error()
    # bad shapes are rejected before touching a device
    buf = np.zeros(64, np.uint8)
    assert lib.qnt_tensor_upload(2, 1, 33, buf.ctypes.data_as(C.c_void_p), C.byref(h)) == -1
    assert lib.qnt_quantize_q8(None, 1, 33, None, None, None) == -1


def _first_entry_offsets(raw: bytes):
    """Byte offsets of the first tensor directory entry's dtype, rank and data-offset fields (.qnt layout: signature,
    version, 12 header words + flags from version 2, tokenizer length + section, tensor count, entries)."""
    import struct
    version = struct.unpack_from("<I", raw, 4)[0]
    at = 8 + 12 * 4 + (4 if version >= 2 else 0)
    tok_len = struct.unpack_from("<I", raw, at)[0]
    at += 4 + tok_len + 4  # tokenizer section, tensor count
    name_len = struct.unpack_from("<I", raw, at)[0]
    at += 4 + name_len
    dtype_at, rank_at = at, at + 4
    rank = struct.unpack_from("<I", raw, rank_at)[0]
    return dtype_at, rank_at, rank_at + 4 + 4 * rank


def _patched(raw: bytes, at: int, value: int, fmt="<I") -> bytes:
    import struct
    b = bytearray(raw)
    struct.pack_into(fmt, b, at, value)
    return bytes(b)


def test_truncated_and_corrupt_files_fail_to_open(qb, models, tmp_path):
    """Every invariant of the file format is checked on open (no GPU needed: the file is parsed before any device
    work) and reported as QNT_ERR_IO with a message naming what is wrong."""
    src = models("tiny_q4sl").read_bytes()
    lib = qb.lib()
    dtype_at, rank_at, off_at = _first_entry_offsets(src)
    cases = {
        "signature": (b"XXXX" + src[4:], b"QNT1"),
        "version": (_patched(src, 4, 3), b"version 3"),
        "zero dim": (_patched(src, 12, 0), b"'dim' = 0"),
        "short header": (src[:20], b"header"),
        "short tokenizer": (_patched(src, 8 + 13 * 4, len(src)), b"tokenizer"),
        "rank": (_patched(src, rank_at, 3), b"rank 3"),
        "dtype": (_patched(src, dtype_at, 9), b"dtype code 9"),
        "extent": (_patched(src, off_at, len(src) - 8, "<Q"), b"file ends at byte"),
        "truncated": (src[: len(src) // 2], b"file ends at byte"),
        "empty": (b"", b"empty file"),
    }
    for name, (data, needle) in cases.items():
        f = tmp_path / f"{name.replace(' ', '_')}.qnt"
        f.write_bytes(data)
        h = C.c_void_p()
        rc = lib.qnt_model_open(str(f).encode(), 0, 0, C.byref(h))
        msg = lib.qnt_last_error()
        assert rc == -3, (name, rc, msg)  # QNT_ERR_IO
        assert needle in msg, (name, msg)
    h = C.c_void_p()
    assert lib.qnt_model_open(str(tmp_path / "absent.qnt").encode(), 0, 0, C.byref(h)) == -3
    assert b"cannot read model file" in lib.qnt_last_error()
