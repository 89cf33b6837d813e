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


def test_truncated_and_corrupt_files_fail_to_open(qb, models, tmp_path):
    src = models("tiny_q4sl").read_bytes()
    lib = qb.lib()
    h = C.c_void_p()
    bad_magic = tmp_path / "bad.qnt"
    bad_magic.write_bytes(b"XXXX" + src[4:])
    assert lib.qnt_model_open(str(bad_magic).encode(), 0, 0, C.byref(h)) < 0
    assert b"magic" in lib.qnt_last_error()
    trunc = tmp_path / "trunc.qnt"
    trunc.write_bytes(src[: len(src) // 2])
    assert lib.qnt_model_open(str(trunc).encode(), 0, 0, C.byref(h)) < 0
    msg = lib.qnt_last_error()
    assert b"bounds" in msg or b"truncated" in msg
