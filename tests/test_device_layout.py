"""The pre-packed device layout (qnt_export_device_layout): the exported copy keeps every original tensor byte for
byte, its b200.* tensors are the original rows in the device's fused order, and the reference (oracle/_ref) and the C
restatement read the copy with the same logits as the original.  CPU only; the GPU side is in
test_gpu_device_layout.py."""
import struct
from pathlib import Path

import numpy as np
import pytest

import ref as R

need_ref = pytest.mark.skipif(not R.have_ref(), reason="reference not built (oracle/_ref)")
QK = 32


def read_qnt(path):
    """name -> (dtype, rank, rows, cols, bytes) from a .qnt's directory (the format of scripts/export.py:290-315)."""
    b = Path(path).read_bytes()
    assert b[:4] == b"QNT1"
    (ver,) = struct.unpack_from("<I", b, 4)
    at = 8 + 4 * 12 + (4 if ver >= 2 else 0)  # twelve v1 header fields, `flags` from v2
    (tl,) = struct.unpack_from("<I", b, at)
    at += 4 + tl
    (n,) = struct.unpack_from("<I", b, at)
    at += 4
    out, order = {}, []
    for _ in range(n):
        (ln,) = struct.unpack_from("<I", b, at)
        name = b[at + 4:at + 4 + ln].decode()
        at += 4 + ln
        dtype, rank = struct.unpack_from("<II", b, at)
        at += 8
        dims = struct.unpack_from(f"<{rank}I", b, at)
        at += 4 * rank
        (off,) = struct.unpack_from("<Q", b, at)
        at += 8
        rows, cols = (1, dims[0]) if rank == 1 else dims
        per = {0: 4 * cols, 1: 2 * cols, 2: cols + cols // QK * 2, 3: cols // 2 + cols // QK * 2}[dtype]
        out[name] = (dtype, rank, rows, cols, b[off:off + rows * per], off)
        order.append(name)
    return out, order


def split_rows(t):
    """(quants [rows, bytes], scales [rows, blocks * 2]) of a quantized tensor's bytes."""
    dtype, _, rows, cols, raw, _ = t
    qb = cols if dtype == 2 else cols // 2
    a = np.frombuffer(raw, np.uint8)
    return a[:rows * qb].reshape(rows, qb), a[rows * qb:].reshape(rows, cols // QK * 2)


def qkv_order(rows_per_part, head_dim):
    """(part, row) per fused q|k|v row: each head's rows i and i + head_dim / 2 adjacent."""
    half = head_dim // 2
    return [(p, u * head_dim + i + s) for p, r in enumerate(rows_per_part) for u in range(r // head_dim)
            for i in range(half) for s in (0, half)]


@pytest.fixture(scope="module")
def exported(models, qb, tmp_path_factory):
    d = tmp_path_factory.mktemp("layout")
    made = {}

    def get(name):
        if name not in made:
            made[name] = qb.export_device_layout(models(name), d / f"{name}.b200.qnt")
        return made[name]

    return get


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl"])
def test_export_keeps_originals_and_adds_fused_rows(models, exported, name):
    src, order = read_qnt(models(name))
    dst, dorder = read_qnt(exported(name))
    assert dorder[:len(order)] == order  # originals first, in their order
    for k, t in src.items():
        assert dst[k][:5] == t[:5], k  # same dtype, rank, shape and bytes
        assert dst[k][5] % 64 == 0
    assert dst["b200.layout"][0] == 0 and np.frombuffer(dst["b200.layout"][4], np.float32)[0] == 1.0
    n_layers = sum(1 for k in src if k.endswith("self_attn.q_proj.weight"))
    hd = 64
    added = {k for k in dst if k.startswith("b200.layers.")}
    assert len(added) == 3 * n_layers
    for l in range(n_layers):
        p = f"model.layers.{l}."
        parts = [src[p + f"self_attn.{x}_proj.weight"] for x in "qkv"]
        fused = dst[f"b200.layers.{l}.qkv"]
        assert fused[0] == parts[0][0] and fused[2] == sum(t[2] for t in parts) and fused[3] == parts[0][3]
        fq, fd = split_rows(fused)
        pq, pd = zip(*(split_rows(t) for t in parts))
        for r, (pi, sr) in enumerate(qkv_order([t[2] for t in parts], hd)):
            assert np.array_equal(fq[r], pq[pi][sr]) and np.array_equal(fd[r], pd[pi][sr]), (l, r)
        biases = [np.frombuffer(src[p + f"self_attn.{x}_proj.bias"][4], np.float32) for x in "qkv"]
        fb = np.frombuffer(dst[f"b200.layers.{l}.qkv_bias"][4], np.float32)
        want = np.array([biases[pi][sr] for pi, sr in qkv_order([b.size for b in biases], hd)], np.float32)
        assert np.array_equal(fb.view(np.uint32), want.view(np.uint32))
        g, u = (split_rows(src[p + f"mlp.{x}_proj.weight"]) for x in ("gate", "up"))
        gq, gd = split_rows(dst[f"b200.layers.{l}.gate_up"])
        for j in range(g[0].shape[0] // QK):
            blk = slice(j * QK, (j + 1) * QK)
            assert np.array_equal(gq[2 * j * QK:(2 * j + 1) * QK], g[0][blk])
            assert np.array_equal(gq[(2 * j + 1) * QK:(2 * j + 2) * QK], u[0][blk])
            assert np.array_equal(gd[2 * j * QK:(2 * j + 1) * QK], g[1][blk])
            assert np.array_equal(gd[(2 * j + 1) * QK:(2 * j + 2) * QK], u[1][blk])


def test_export_is_idempotent_and_rejects_bad_paths(qb, models, exported, tmp_path):
    again = qb.export_device_layout(exported("tiny_q8"), tmp_path / "again.qnt")
    assert again.read_bytes() == exported("tiny_q8").read_bytes()  # the b200.* tensors are rebuilt, not doubled
    with pytest.raises(qb.QntError) as e:
        qb.export_device_layout(tmp_path / "missing.qnt", tmp_path / "x.qnt")
    assert e.value.code == -3
    with pytest.raises(qb.QntError):
        qb.export_device_layout(models("tiny_q8"), models("tiny_q8"))
    before = models("tiny_q8").read_bytes()
    alias = tmp_path / "alias.qnt"  # the same file under another name: refused, the input untouched
    alias.symlink_to(models("tiny_q8"))
    with pytest.raises(qb.QntError):
        qb.export_device_layout(models("tiny_q8"), alias)
    assert models("tiny_q8").read_bytes() == before
    with pytest.raises(qb.QntError):
        qb.export_device_layout(models("tiny_q8"), tmp_path / "no_such_dir" / "x.qnt")


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl"])
def test_restatement_reads_exported_file_unchanged(models, exported, name):
    a, b = R.OracleModel(models(name)), R.OracleModel(exported(name))
    ids = np.random.default_rng(5).integers(0, a.vocab, 12)
    for p, t in enumerate(ids):
        assert np.array_equal(a.forward(t, p), b.forward(t, p)), p


@need_ref
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl"])
def test_reference_reads_exported_file_unchanged(models, exported, name):
    a, b = R.RefModel(models(name), threads=2), R.RefModel(exported(name), threads=2)
    ids = np.random.default_rng(6).integers(0, a.vocab, 12)
    for p, t in enumerate(ids):
        assert np.array_equal(a.forward(t, p), b.forward(t, p)), p
    nv = a.n_tokens
    assert np.array_equal(a.head(top_k=20, n_valid=nv), b.head(top_k=20, n_valid=nv))


def test_cli_export_layout_writes_the_same_file(qb, models, exported, tmp_path):
    """`quanta_b200 export-layout IN OUT` (host code only, no GPU) writes the same bytes as the C ABI entry."""
    import subprocess
    cli = Path(qb.__file__).resolve().parent / "lib" / "quanta_b200"
    out = tmp_path / "cli.qnt"
    r = subprocess.run([str(cli), "export-layout", str(models("tiny_q8")), str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert out.read_bytes() == exported("tiny_q8").read_bytes()
    r = subprocess.run([str(cli), "export-layout", str(tmp_path / "missing.qnt"), str(tmp_path / "y.qnt")],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "export-layout:" in r.stderr
