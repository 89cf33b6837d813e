"""A .qnt exported with the device's fused tensors pre-packed (qnt_export_device_layout) loads without the host row
reorder and gives the same results bit for bit as the original file: logits of token-by-token and batched forwards,
the shortlist head, and sampled ids.  The load times of both are printed."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def exported(models, qb, tmp_path_factory):
    d = tmp_path_factory.mktemp("layout_gpu")
    made = {}

    def get(name):
        if name not in made:
            made[name] = qb.export_device_layout(models(name), d / f"{name}.b200.qnt")
        return made[name]

    return get


def _open(qb, path, **kw):
    t = time.perf_counter()
    m = qb.Model(path, ctx_len=1024, **kw)
    return m, time.perf_counter() - t


@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4sl", "q4mix_sl"])
def test_exported_layout_loads_packed_and_matches(qb, models, exported, name):
    a, ta = _open(qb, models(name))
    b, tb = _open(qb, exported(name))
    try:
        assert a.packed_tensors == 0
        assert b.packed_tensors == 3 * a.hp.n_layers  # q|k|v, gate|up and the q|k|v bias of every layer
        assert b.weight_bytes == a.weight_bytes
        nv = a.hp.n_tokens
        prompt = np.random.default_rng(41).integers(0, nv, 96)
        assert np.array_equal(a.forward_batch(prompt, 0), b.forward_batch(prompt, 0))
        tok = 7
        for p in range(96, 104):
            la, lb = a.forward(tok, p), b.forward(tok, p)
            assert np.array_equal(la, lb), p
            tok = int(np.argmax(la[:nv]))
        if a.has_shortlist:
            hist = prompt[-32:]
            assert np.array_equal(a.head(dict(top_k=20, n_valid=nv, must=hist)), b.head(dict(top_k=20, n_valid=nv, must=hist)))
        print(f"{name}: load {ta * 1e3:.1f} ms (fused at load) vs {tb * 1e3:.1f} ms (pre-packed)")
    finally:
        a.close()
        b.close()


def test_exported_layout_samples_the_same_ids(qb, models, exported):
    sp = qb.SamplerParams(temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1, seed=5)
    prompt = np.random.default_rng(8).integers(0, 4000, 200)
    got = []
    for path in (models("q4mix_sl"), exported("q4mix_sl")):
        m = qb.Model(path, ctx_len=1024)
        try:
            ids, _ = m.generate(prompt, sp, 32)
            got.append(ids)
        finally:
            m.close()
    assert np.array_equal(got[0], got[1])


def test_exported_layout_with_nibble_screen(qb, models, exported):
    """The pre-packed tensors and the load-time nibble plane combine: same logits as the original file's."""
    a = qb.Model(models("tiny_q8"), ctx_len=512, nibble_screen=True)
    b = qb.Model(exported("tiny_q8"), ctx_len=512, nibble_screen=True)
    try:
        nv = a.hp.n_tokens
        prompt = np.random.default_rng(2).integers(0, nv, 40)
        a.forward_batch(prompt, 0)
        b.forward_batch(prompt, 0)
        q = dict(top_k=20, n_valid=nv, must=prompt[-16:])
        assert np.array_equal(a.head(q), b.head(q))
        assert a.last_head_rows == b.last_head_rows
    finally:
        a.close()
        b.close()


def test_stale_packed_tensor_is_fused_at_load(qb, models, exported, tmp_path):
    """A pre-packed matrix whose rows no longer match the file's own q|k|v (one byte changed in its first row) is not
    uploaded: the engine fuses that layer's rows itself, and the logits stay the original file's."""
    from test_device_layout import read_qnt
    src = exported("tiny_q8")
    tensors, _ = read_qnt(src)
    off = tensors["b200.layers.0.qkv"][5]
    data = bytearray(src.read_bytes())
    data[off] ^= 0x5A
    bad = tmp_path / "stale.qnt"
    bad.write_bytes(bytes(data))
    a, b = qb.Model(models("tiny_q8"), ctx_len=256), qb.Model(bad, ctx_len=256)
    try:
        assert b.packed_tensors == 3 * a.hp.n_layers - 1
        prompt = np.random.default_rng(3).integers(0, a.hp.n_tokens, 32)
        assert np.array_equal(a.forward_batch(prompt, 0), b.forward_batch(prompt, 0))
    finally:
        a.close()
        b.close()
