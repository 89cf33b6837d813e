"""Ops-level parity on the GPU, through the C ABI, against the reference's own scalar kernels (oracle/_ref).

Q8_0 x Q8_0 matvec 4864x896, N(0,0.02) weights, N(0,1) activation: int32 block sums exact and
the f32 output bit-identical to matvec_q_ref (stricter than the 1e-5 relative the spec asks).
GPTQ-sym int4 (g128) gate/up 4864x896 and down 896x4864 at M=1 and M=32, and 4096 rows checked
as 128 chunks of 32 bit-identical to 32 separate M=1 calls (the invariant of checks.cpp:113-130).
Also the reference's own selftest fixture (xorshift bytes, scales 0x2000-0x27FF, checks.cpp:64-89).
"""
import numpy as np
import pytest

import ref as R

pytestmark = pytest.mark.gpu
Q8, Q4 = 2, 3


def q8_weights(rng, rows, cols, std=0.02):
    """Q8_0 bytes of N(0, std) weights (scripts/export.py:84-90 quantizer)."""
    w = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
    b = w.reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    inv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.round(b * inv[:, None]), -127, 127).astype(np.int8)
    return np.concatenate([q.view(np.uint8).ravel(), d.astype(np.float16).view(np.uint8)])


def q4_gptq_weights(rng, rows, cols, std=0.02, group=128):
    """GPTQ-sym int4: codes uniform in [-8, 7], one fp16 scale per `group` columns replicated per 32-block."""
    codes = rng.integers(-8, 8, size=(rows, cols)).astype(np.int16)
    qi = (codes + 8).astype(np.uint8).reshape(-1, 32)
    packed = ((qi[:, :16] & 0xF) | (qi[:, 16:] << 4)).astype(np.uint8)
    base = std / np.sqrt(255 / 12)
    sg = (base * rng.uniform(0.75, 1.25, size=(rows, cols // group))).astype(np.float16)
    d = np.repeat(sg, group // 32, axis=1)
    return np.concatenate([packed.ravel(), d.view(np.uint8).ravel()])


def selftest_fixture(dt):
    """engine/src/checks.cpp:64-89: xorshift64 quant bytes, fp16 scales 0x2000 + r % 0x800, x in [-1, 1] step 1e-3."""
    rows, cols = 4864, 896
    state = [0x9E3779B97F4A7C15]
    M = (1 << 64) - 1

    def nxt():
        s = state[0]
        s ^= (s << 13) & M
        s ^= s >> 7
        s ^= (s << 17) & M
        state[0] = s
        return s

    qbytes = rows * cols if dt == Q8 else rows * cols // 2
    buf = np.empty(qbytes + rows * cols // 32 * 2, np.uint8)
    buf[:qbytes] = np.fromiter((nxt() & 0xFF for _ in range(qbytes)), np.uint8, qbytes)
    sc = np.fromiter((0x2000 + nxt() % 0x800 for _ in range(rows * cols // 32)), np.uint16, rows * cols // 32)
    buf[qbytes:] = sc.view(np.uint8)
    x = np.array([float(int(nxt() % 2001) - 1000) / 1000.0 for _ in range(cols)], np.float32)
    return buf, x


def block_sums(dtype, raw, rows, cols, q):
    """Exact int32 per-block sums (the integer half of matvec_q_ref)."""
    nb = cols // 32
    if dtype == Q8:
        w = raw[: rows * cols].view(np.int8).reshape(rows, nb, 32).astype(np.int32)
    else:
        p = raw[: rows * cols // 2].reshape(rows, nb, 16)
        w = np.concatenate([(p & 0xF).astype(np.int32) - 8, (p >> 4).astype(np.int32) - 8], axis=2)
    return np.einsum("rbi,bi->rb", w, q.reshape(nb, 32).astype(np.int32))


def test_quantize_q8_bit_exact(qb):
    rng = np.random.default_rng(1)
    for n in (32, 896, 4864):
        x = rng.standard_normal(n).astype(np.float32)
        x[:32] *= 0  # an all-zero block (d = 0, inv = 0)
        q, d = qb.quantize_q8(x)
        rq, rd = R.quantize_q8(x)
        assert np.array_equal(q, rq) and np.array_equal(d.view(np.uint32), rd.view(np.uint32))


def test_config1_q8_matvec_bit_exact(qb):
    rng = np.random.default_rng(1234)
    rows, cols = 4864, 896
    raw = q8_weights(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    q, d = R.quantize_q8(x)
    W = qb.DeviceTensor(Q8, rows, cols, raw)
    got = W.matvec(q, d)
    want = R.matvec_q(Q8, rows, cols, raw, q, d)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
    # the spec's own bar, stated: within 1e-5 relative (here exact)
    assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want))
    # int32 block sums: the device sums equal numpy's exact integer sums, so the f32 terms start from the same ints
    s = block_sums(Q8, raw, rows, cols, q)
    dw = raw[rows * cols:].view(np.float16).astype(np.float32).reshape(rows, -1)
    acc = np.zeros(rows, np.float32)
    for b in range(cols // 32):
        acc = (acc + (s[:, b].astype(np.float32) * dw[:, b]) * d[b]).astype(np.float32)
    assert np.array_equal(acc.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("dt", [Q8, Q4])
def test_reference_selftest_fixture(qb, dt):
    raw, x = selftest_fixture(dt)
    rows, cols = 4864, 896
    q, d = R.quantize_q8(x)
    W = qb.DeviceTensor(dt, rows, cols, raw)
    got = W.matvec(q, d)
    want = R.matvec_q(dt, rows, cols, raw, q, d)
    assert np.array_equal(got, want)
    # ragged row range
    got2 = W.matvec(q, d, 17, 4001)
    assert np.array_equal(got2[17:4001], want[17:4001]) and not got2[:17].any() and not got2[4001:].any()


@pytest.mark.parametrize("shape", [(4864, 896), (896, 4864)])
def test_config2_gptq_int4_m1_m32_and_4096_rows(qb, shape):
    rows, cols = shape
    rng = np.random.default_rng(99)
    raw = q4_gptq_weights(rng, rows, cols)
    W = qb.DeviceTensor(Q4, rows, cols, raw)
    X = rng.standard_normal((4096, cols)).astype(np.float32)
    qs, ds = [], []
    for t in range(4096):
        q, d = R.quantize_q8(X[t])
        qs.append(q)
        ds.append(d)
    Q = np.stack(qs)
    D = np.stack(ds)
    # M = 1 vs the reference
    got1 = W.matvec(Q[0], D[0])
    want1 = R.matvec_q(Q4, rows, cols, raw, Q[0], D[0])
    assert np.array_equal(got1, want1)
    # M = 32 vs the reference's matmul and vs 32 device M=1 calls
    got32 = W.matmul(Q[:32], D[:32])
    assert np.array_equal(got32, R.matmul_q(Q4, rows, cols, raw, Q[:32], D[:32]))
    mv = np.stack([W.matvec(Q[t], D[t]) for t in range(32)])
    assert np.array_equal(got32, mv)
    # 4096 rows as 128 chunks of 32, every chunk bit-identical to its M=1 results (checked against the reference)
    want_all = R.matmul_q(Q4, rows, cols, raw, Q, D)
    for c in range(128):
        got = W.matmul(Q[32 * c:32 * c + 32], D[32 * c:32 * c + 32])
        assert np.array_equal(got, want_all[32 * c:32 * c + 32]), c


@pytest.mark.parametrize("dt", [Q8, Q4])
@pytest.mark.parametrize("n", [1, 7, 32, 33, 100])
def test_matmul_equals_matvec_ragged(qb, dt, n):
    rng = np.random.default_rng(n)
    rows, cols = 300, 256
    raw = q8_weights(rng, rows, cols) if dt == Q8 else q4_gptq_weights(rng, rows, cols)
    W = qb.DeviceTensor(dt, rows, cols, raw)
    X = rng.standard_normal((n, cols)).astype(np.float32)
    Q, D = zip(*(R.quantize_q8(x) for x in X))
    Q, D = np.stack(Q), np.stack(D)
    got = W.matmul(Q, D, 5, 293)
    for t in range(n):
        mv = W.matvec(Q[t], D[t], 5, 293)
        assert np.array_equal(got[t, 5:293], mv[5:293])
    assert np.array_equal(got[:, 5:293], R.matmul_q(dt, rows, cols, raw, Q, D)[:, 5:293])
