"""Tensor-core (tcgen05) matmul, qnt_matmul(impl=2), against the CUDA-core matmul (impl=1) and the reference's
matmul_q_ref (oracle/_ref): bit-identical outputs for Q8_0 and GPTQ-style Q4_0 weights at the BASELINE shapes, ragged
token counts (tails of the 64-token tile) and ragged row ranges (tails of the 128-row tile)."""
import numpy as np
import pytest

import ref as R
from test_gpu_ops import q4_gptq_weights, q8_weights

pytestmark = pytest.mark.gpu
Q8, Q4 = 2, 3


def acts(rng, n, cols):
    X = rng.standard_normal((n, cols)).astype(np.float32)
    Q, D = zip(*(R.quantize_q8(x) for x in X))
    return np.stack(Q), np.stack(D)


@pytest.mark.parametrize("dt", [Q8, Q4])
@pytest.mark.parametrize("shape", [(1152, 896), (896, 4864)])
@pytest.mark.parametrize("n", [1, 33, 64, 100])
def test_tc_matmul_bit_exact(qb, dt, shape, n):
    rows, cols = shape
    rng = np.random.default_rng(rows + n + dt)
    raw = q8_weights(rng, rows, cols) if dt == Q8 else q4_gptq_weights(rng, rows, cols)
    W = qb.DeviceTensor(dt, rows, cols, raw)
    Q, D = acts(rng, n, cols)
    tc = W.matmul(Q, D, impl=2)
    simt = W.matmul(Q, D, impl=1)
    assert np.array_equal(tc.view(np.uint32), simt.view(np.uint32)), np.abs(tc - simt).max()
    if n <= 33:
        assert np.array_equal(tc, R.matmul_q(dt, rows, cols, raw, Q, D))


@pytest.mark.parametrize("dt", [Q8, Q4])
def test_tc_matmul_ragged_rows_and_256_tokens(qb, dt):
    rows, cols = 4864, 896
    rng = np.random.default_rng(7 + dt)
    raw = q8_weights(rng, rows, cols) if dt == Q8 else q4_gptq_weights(rng, rows, cols)
    W = qb.DeviceTensor(dt, rows, cols, raw)
    Q, D = acts(rng, 256, cols)
    tc = W.matmul(Q, D, 37, 4801, impl=2)
    simt = W.matmul(Q, D, 37, 4801, impl=1)
    assert np.array_equal(tc, simt)
    assert not tc[:, :37].any() and not tc[:, 4801:].any()


def test_bounded_wait_runs_out_and_reports(qb):
    """A device wait that nothing completes, with a short limit, ends in QNT_ERR_DEVICE (the timeout bit the matmul's
    waits set), not a hang or a fault; the thread's status is cleared and the device stays usable."""
    L = qb.lib()
    rc = L.qnt_wait_probe(200, None)
    assert rc == -6, (rc, L.qnt_last_error())
    assert b"status bits 1" in L.qnt_last_error()
    assert L.qnt_ops_check(None) == 0  # the bit was cleared
    rng = np.random.default_rng(0)
    W = qb.DeviceTensor(2, 128, 256, np.concatenate([rng.integers(-127, 128, 128 * 256).astype(np.int8).view(np.uint8),
                                                      np.full(128 * 8, 0x2000, np.uint16).view(np.uint8)]))
    q, d = qb.quantize_q8(rng.standard_normal(256).astype(np.float32))
    assert np.isfinite(W.matvec(q, d)).all()
    W.close()
