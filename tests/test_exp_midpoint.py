"""exp_ref's near-midpoint test (quanta.cpp_b200/csrc/exp_table.h) reads the 29 mantissa bits r that a float drops
from the double e^x: it probes the exception table when |r - 2^28| < 2^22.  The table holds every input whose libm
expf differs from the once-rounded double, so the test stays exact as long as it flags every y that the direct
window test (within kExpNearMidpoint of a half-ulp of the midpoint) flags.  Checked here for every r of two binades:
the top of [1, 2) (where the float rounds up to the next power of two) and the smallest normal binade."""
import numpy as np
import pytest

NEAR = 0.008  # kExpNearMidpoint


def _old_not_new(exp_field, top):
    bad = 0
    for c in range(128):  # 2^22 values per step keeps the arrays to a few hundred MB
        r = np.arange(c << 22, (c + 1) << 22, dtype=np.uint64)
        y = ((np.uint64(exp_field) << np.uint64(52)) | (np.uint64(top) << np.uint64(29)) | r).view(np.float64)
        f = y.astype(np.float32)
        df = f.astype(np.float64)
        e = y - df
        nb = np.where(e >= 0, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf)))
        half = np.abs(nb.astype(np.float64) - df) * 0.5
        old = (half - np.abs(e)) < half * NEAR
        new = np.abs(r.astype(np.int64) - (1 << 28)) < (1 << 22)
        bad += int(np.count_nonzero(old & ~new))
    return bad


@pytest.mark.parametrize("exp_field,top", [(1023, (1 << 23) - 1), (1023 - 126, 0)])
def test_bit_test_covers_the_midpoint_window(exp_field, top):
    assert _old_not_new(exp_field, top) == 0
