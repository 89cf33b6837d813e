"""quanta.cpp_b200/timeline.py's summary of phase records (the phase-timed build's reader), on synthetic records: the
per-phase medians, the last-CTA tail, the segment after the last layer and the gaps.  CPU only."""
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent / "quanta.cpp_b200"
sys.path.insert(0, str(PKG))

import timeline as T  # noqa: E402


def rec(kind, g0, g1, marks, g_last=0):
    r = T.PhaseRec()
    r.kind, r.g0, r.g1, r.n, r.g_last = kind, g0, g1, len(marks), g_last
    for i, c in enumerate(marks):
        r.c[i] = c
    return r


def test_summary_of_synthetic_records():
    recs = []
    t = 0
    for step in range(3):  # one layer (attention, gate|up, down) then the final norm, 1 cycle per ns
        recs.append(rec(1, t, t + 16_000, [0, 2_000, 5_000, 7_000, 8_000, 10_000, 11_500, 14_000, 16_000], t + 17_000))
        recs.append(rec(2, t + 5_000, t + 26_000, [0, 13_000, 15_000, 18_000, 19_000, 19_500, 21_000], t + 27_000))
        recs.append(rec(3, t + 20_000, t + 31_000, [0, 8_000, 9_000, 10_000, 11_000], t + 31_500))
        recs.append(rec(6, t + 30_000, t + 37_000, [0, 2_000, 6_000, 7_000]))
        t += 100_000
    out = T.summarize(recs)
    assert "3 launches, median span 16.00 µs" in out
    assert "last CTA ends 1.00 µs after CTA 0" in out
    assert "| rmsnorm + quantize | 3.00 |" in out
    assert "| k_head_input (final norm + quantize) | 3 | -1.50 | 5.50 | 5.50 |" in out  # after the down kernel's last CTA
    assert "| 1 -> 2 | 3 | -11.00 | -12.00 |" in out
