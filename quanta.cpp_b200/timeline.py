"""Per-phase in-graph timeline of b = 1 decode (the three layer kernels), from the phase-timed library.

    python quanta.cpp_b200/build.py --stamps
    python quanta.cpp_b200/timeline.py [MODEL.qnt] [--steps N]

Without a model path it uses the bench's config-4 model (q4mix 0.5B + shortlist, written by bench.py's model_path()).
It runs a 512-token prompt, then N sampled decode steps (T 0.7, top-k 20, top-p 0.8, repetition penalty 1.1) through
the step's CUDA graph, and prints, per kernel kind, the median duration of each phase of its first CTA (SM cycles at
that SM's own cycles-per-ns, from the records' global-timer span), the kernels' spans and the gaps between them.
"""
from __future__ import annotations

import ctypes as C
import os
import statistics
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent

KINDS = {1: "k_attn (q|k|v + attention + o_proj terms)", 2: "k_gateup_dec (o_proj residual + norm + gate|up + SwiGLU)",
         3: "k_resid_dec (down + residual)", 4: "k_embed", 5: "k_sl_mark (must ids)",
         6: "k_head_input (final norm + quantize)", 7: "k_head_rows (coarse pass)", 8: "k_sl_seeds (seeds, tau)",
         9: "k_sl_cands (candidate rows + sampler lists)", 10: "k_sample_final (merge + draw)"}
PHASES = {
    1: ["launch -> previous kernel done", "rmsnorm + quantize", "q|k|v rows, bias, RoPE, exchange",
        "scores + maxima exchange", "exps + exchange", "softmax sum (ordered)", "output chains (ordered)",
        "o_proj terms"],
    2: ["launch -> previous kernel done", "o_proj residual rows + exchange", "rmsnorm + quantize",
        "gate|up block terms", "row chains", "SwiGLU + quantize"],
    3: ["launch -> previous kernel done", "input activation", "down block terms", "row chains + residual"],
    4: ["launch -> previous kernel done", "embedding row"],
    5: ["launch -> previous kernel done", "marks"],
    6: ["launch -> previous kernel done", "rmsnorm + quantize", "block sums and norms"],
    7: ["launch -> previous kernel done", "tiles (coarse scores, bounds, lists)", "list merge"],
    8: ["launch -> previous kernel done", "merge of the CTA lists", "exact seed rows", "tau"],
    9: ["launch -> previous kernel done", "mark / upper scan", "exact candidate rows", "seed offers + list merge"],
    10: ["launch -> previous kernel done", "merge of the lists", "softmax + draw"],
}


class PhaseRec(C.Structure):
    _fields_ = [("g0", C.c_ulonglong), ("g1", C.c_ulonglong), ("c", C.c_longlong * 12), ("kind", C.c_int), ("n", C.c_int),
                ("g_last", C.c_ulonglong)]


def read(L, reset):
    out = []
    for name in ("qnt_phase_read_attn", "qnt_phase_read_layers", "qnt_phase_read_head"):
        fn = getattr(L, name)
        fn.argtypes = [C.c_void_p, C.c_int, C.c_int]
        buf = (PhaseRec * 8192)()
        n = fn(C.cast(buf, C.c_void_p), 8192, 1 if reset else 0)
        if n < 0:
            raise RuntimeError(name + " failed")
        out += [buf[i] for i in range(n)]
    return sorted(out, key=lambda r: r.g0)


def summarize(recs):
    """Markdown table: per kind the median phase durations (µs) and the median span; then the gaps between kernels."""
    lines = []
    by_kind = {}
    for r in recs:
        if r.n >= 2 and r.g1 > r.g0:
            by_kind.setdefault(r.kind, []).append(r)
    for kind in sorted(by_kind):
        rs = by_kind[kind]
        names = PHASES.get(kind, [])
        tails = [(int(r.g_last) - int(r.g1)) / 1e3 for r in rs if r.g_last]
        tail = f", last CTA ends {statistics.median(tails):.2f} µs after CTA 0" if tails else ""
        lines.append(f"\n**{KINDS.get(kind, kind)}**: {len(rs)} launches, median span "
                     f"{statistics.median((r.g1 - r.g0) / 1e3 for r in rs):.2f} µs (global timer){tail}\n")
        lines.append("| phase | median µs | share of the span |")
        lines.append("|---|---|---|")
        nmark = min(r.n for r in rs)
        spans = []
        for k in range(1, nmark):
            vals = []
            for r in rs:
                cyc_per_ns = (r.c[r.n - 1] - r.c[0]) / max(r.g1 - r.g0, 1)
                vals.append((r.c[k] - r.c[k - 1]) / cyc_per_ns / 1e3)
            spans.append(statistics.median(vals))
        tot = sum(spans) or 1.0
        for k, v in enumerate(spans):
            name = names[k] if k < len(names) else f"phase {k + 1}"
            lines.append(f"| {name} | {v:.2f} | {v / tot:.2f} |")
    # gaps: each kernel's CTA-0 start after the previous kernel's CTA-0 end (negative: overlapped by the launch)
    gaps = {}
    for a, b in zip(recs, recs[1:]):
        if a.g1 and b.g0:
            last = int(a.g_last) if a.g_last else int(a.g1)
            gaps.setdefault((a.kind, b.kind), []).append(((int(b.g0) - int(a.g1)) / 1e3, (int(b.g0) - last) / 1e3))
    # the step outside the layers: each non-layer kernel's start and end after the last layer kernel's end
    outside = {}
    last_layer_end = None
    for r in recs:
        if r.kind in (1, 2, 3):
            last_layer_end = int(r.g_last or r.g1) if r.kind == 3 else last_layer_end
        elif last_layer_end is not None and r.g1:
            outside.setdefault(r.kind, []).append(((int(r.g0) - last_layer_end) / 1e3, (int(r.g1) - last_layer_end) / 1e3,
                                                   (int(r.g_last or r.g1) - last_layer_end) / 1e3))
    if outside:
        lines.append("\n| kernel after the last layer (its last CTA's end = 0) | launches | median start µs | "
                     "median CTA 0 end µs | median last CTA end µs |")
        lines.append("|---|---|---|---|---|")
        for kind, v in sorted(outside.items(), key=lambda kv: statistics.median(x[0] for x in kv[1])):
            lines.append(f"| {KINDS.get(kind, kind)} | {len(v)} | {statistics.median(x[0] for x in v):.2f} | "
                         f"{statistics.median(x[1] for x in v):.2f} | {statistics.median(x[2] for x in v):.2f} |")
    lines.append("\n| from -> to | launches | median gap µs (next start - previous CTA 0 end) | (next start - previous last end) |")
    lines.append("|---|---|---|---|")
    for (ka, kb), v in sorted(gaps.items()):
        lines.append(f"| {ka} -> {kb} | {len(v)} | {statistics.median(x[0] for x in v):.2f} | "
                     f"{statistics.median(x[1] for x in v):.2f} |")
    return "\n".join(lines)


def main():
    # the phase-timed library, chosen before the binding is first imported (importing this module has no such effect)
    os.environ.setdefault("QNT_LIB_DIR", str(PKG / "lib_stamps"))
    sys.path.insert(0, str(PKG))
    sys.path.insert(0, str(PKG.parent))
    import numpy as np
    import quanta_b200 as qb
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    steps = int(sys.argv[sys.argv.index("--steps") + 1]) if "--steps" in sys.argv else 32
    if args and not args[0].isdigit():
        path = args[0]
    else:
        import bench
        path = bench.model_path()
    L = qb.lib()
    if not hasattr(L, "qnt_phase_read_attn"):
        raise SystemExit(f"{qb.lib_path()} has no phase records: build it with `python quanta.cpp_b200/build.py --stamps`")
    m = qb.Model(path, ctx_len=4096)
    prompt = np.random.default_rng(1234).integers(0, m.hp.n_tokens, 512).astype(np.int32)
    sp = qb.SamplerParams(temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1, seed=7)
    m.session_begin(prompt, sp)
    m.session_step(8)
    read(L, reset=True)
    m.session_step(steps)
    recs = read(L, reset=True)
    m.close()
    attn = [r for r in recs if r.kind == 1]
    per_step = len(attn) // steps if steps else 0
    step_ns = [(int(attn[i + per_step].g0) - int(attn[i].g0)) for i in range(0, len(attn) - per_step, per_step)] if per_step else []
    print(f"{len(recs)} records over {steps} decode steps; {per_step} layers per step; median step "
          f"{statistics.median(step_ns) / 1e3 if step_ns else float('nan'):.1f} µs (first attention to first attention)")
    print(summarize(recs))


if __name__ == "__main__":
    main()
