"""Benchmark of the quantized-transformer hot path on B200 (one process per GPU).

Workload (the metric's b=1 case): random-init Qwen2.5-0.5B q4mix (attention Q8_0, MLP GPTQ-sym int4
g128) with the Exact Shortlist Head; 512 uniform-random prompt ids; decode at temperature 0.7, top-k 20, top-p 0.8,
repetition penalty 1.1 (the reference's SamplerParams defaults), fixed seed.  One step = one decode token on the
device: sample -> append -> 24-layer forward -> shortlist head (one CUDA-graph replay).  With N GPUs every rank
decodes its own sequence (independent sequences, no data-path collective: weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` = decode tok/s over all ranks, timed with CUDA events on the model's stream
(max over ranks).  `e2e` = the same workload through the public C ABI call qnt_generate with host buffers
(prompt in, ids out) timed by the host clock, prefill included.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "quanta.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
import dp  # noqa: E402  (quanta.cpp_b200/dp.py: data-parallel plumbing)

MODEL_DIR = Path(os.environ.get("QNT_MODEL_DIR", "/tmp/qnt_models"))
PROMPT = 512
SEED = 1234
METRIC = "decode tok/s (q4mix 0.5B + shortlist head, b=1)"
PEAKS = ROOT / "MEASURED_PEAKS.json"


# DRAM bytes of one decode step of this workload, summed over its launches from one ncu capture (the command and the
# per-kernel table are in profiles/decode_step_traffic_q4mix_sl.md)
STEP_TRAFFIC_BYTES = 339_039_744


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def peaks():
    try:
        p = json.loads(PEAKS.read_text())
        return p["hbm_gbs"], "measured"
    except Exception:
        return 6650.0, "fallback"


def tc_matmul_measure(tokens, iters=20):
    """The tensor-core int8 matmul alone on the gate|up shape (9728 x 896, GPTQ-style Q4 weights, their int8 copy L2
    resident) at `tokens` tokens, through qnt_matmul(impl=2) with device buffers: CUDA-event time per call and the
    int8 rate against twice the measured dense bf16 rate (int8 dense peak = 2 x bf16 on this GPU)."""
    import torch
    import quanta_b200 as qb
    rows, cols = 9728, 896
    rng = np.random.default_rng(SEED + 11)
    qi = (rng.integers(-8, 8, (rows, cols)) + 8).astype(np.uint8).reshape(-1, 32)
    packed = (qi[:, :16] & 0xF) | (qi[:, 16:] << 4)
    d = (0.02 / 4.6 * rng.uniform(0.75, 1.25, (rows, cols // 32))).astype(np.float16)
    W = qb.DeviceTensor(3, rows, cols, np.concatenate([packed.astype(np.uint8).ravel(), d.view(np.uint8).ravel()]))
    L = qb.lib()
    x = torch.randn(tokens, cols, device="cuda")
    qx = torch.empty(tokens, cols, dtype=torch.int8, device="cuda")
    dx = torch.empty(tokens, cols // 32, device="cuda")
    out = torch.empty(tokens, rows, device="cuda")
    st = torch.cuda.current_stream()
    sp = C.c_void_p(st.cuda_stream)
    qb._check(L.qnt_quantize_q8(C.c_void_p(x.data_ptr()), tokens, cols, C.c_void_p(qx.data_ptr()), C.c_void_p(dx.data_ptr()), sp))
    call = lambda: qb._check(L.qnt_matmul(W.h, C.c_void_p(qx.data_ptr()), C.c_void_p(dx.data_ptr()), tokens, 0, rows,
                                          C.c_void_p(out.data_ptr()), rows, 2, sp))
    for _ in range(3):
        call()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(iters):
        call()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    tops = 2.0 * rows * cols * tokens / (us * 1e-6) / 1e12
    try:
        bf16 = json.loads(PEAKS.read_text())["bf16_tflops"]
        peak, kind = 2 * bf16, "measured (2 x bf16 dense)"
    except Exception:
        peak, kind = 2 * 1590.0, "fallback (2 x bf16 dense)"
    W.close()
    return {"shape": f"{rows}x{cols} Q4 (gate|up) x {tokens} tokens", "us_per_call": round(us, 2),
            "achieved": round(tops, 1), "peak": round(peak, 1), "unit": "TOP/s", "frac": round(tops / peak, 4),
            "peak_kind": kind, "bound": "epilogue: three rounded f32 ops per (row, token, 32-block)"}


def model_path():
    import quanta_b200 as qb
    return qb.synth_model(MODEL_DIR / "q4mix_sl.qnt", shape=qb.QWEN05B, mlp_q4=True, shortlist=True, seed=SEED)


def prompt_ids(rank, n_tokens):
    return np.random.default_rng(dp.rank_seed(SEED, rank)).integers(0, n_tokens, PROMPT).astype(np.int32)


def cpu_baseline(path, steps):
    """The reference's own CPU path (oracle/_ref) on this host's cores, bounded sample: 512-token prefill then `steps`
    decode tokens with the same sampler, timed by the reference's Session (engine/src/session.cpp:33-52)."""
    import ref as R
    threads = os.cpu_count() or 1
    if R.have_ref():
        r = R.RefModel(path, ctx=4096, threads=threads)
        kind = "reference"
    else:
        return None
    ids, st = r.generate(prompt_ids(0, r.n_tokens), steps, temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1,
                         seed=SEED, batch_prefill=True, shortlist=True)
    r.close()
    return {"value": round(len(ids) / st["decode_s"], 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"512-token prompt prefilled ({st['prefill_s']:.1f} s, untimed) then {len(ids)} decode tokens",
            "prefill_tok_s": round(PROMPT / st["prefill_s"], 2), "head_fraction": round(st["head_fraction"], 4)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    import quanta_b200 as qb  # noqa: F401  (only for the synthetic model writer)
    import ref as R
    path = model_path()
    if not R.have_ref():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libquanta_ref.so not built"}))
        return
    n = args.warmup + args.steps
    base = cpu_baseline(path, n)
    out = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / base["value"], 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int8/int4 x int8 -> f32", "data": "synthetic",
           "config": {"workload": "config4: q4mix 0.5B + shortlist, 512-token prompt, b=1 decode, T=0.7 k=20 p=0.8 rp=1.1"},
           "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def run_ours(args, rank, world, local_rank):
    import quanta_b200 as qb
    qb.set_device(local_rank)
    import torch
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    path = model_path() if rank == 0 or world == 1 else None
    if dist:
        dist.barrier()
        path = model_path()
    m = qb.Model(path, ctx_len=4096)
    prompt = prompt_ids(rank, m.hp.n_tokens)
    sp = qb.SamplerParams(temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1, seed=SEED + rank)
    stream = torch.cuda.ExternalStream(m.stream)

    # prefill (timed separately: prompt tok/s)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    m.session_begin(prompt, sp)  # compiles the graphs of the first call
    m.session_begin(prompt, sp)
    torch.cuda.nvtx.range_push("prefill")
    t0 = time.perf_counter()
    m.session_begin(prompt, sp)
    prefill_s = time.perf_counter() - t0
    torch.cuda.nvtx.range_pop()
    # warm-up, then exactly K steps bracketed by barrier + synchronize, CUDA events on the model's stream
    m.session_step(args.warmup)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank) as clk:
        torch.cuda.nvtx.range_push("decode")  # lets a profiler select the timed steps (ncu --nvtx-include "decode/")
        ev[0].record(stream)
        m.session_step(args.steps)
        ev[1].record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = ev[0].elapsed_time(ev[1])
    if dist:
        dist.barrier()
    ids, st = m.session_read()
    kps = st["kernels_per_step"]
    ms_max = dp.max_over_ranks(ms, dist, device="cuda")  # the slowest rank's time is the job's
    value = world * args.steps / (ms_max / 1e3)

    # algorithmic bytes of one decode step (layers + head + KV), per rank
    hp = m.hp
    head_rows_mean = st["head_rows"] / max(st["head_calls"], 1)
    layer_bytes = m.weight_bytes - (hp.vocab_size * (hp.dim + hp.dim // 32 * 2))  # minus embedding/Q8 head
    # (the shortlist pass reads the Q4 copy + err, and head_rows exact Q8 rows)
    q4 = hp.vocab_size * (hp.dim // 2 + hp.dim // 32 * 2)
    err = hp.vocab_size * (hp.dim // 32) * 2
    layer_only = layer_bytes - q4 - err
    pos_mid = PROMPT + args.warmup + args.steps / 2
    kv = 12288 / 24 * hp.n_layers * pos_mid * (hp.n_kv_heads * hp.head_dim / 128)
    step_bytes = layer_only + q4 + err + head_rows_mean * (hp.dim + hp.dim // 32 * 2) + kv + hp.dim
    peak, peak_kind = peaks()
    achieved = step_bytes / (ms_max / args.steps / 1e3) / 1e9

    # e2e through the public C-ABI call with host buffers: qnt_generate (prompt in, ids out), prefill included
    pin_prompt = torch.from_numpy(prompt).pin_memory().numpy()
    m.generate(pin_prompt, sp, 4)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids_e2e, st_e2e = m.generate(pin_prompt, sp, args.steps)
    e2e_s = time.perf_counter() - t0
    e2e_value = world * len(ids_e2e) / dp.max_over_ranks(e2e_s, dist, device="cuda")

    # config 5 style throughput serving on this rank: BATCH sequences of PROMPT tokens, then greedy steps of all of
    # them at once (qnt_decode_batch: tensor-core layers, fused greedy head); device time with CUDA events
    batch = None
    if args.batch > 0:
        B, bsteps = args.batch, args.batch_steps
        m.batch_init(B, PROMPT + bsteps + 8)
        rngb = np.random.default_rng(dp.rank_seed(SEED + 7, rank))
        prompts = rngb.integers(0, m.hp.n_tokens, (B, PROMPT)).astype(np.int32)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        last = np.array([m.prefill_batch(s, prompts[s]) for s in range(B)], np.int32)
        torch.cuda.synchronize()
        bprefill_s = time.perf_counter() - t0
        seqs = np.arange(B, dtype=np.int32)
        for _ in range(2):  # warm-up steps
            last = m.decode_batch(seqs, last)
        torch.cuda.synchronize()
        eb = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.nvtx.range_push("batch")  # lets a profiler select the timed batched steps
        eb[0].record(stream)
        for _ in range(bsteps):
            last = m.decode_batch(seqs, last)
        eb[1].record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        bms = dp.max_over_ranks(eb[0].elapsed_time(eb[1]), dist, device="cuda")
        batch = {"workload": f"config5 style: {B} sequences x {PROMPT}-token prompts per GPU, greedy, batched decode",
                 "value": round(world * B * bsteps / (bms / 1e3), 1), "unit": "tok/s", "steps": bsteps,
                 "ms_per_step": round(bms / bsteps, 3), "prefill_tok_s": round(B * PROMPT / bprefill_s, 1),
                 "note": "each step: one token for every sequence, ids copied to the host",
                 "tc_matmul": tc_matmul_measure(B)}
        m.batch_init(1, 2)  # release the batch caches

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base = cpu_baseline(path, 16)
        except Exception as e:  # the checker is optional on a box without it
            base = {"error": str(e)}
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/int4 x int8 -> f32 (f16 KV)", "data": "synthetic",
            "config": {"workload": "config4: q4mix 0.5B + shortlist, 512-token prompt, b=1 decode, T=0.7 k=20 p=0.8 rp=1.1",
                       "parallelism": f"dp{world} (independent sequences)", "l2": "inputs larger than L2 (~309 MB read per step)"},
            "prefill_tok_s": round(PROMPT / prefill_s, 1),
            "head_rows_mean": round(head_rows_mean, 1),
            "bytes_per_token": int(step_bytes),
            "roofline": {"bound": "hbm", "kernel": "whole decode step (all kernels of one graph replay)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind, "traffic": STEP_TRAFFIC_BYTES,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum summed over one step's launches "
                                           "(profiles/decode_step_traffic_q4mix_sl.md)"},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": round(PROMPT * 4 / args.steps, 1),
                    "d2h_bytes_per_step": 4, "note": "qnt_generate wall clock incl. 512-token prefill"},
            "gpu_launches": kps * args.steps,
            "kernels_per_step": kps,
            "clocks": clk.summary(),
            "cpu_baseline": base,
            "batch_decode": batch,
        }
        print(json.dumps(out))
    m.close()
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=256, help="sequences of the batched-serving measurement (0: skip)")
    ap.add_argument("--batch-steps", type=int, default=32)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
