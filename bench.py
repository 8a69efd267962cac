#!/usr/bin/env python3
"""Benchmark of the packed matrix-product path (one JSON line on rank 0).

Workload (the headline benchmark's configuration 1): the Q8_0 matvec at TinyLlama lm_head shape,
W 32000 x 2048 drawn N(0, 0.02) and quantized with the reference's Q8_0 rule (bit-exact
GPU quantizer), x ~ N(0, 1). A step is one matvec. Six device copies of W (418 MB,
> 3x the 126 MB L2) are used in rotation, so every step streams its weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W]      # our B200 path
  python bench.py --impl reference                           # the reference's CPU path

Metric: algorithmic bytes per step (packed W + x + y = 69,768,192 B) / time, in GB/s.
value: device time of K steps (CUDA events, a CUDA graph of the C-ABI launches, max over
ranks). e2e: the same steps through the host-pointer C-ABI call efg_host_matvec (pinned
x in, y out every step; W resident after its first upload), wall clock.
N > 1: each rank runs its own config-1 matvecs (weak scaling, no collective in the data
path); value = bytes of all ranks / max time.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 32000, 2048
Q8_0, Q4_0 = 3, 4
N_COPIES = 6
METRIC = "Q8_0 matvec HBM GB/s (lm_head 32000x2048)"


def algo_bytes(qt, rows, cols):
    return rows * (cols // 32) * (18 if qt == Q4_0 else 34) + 4 * cols + 4 * rows


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def rank_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """Samples SM clock and throttle reasons every 10 ms while running."""

    NAMES = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sync_boost", 0x40: "sw_thermal_slowdown",
             0x80: "hw_thermal_slowdown", 0x100: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.stop_ev = [], 0, threading.Event()
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nvml = None

    def _sample(self):
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            self.reasons |= int(self.get_reasons(self.h))
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self.stop_ev.is_set():
            self._sample()
            self.stop_ev.wait(0.01)

    def __enter__(self):
        if self.nvml:
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.nvml:
            self.stop_ev.set()
            self.t.join()
            self._sample()

    def summary(self):
        if not self.nvml or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for b, n in self.NAMES.items() if self.reasons & b]
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ---------------------------------------------------------------- reference CPU leg
def cpu_reference_matvec(seconds: float, qt=Q8_0, rows=ROWS, cols=COLS, copies=N_COPIES, steps=None, warmup=3,
                         cap_seconds=150.0):
    """The reference's AVX2 matvec (kern::matvec + ThreadPool, oracle/_ref) on the host
    cores: rotating W copies (418 MB, larger than the host's last-level cache). Runs
    `steps` matvecs (or for `seconds` when steps is None), never longer than cap_seconds."""
    from oracle.oracle import Oracle, Reference

    ref, orc = Reference(), Oracle()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    X = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    W = orc.quantize_rows(qt, X, threads=threads)
    del X
    Ws = [W.copy() for _ in range(copies)]
    x = rng.standard_normal(cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    with ref.pool(threads) as pool:
        for i in range(max(warmup, copies)):  # warm-up: page in every copy
            ref.matvec_backend(qt, Ws[i % copies], x, rows, avx2=True, pool=pool, y=y)
        n, t0 = 0, time.perf_counter()
        while True:
            ref.matvec_backend(qt, Ws[n % copies], x, rows, avx2=True, pool=pool, y=y)
            n += 1
            el = time.perf_counter() - t0
            if (steps is not None and n >= steps) or (steps is None and el >= seconds) or el >= cap_seconds:
                break
    return algo_bytes(qt, rows, cols) * n / el / 1e9, threads, n, el


def run_reference_arm(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return 0
    if not (ROOT / "oracle" / "_ref" / "libefref.so").exists():
        emit({"impl": "reference", "unavailable": "oracle/_ref/libefref.so was not built"})
        return 0
    # W untimed warm-up steps, then K timed steps (each one CPU matvec of the workload;
    # stopped after 150 s, in which case "steps" reports the count actually timed)
    gbs, threads, n, el = cpu_reference_matvec(0.0, steps=args.steps, warmup=args.warmup)
    args.steps = n
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el / n * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (Q8_0 weights)", "data": "synthetic (seeded N(0,0.02) W, N(0,1) x)",
        "config": {"workload": "config1_q8_0_matvec_32000x2048", "rows": ROWS, "cols": COLS, "copies": N_COPIES,
                   "l2": "host LLC exceeded by rotating copies"},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": f"{n} matvecs of the reference AVX2 kernel, ThreadPool({threads})"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ---------------------------------------------------------------- our GPU arm
def make_weights(efg, torch, qt, rows, cols, copies, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(rows, cols, generator=g, device="cuda", dtype=torch.float32) * 0.02
    W = torch.empty(rows * (cols // 32) * (18 if qt == Q4_0 else 34), dtype=torch.uint8, device="cuda")
    efg.quantize_rows(qt, X, rows, cols, W, True)
    del X
    return [W] + [W.clone() for _ in range(copies - 1)]


def graph_of_steps(efg, torch, qt, Ws, x, y, rows, cols, n):
    """A CUDA graph of n matvec launches made through the C ABI (rotating copies)."""
    s = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        for i in range(2):  # launch once outside capture (attributes, lazy init)
            efg.matvec(qt, y, Ws[i % len(Ws)], x, rows, cols)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            for i in range(n):
                efg.matvec(qt, y, Ws[i % len(Ws)], x, rows, cols)
    return graph


def time_steps(efg, torch, qt, Ws, x, y, rows, cols, steps, warmup, chunk=60):
    """Device time (ms) of exactly `steps` matvecs, launched as CUDA graphs."""
    chunk = max(len(Ws), min(chunk, steps))
    g_full = graph_of_steps(efg, torch, qt, Ws, x, y, rows, cols, chunk)
    rem = steps % chunk
    g_rem = graph_of_steps(efg, torch, qt, Ws, x, y, rows, cols, rem) if rem else None
    g_warm = graph_of_steps(efg, torch, qt, Ws, x, y, rows, cols, max(warmup, 1))
    g_warm.replay()
    torch.cuda.synchronize()
    return g_full, g_rem, chunk


def run_ours(args):
    import torch

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    import edgeforge_b200 as efg

    efg.set_weight_prefetch(True)  # static weights: stream them during the previous kernel's tail
    hbm_peak, peak_kind = peaks()
    bf16_peak = bf16_peak_tflops()
    nbytes = algo_bytes(Q8_0, ROWS, COLS)

    Ws = make_weights(efg, torch, Q8_0, ROWS, COLS, N_COPIES, seed=1 + rank)
    x = torch.randn(COLS, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    y = torch.empty(ROWS, device="cuda")
    g_full, g_rem, chunk = time_steps(efg, torch, Q8_0, Ws, x, y, ROWS, COLS, args.steps, args.warmup)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps // chunk):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()
        end.record()
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = nbytes * world * args.steps / (ms / 1e3) / 1e9
    achieved = nbytes / (ms_step / 1e3) / 1e9  # per launch, one GPU

    # ---- e2e: the host-pointer C-ABI call, pinned x in and y out every step
    x_h = torch.empty(COLS, dtype=torch.float32).pin_memory().numpy()
    y_h = torch.empty(ROWS, dtype=torch.float32).pin_memory().numpy()
    x_h[:] = x.cpu().numpy()
    Wh = Ws[0].cpu().numpy()
    Whs = [Wh.copy() for _ in range(N_COPIES)]
    for w in Whs:  # like a model load: each weight copy is registered (uploaded) once
        efg.host_register_weights(w)
    for i in range(args.warmup):
        efg.host_matvec(Q8_0, Whs[i % N_COPIES], x_h, ROWS, y=y_h)
    barrier()
    e2e_steps = max(args.steps, 1)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        efg.host_matvec(Q8_0, Whs[i % N_COPIES], x_h, ROWS, y=y_h)
    el = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([el], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        el = float(t.item())
    e2e = nbytes * world * e2e_steps / el / 1e9
    efg.host_release_weights()
    assert efg.device_error() == 0

    # ---- extra: the Q4_0 matvec at TinyLlama gate_proj shape (config 0), same protocol
    q4_rows, q4_cols = 5632, 2048
    q4_copies = 64  # 64 x 6.5 MB = 415 MB in rotation
    W4 = make_weights(efg, torch, Q4_0, q4_rows, q4_cols, q4_copies, seed=3)
    y4 = torch.empty(q4_rows, device="cuda")
    k4 = 1280  # kept well below the headline's launch count so the Q8_0 kernel dominates
    g4, _, c4 = time_steps(efg, torch, Q4_0, W4, x, y4, q4_rows, q4_cols, k4, 64, chunk=640)
    torch.cuda.synchronize()
    s4, e4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s4.record()
    for _ in range(k4 // c4):
        g4.replay()
    e4.record()
    torch.cuda.synchronize()
    ms4 = s4.elapsed_time(e4) / k4
    gbs4 = algo_bytes(Q4_0, q4_rows, q4_cols) / (ms4 / 1e3) / 1e9
    del W4

    dec = decode_extra(hbm_peak, with_cpu=not args.no_cpu_baseline) if world == 1 and not args.no_decode else None
    shard = None if args.no_sharded else sharded_extra(torch, efg, world, rank, hbm_peak)
    lmh = None if args.no_sharded else lm_head_extra(torch, efg, world, rank)
    gemm = gemm_extra(torch, efg, bf16_peak) if world == 1 and not args.no_gemm else None
    quant = quant_extra(torch, efg, hbm_peak) if world == 1 and not args.no_gemm else None

    # DRAM bytes per launch of this kernel from the committed ncu capture summary
    traffic = None
    tpath = ROOT / "profiles" / "matvec_q8_0_32000x2048.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get("dram_bytes_per_launch")

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and (ROOT / "oracle" / "_ref" / "libefref.so").exists():
            gbs_c, thr, n_c, el_c = cpu_reference_matvec(args.cpu_seconds)
            cpu = {"value": round(gbs_c, 3), "unit": "GB/s", "cores": thr, "kind": "reference",
                   "sample": f"{n_c} matvecs ({el_c:.1f} s) of the reference AVX2 kernel + ThreadPool({thr}) "
                             f"on config 1, {N_COPIES} rotating W copies"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (Q8_0 weights)", "data": "synthetic (seeded N(0,0.02) W, N(0,1) x)",
            "config": {"workload": "config1_q8_0_matvec_32000x2048", "rows": ROWS, "cols": COLS,
                       "copies": N_COPIES, "l2": "inputs larger than L2: 6 rotating W copies (418 MB)",
                       "launch": "CUDA graph of C-ABI launches with early weight prefetch (PDL)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": nbytes},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * COLS,
                    "d2h_bytes_per_step": 4 * ROWS,
                    "api": "efg_host_matvec (host pointers; W registered resident once, like a model load)"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "extra": {"config0_q4_0_matvec_5632x2048": {
                "gbs": round(gbs4, 1), "frac_of_hbm": round(gbs4 / hbm_peak, 4), "us_per_launch": round(ms4 * 1e3, 3),
                "bytes_per_launch": algo_bytes(Q4_0, q4_rows, q4_cols), "copies": q4_copies},
                "config2_decode_tinyllama": dec,
                "config4_sharded_q4_0_131072x8192": shard,
                "lm_head_sharded_argmax_32000x2048": lmh,
                "config3_gemm_q4_0": gemm,
                "config1_quantize_round_trip": quant},
        }
        emit(line)
    if world > 1:
        del g_full, g_rem
        torch.distributed.destroy_process_group()
    return 0


def decode_model():
    """The config-2 model: a random TinyLlama-1.1B-shaped checkpoint (seed 0) quantized by
    this library's GPU writer with the reference's "auto" policy; cached in the temp dir."""
    import tempfile

    import edgeforge_b200 as efg
    from edgeforge_b200 import synthetic

    d = Path(os.environ.get("EFG_TEST_CACHE", tempfile.gettempdir())) / "efg_tinyllama_seed0"
    if not (d / "model.safetensors").exists() or not (d / "config.json").exists():
        synthetic.write_checkpoint(d, synthetic.TINYLLAMA, seed=0)
    efq = d / "model-gpu.efq"
    if not efq.exists():
        part = d / "model-gpu.efq.part"
        efg.quantize_model(d, part, policy="auto")
        part.rename(efq)
    return efq


def decode_extra(hbm_peak, with_cpu, prompt_len=23, steps=32, reps=5):
    """Config 2: a 23-token prompt, then 32 greedy decode steps (device time of the decode
    loop, best of `reps` runs after one warm-up run)."""
    import edgeforge_b200 as efg

    efq = decode_model()
    prompt = np.random.default_rng(2).integers(0, 32000, prompt_len).astype(np.int32)
    with efg.Decoder(efq, prompt_len + steps) as dec:
        dec.generate(prompt, steps)
        runs = []
        for _ in range(reps):
            t0 = time.perf_counter()
            r = dec.generate(prompt, steps)
            runs.append((r.decode_seconds, r.prefill_seconds, time.perf_counter() - t0))
        bpt = dec.bytes_per_token
        tokens = r.tokens
        # several sequences at once (efg_decoder_step_slots): S slots, each fed its own
        # 23-token prompt through the batch step, then `steps` greedy steps of all S rows
        batch = {}
        rng = np.random.default_rng(3)
        for S in (8, 32, 64):
            dec.set_slots(S)
            prompts = rng.integers(0, 32000, (S, prompt_len)).astype(np.int32)
            slots = np.arange(S, dtype=np.int32)
            for t in range(prompt_len):
                _, nxt = dec.step_slots(slots, prompts[:, t], np.full(S, t, np.int32), compute_logits=False)
            t0 = time.perf_counter()
            for k in range(steps - 1):
                _, nxt = dec.step_slots(slots, nxt, np.full(S, prompt_len + k, np.int32), compute_logits=False)
            el = time.perf_counter() - t0
            batch[f"S{S}"] = {"tok_s": round(S * (steps - 1) / el, 1), "ms_per_step": round(el / (steps - 1) * 1e3, 3)}
        dec.set_slots(1)
    dsec, psec, wall = min(runs)
    tok_s = (steps - 1) / dsec
    out = {"decode_tok_s": round(tok_s, 1), "prefill_tok_s": round(prompt_len / psec, 1),
           "weight_gbs": round(bpt * tok_s / 1e9, 1), "frac_of_hbm": round(bpt * tok_s / 1e9 / hbm_peak, 4),
           "ms_per_token": round(dsec / (steps - 1) * 1e3, 4), "bytes_per_token": bpt,
           "e2e_generate_s": round(wall, 5), "prompt": prompt_len, "steps": steps,
           "batch_decode": dict(batch, note="efg_decoder_step_slots, S sequences per step, host wall time per step"),
           "model": "random TinyLlama-1.1B shape, .efq from efg_quantize_model (policy auto)"}
    if with_cpu and (ROOT / "oracle" / "_ref" / "libefref.so").exists():
        from oracle.oracle import Reference

        threads = os.cpu_count() or 1
        rd = Reference().decoder(efq, prompt_len + steps, threads=threads)
        pos = 0
        for i, t in enumerate(prompt):
            lg = rd.forward(int(t), pos, 32000, logits=i + 1 == prompt_len)
            pos += 1
        t0 = time.perf_counter()
        ref_tokens = []
        for step in range(steps):
            ref_tokens.append(int(np.argmax(lg)))
            if step + 1 == steps:
                break
            lg = rd.forward(ref_tokens[-1], pos, 32000)
            pos += 1
        el = time.perf_counter() - t0
        rd.close()
        out["cpu_reference_tok_s"] = round((steps - 1) / el, 2)
        out["cpu_reference_threads"] = threads
        out["greedy_tokens_match_reference"] = ref_tokens == list(tokens)
    return out


def sharded_extra(torch, efg, world, rank, hbm_peak, steps=200, warmup=10, rows=131072, cols=8192):
    """Config 4: the Q4_0 131072 x 8192 matvec (604 MB) row-sharded over the job's GPUs, y
    all-gathered over NVLink every step (efg_matvec_sharded). Strong scaling: the matrix is
    fixed, each rank holds rows/world of it. Device time of `steps` steps, max over ranks."""
    b, c = efg.shard_rows(rows, world, rank)
    rb = cols // 32 * 18
    W = torch.empty(max(c, 1) * rb, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for r0 in range(0, c, 8192):  # quantize the shard in 8192-row pieces (bounded FP32 temp)
        n = min(8192, c - r0)
        X = torch.randn(n, cols, generator=g, device="cuda") * 0.02
        efg.quantize_rows(Q4_0, X, n, cols, W[r0 * rb:], True)
    del X
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda")
    y = torch.empty(rows, device="cuda")
    comm = efg.Comm.from_torch() if world > 1 else efg.Comm(efg.Comm.unique_id(), 1, 0)

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(n):
            fn()
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms / n

    ms_all = timed(lambda: efg.matvec_sharded(Q4_0, y, W, x, rows, cols, comm), steps)
    ms_local = timed(lambda: efg.matvec(Q4_0, y[b:], W, x, c, cols), steps)
    efg.set_q4_mma(False)  # the same local matvec on the CUDA-core kernel, for comparison
    try:
        ms_local_cc = timed(lambda: efg.matvec(Q4_0, y[b:], W, x, c, cols), steps)
    finally:
        efg.set_q4_mma(True)
    comm.close()
    assert efg.device_error() == 0
    total = rows * rb + 4 * cols + 4 * rows
    shard_bytes = c * rb + 4 * cols + 4 * c
    del W
    return {"us_per_step": round(ms_all * 1e3, 3), "gbs_total": round(total / (ms_all / 1e3) / 1e9, 1),
            "local_matvec_us": round(ms_local * 1e3, 3),
            "local_frac_of_hbm": round(shard_bytes / (ms_local / 1e3) / 1e9 / hbm_peak, 4),
            "local_kernel": "int8 tensor-core MMA (efg_matvec_mma.cu)",
            "local_matvec_us_cuda_cores": round(ms_local_cc * 1e3, 3),
            "local_frac_of_hbm_cuda_cores": round(shard_bytes / (ms_local_cc / 1e3) / 1e9 / hbm_peak, 4),
            "gather_bytes": 4 * rows, "ranks": world, "rows_per_rank": c, "matrix_bytes": rows * rb,
            "scaling": "strong"}


def lm_head_extra(torch, efg, world, rank, steps=200, warmup=10, rows=32000, cols=2048):
    """The decode step's last operation with lm_head (Q8_0 32000 x 2048) row-sharded over the
    job's GPUs: this rank's logits with the final RMSNorm fused, then the argmax over all
    ranks (efg_lm_head_argmax_sharded: one 8-byte-per-rank all-gather). Device time per call,
    max over ranks; strong scaling."""
    b, c = efg.shard_rows(rows, world, rank)
    rb = cols // 32 * 34
    g = torch.Generator(device="cuda").manual_seed(200)
    X = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    W = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    efg.quantize_rows(Q8_0, X, rows, cols, W, True)
    del X
    shard = W[b * rb:(b + c) * rb].clone()
    del W
    x = torch.randn(cols, generator=g, device="cuda")
    nw = torch.ones(cols, device="cuda")
    logits = torch.empty(max(c, 1), device="cuda")
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    comm = efg.Comm.from_torch() if world > 1 else efg.Comm(efg.Comm.unique_id(), 1, 0)
    for _ in range(warmup):
        efg.lm_head_argmax_sharded(Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        efg.lm_head_argmax_sharded(Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)
    s1.record()
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    comm.close()
    assert efg.device_error() == 0
    return {"us_per_call": round(ms * 1e3, 3), "ranks": world, "rows_per_rank": c, "token": int(tok.item()),
            "scaling": "strong"}


def quant_extra(torch, efg, hbm_peak, reps=5):
    """Config 1's round trip: the 32000 x 2048 FP32 matrix quantized to Q4_0 (with the MSE
    scale search) and Q8_0, and dequantized back, on the device (bit-exact kernels);
    GB/s = bytes read + written per call."""
    g = torch.Generator(device="cuda").manual_seed(11)
    X = torch.randn(ROWS, COLS, generator=g, device="cuda") * 0.02
    out = {}
    for name, qt in (("q4_0", Q4_0), ("q8_0", Q8_0)):
        rb = COLS // 32 * (18 if qt == Q4_0 else 34)
        Wq = torch.empty(ROWS * rb, dtype=torch.uint8, device="cuda")
        Xd = torch.empty_like(X)
        for fn, label in ((lambda: efg.quantize_rows(qt, X, ROWS, COLS, Wq, True), "quantize"),
                          (lambda: efg.dequantize_rows(qt, Wq, ROWS, COLS, Xd), "dequantize")):
            fn()
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            for _ in range(reps):
                fn()
            s1.record()
            torch.cuda.synchronize()
            ms = s0.elapsed_time(s1) / reps
            nb = X.numel() * 4 + Wq.numel()
            out[f"{label}_{name}"] = {"ms": round(ms, 4), "gbs": round(nb / ms / 1e6, 1),
                                      "frac_of_hbm": round(nb / ms / 1e6 / hbm_peak, 4)}
    del X
    return out


def gemm_extra(torch, efg, bf16_peak, reps=20):
    """Config 3: Q4_0 GEMM Y[B][M] = W X^T on the tensor cores for (M, K) = gate/up and down
    shapes and B in {1, 16, 64, 256}: device time per call, useful TFLOP/s (2 M K B) and
    the tensor-pipe rate the three BF16 MMAs per product imply."""
    out = {}
    for M, K in ((5632, 2048), (2048, 5632)):
        W = make_weights(efg, torch, Q4_0, M, K, 1, seed=7)[0]
        for B in (1, 16, 64, 256):
            X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(8), device="cuda")
            Y = torch.empty(B, M, device="cuda")
            for _ in range(3):
                efg.gemm_q4_0(Y, W, X, M, K, B)
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            for _ in range(reps):
                efg.gemm_q4_0(Y, W, X, M, K, B)
            s1.record()
            torch.cuda.synchronize()
            us = s0.elapsed_time(s1) / reps * 1e3
            fl = 2.0 * M * K * B
            # tensor work issued: two BF16 weight terms, each against the X hi / lo parts
            # stacked along N, with B padded to the 16-column tile
            issued = 4 * 2.0 * M * K * ((B + 15) // 16 * 16)
            out[f"{M}x{K}_B{B}"] = {"us": round(us, 2), "useful_tflops": round(fl / us / 1e6, 2),
                                    "issued_tflops": round(issued / us / 1e6, 2),
                                    "issued_frac_of_bf16": round(issued / us / 1e6 / bf16_peak, 4)}
        del W
    assert efg.device_error() == 0
    return out


def run_profile(args):
    """A few plain launches for ncu (no CPU legs): --profile q8 -> config 1 (Q8_0 32000x2048),
    q4 -> config 0 (Q4_0 5632x2048), q4big -> Q4_0 65536x8192 (302 MB, half of config 4's
    rows, on the tensor-core kernel), gemm -> config 3 (5632x2048, B=64), decode / decode_persistent -> config 2, four
    single-token forwards in each decode mode, prefill / batch -> config 2's batched paths (the 23-token prompt, one
    32-sequence step), the second run only between cudaProfilerStart and Stop."""
    import torch

    import edgeforge_b200 as efg

    torch.cuda.set_device(0)
    if args.profile in ("prefill", "batch"):
        # config 2's batched paths: the 23-token prompt through efg_decoder_prefill, or one
        # step of 32 sequences through efg_decoder_step_slots; the second run is bracketed by
        # cudaProfilerStart/Stop (ncu --profile-from-start off captures only that run)
        prompt = np.random.default_rng(2).integers(0, 32000, 23).astype(np.int32)
        with efg.Decoder(decode_model(), 64) as dec:
            if args.profile == "batch":
                S = 32
                dec.set_slots(S)
                slots = np.arange(S, dtype=np.int32)
                toks = prompt[:S] if S <= len(prompt) else np.resize(prompt, S)
                for t in range(2):
                    if t == 1:
                        torch.cuda.synchronize()
                        torch.cuda.profiler.start()
                    _, toks = dec.step_slots(slots, toks, np.full(S, t, np.int32), compute_logits=False)
            else:
                for t in range(2):
                    if t == 1:
                        torch.cuda.synchronize()
                        torch.cuda.profiler.start()
                    dec.prefill(prompt, 0)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        assert efg.device_error() == 0
        print(json.dumps({"profile": args.profile, "rows": 32 if args.profile == "batch" else len(prompt)}))
        return 0
    if args.profile == "gemm":  # config 3, M=5632 K=2048 B=64: 3 calls
        M, K, B = 5632, 2048, 64
        W = make_weights(efg, torch, Q4_0, M, K, 1, seed=7)[0]
        X = torch.randn(B, K, device="cuda")
        Y = torch.empty(B, M, device="cuda")
        for _ in range(3):
            efg.gemm_q4_0(Y, W, X, M, K, B)
        torch.cuda.synchronize()
        assert efg.device_error() == 0
        print(json.dumps({"profile": "gemm", "M": M, "K": K, "B": B, "calls": 3}))
        return 0
    if args.profile in ("decode", "decode_persistent"):  # config 2: 4 forwards, one token each
        with efg.Decoder(decode_model(), 64) as dec:
            dec.persistent = args.profile == "decode_persistent"
            for i in range(4):
                dec.forward(3 + i, i)
        assert efg.device_error() == 0
        print(json.dumps({"profile": args.profile, "forwards": 4}))
        return 0
    qt, rows, cols, copies = {"q8": (Q8_0, ROWS, COLS, 3), "q4": (Q4_0, 5632, 2048, 24),
                              "q4big": (Q4_0, 65536, 8192, 1)}[args.profile]
    Ws = make_weights(efg, torch, qt, rows, cols, copies, seed=1)
    x = torch.randn(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    for i in range(2 * copies + 3):
        efg.matvec(qt, y, Ws[i % copies], x, rows, cols)
    torch.cuda.synchronize()
    assert efg.device_error() == 0
    print(json.dumps({"profile": args.profile, "rows": rows, "cols": cols, "launches": 2 * copies + 3,
                      "bytes_per_launch": algo_bytes(qt, rows, cols)}))
    return 0


_RESULT_FD = None


def emit(line: dict) -> None:
    """Writes the JSON result line to the process's original stdout. Everything else that
    the run prints (libraries included, e.g. NCCL's version banner) goes to stderr, so
    stdout carries exactly one JSON line."""
    out = os.fdopen(os.dup(_RESULT_FD), "w") if _RESULT_FD is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=6000)
    ap.add_argument("--warmup", type=int, default=60)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-2 decode measurement")
    ap.add_argument("--no-sharded", action="store_true", help="skip the config-4 sharded matvec measurement")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-3 GEMM measurement")
    ap.add_argument("--profile", choices=["q8", "q4", "q4big", "gemm", "decode", "decode_persistent", "prefill", "batch"],
                    help="a few plain launches for ncu")
    args = ap.parse_args()
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)  # the JSON line goes here; fd 1 then points at stderr
    os.dup2(2, 1)
    if args.profile:
        return run_profile(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
