#!/usr/bin/env python3
"""Benchmark of the packed matrix-product path (one JSON line on rank 0).

Workload (the headline benchmark's configuration 4): the Q4_0 matvec W x with W 131072 x 8192
drawn N(0, 0.02) and quantized with the reference's Q4_0 rule (bit-exact GPU quantizer,
603,979,776 packed bytes), x ~ N(0, 1), row-sharded over the job's GPUs: rank r holds the
rows [R r / N, R (r + 1) / N) (ThreadPool::chunk_begin's split) and every rank ends the step
with all 131072 outputs (efg_matvec_sharded). A step is one sharded matvec. Strong scaling:
the matrix is the same at every N. Enough rotating copies of each rank's shard are used that
they exceed twice the 126 MB L2, so every step streams its weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W]      # our B200 path
  python bench.py --impl reference                           # the reference's CPU path

Metric: algorithmic bytes per step (packed W + x + y = 604,536,832 B) / time, in GB/s.
value: device time of K steps (CUDA events around CUDA graphs of the C-ABI calls, max over
ranks). e2e: the same steps through the C ABI with host buffers, every step (wall clock, max
over ranks): on one GPU efg_host_matvec (x from page-locked memory, y stored by the kernel into
page-locked memory, W registered once as at model load); on several, x copied in from
page-locked memory, efg_matvec_sharded, y read back to page-locked memory. After timing, every rank checks that its slice of the gathered y is bit-identical
to its own local matvec and that all ranks hold the same y ("verified").
Extras at N = 1: configs 0 (Q4_0 5632 x 2048), 1 (Q8_0 32000 x 2048 and its quantize round
trip), 2 (decode), 3 (GEMM); at every N: the row-sharded lm_head with its distributed argmax.
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

ROWS, COLS = 32000, 2048          # config 1 (extra)
ROWS4, COLS4 = 131072, 8192       # config 4 (headline)
Q8_0, Q4_0 = 3, 4
N_COPIES = 6
METRIC = "Q4_0 matvec HBM GB/s (config 4: 131072x8192, row-sharded over the job's GPUs)"
L2_BYTES = 126 * 1024 * 1024


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
def physical_cores():
    """Physical cores the way the reference's sysinfo counts them on Linux
    (src/sysinfo.cpp:177-195): distinct (physical id, core id) pairs in /proc/cpuinfo."""
    cores, phys = set(), "0"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "physical id":
                    phys = v
                elif k == "core id":
                    cores.add((phys, v))
    except OSError:
        return None
    return len(cores) or None


def host_threads():
    """Threads for the CPU legs: every logical CPU this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_info(threads):
    return {"cores": threads, "physical_cores": physical_cores(), "logical_cpus": os.cpu_count()}


def cpu_reference_matvec(qt, Ws, x, rows, cols, seconds=None, steps=None, warmup=1, cap_seconds=150.0):
    """The reference's AVX2 matvec (kern::matvec + ThreadPool, oracle/_ref, its own sources)
    on the host cores over the packed matrices Ws in rotation. Runs `steps` matvecs (or for
    `seconds` when steps is None), never longer than cap_seconds. Returns (GB/s, threads,
    matvecs, seconds)."""
    from oracle.oracle import Reference

    ref = Reference()
    threads = host_threads()
    y = np.zeros(rows, np.float32)
    with ref.pool(threads) as pool:
        for i in range(max(warmup, len(Ws))):  # warm-up: page in every copy
            ref.matvec_backend(qt, Ws[i % len(Ws)], x, rows, avx2=True, pool=pool, y=y)
        n, t0 = 0, time.perf_counter()
        while True:
            ref.matvec_backend(qt, Ws[n % len(Ws)], x, rows, avx2=True, pool=pool, y=y)
            n += 1
            el = time.perf_counter() - t0
            if (steps is not None and n >= steps) or (steps is None and el >= seconds) or el >= cap_seconds:
                break
    return algo_bytes(qt, rows, cols) * n / el / 1e9, threads, n, el


def host_config4_weights(threads):
    """Config 4's matrix on the host: 131072 x 8192 weights ~ N(0, 0.02) (numpy, seed 0) quantized
    to Q4_0 by the reference's own quantize_rows (MSE search), 4096 rows at a time."""
    from oracle.oracle import Reference

    ref = Reference()
    rng = np.random.default_rng(0)
    W = np.empty((ROWS4, COLS4 // 32 * 18), np.uint8)
    with ref.pool(threads) as pool:
        for r0 in range(0, ROWS4, 4096):
            X = rng.standard_normal((4096, COLS4), dtype=np.float32) * np.float32(0.02)
            W[r0:r0 + 4096] = ref.quantize_rows(Q4_0, X, pool=pool)
    return W


def run_reference_arm(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return 0
    if not (ROOT / "oracle" / "_ref" / "libefref.so").exists():
        emit({"impl": "reference", "unavailable": "oracle/_ref/libefref.so was not built"})
        return 0
    threads = host_threads()
    W = host_config4_weights(threads)
    x = np.random.default_rng(1).standard_normal(COLS4).astype(np.float32)
    # W untimed warm-up steps, then K timed steps, each one CPU matvec of the whole matrix
    # (stopped after 150 s, in which case "steps" reports the count actually timed)
    gbs, threads, n, el = cpu_reference_matvec(Q4_0, [W], x, ROWS4, COLS4, steps=args.steps, warmup=args.warmup)
    args.steps = n
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el / n * 1e3, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (Q4_0 weights)", "data": "synthetic (seeded N(0,0.02) W, N(0,1) x)",
        "config": {"workload": "config4_q4_0_matvec_131072x8192", "rows": ROWS4, "cols": COLS4,
                   "l2": "604 MB matrix, far larger than the host's last-level cache"},
        "impl": "reference",
        "cpu_baseline": dict(value=round(gbs, 3), unit="GB/s", kind="reference", **cpu_info(threads),
                             sample=f"{n} matvecs of the whole 604 MB matrix by the reference AVX2 kernel, "
                                    f"ThreadPool({threads})"),
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


def config4_shard(efg, torch, begin, count, piece=8192):
    """This rank's rows [begin, begin + count) of config 4's matrix, quantized on the device.
    The matrix is drawn in 8192-row pieces, piece i from its own seeded generator, so every
    rank at every N sees the same matrix."""
    rb = COLS4 // 32 * 18
    W = torch.empty(max(count, 1) * rb, dtype=torch.uint8, device="cuda")
    for p0 in range(begin // piece * piece, begin + count, piece):
        g = torch.Generator(device="cuda").manual_seed(1000 + p0 // piece)
        X = torch.randn(piece, COLS4, generator=g, device="cuda") * 0.02
        lo, hi = max(p0, begin), min(p0 + piece, begin + count)
        efg.quantize_rows(Q4_0, X[lo - p0:hi - p0].contiguous(), hi - lo, COLS4, W[(lo - begin) * rb:], True)
        del X
    return W


def graphs_of(torch, fn, steps, warmup, chunk=60):
    """CUDA graphs of `fn(i)` for i in a step range: (full graph of `chunk` steps, graph of the
    remainder or None, chunk), after `warmup` plain calls outside capture (lazy set-up)."""
    chunk = max(1, min(chunk, steps))
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def cap(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for i in range(n):
                fn(i)
        return g

    g_full = cap(chunk)
    rem = steps % chunk
    g_rem = cap(rem) if rem else None
    torch.cuda.synchronize()
    return g_full, g_rem, chunk


def replay_timed(torch, g_full, g_rem, chunk, steps, barrier, world, clocks=None):
    """Device time (ms) of exactly `steps` steps replayed from the graphs, bracketed by a
    barrier and a device synchronize on both sides; the max over ranks. The clock sampler
    starts before the barrier: its first NVML query takes a different time on every rank,
    and a rank that starts early waits inside the first step for the others."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        barrier()
        start.record()
        for _ in range(steps // chunk):
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
    return ms


def time_calls(torch, fn, steps, warmup, barrier, world):
    """ms per call of fn(i): CUDA graphs of the calls when they can be captured, otherwise
    (a library that refuses capture) the same calls launched one by one; max over ranks."""
    try:
        gf, gr, ch = graphs_of(torch, fn, steps, warmup)
    except Exception:  # noqa: BLE001 - measured eagerly instead
        torch.cuda.synchronize()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for i in range(steps):
            fn(i)
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms / steps
    gf.replay()
    ms = replay_timed(torch, gf, gr, ch, steps, barrier, world) / steps
    del gf, gr
    return ms


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def y_digest(torch, y):
    """An order-sensitive 64-bit digest of y's bits (equal digests on all ranks = same y)."""
    v = y.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    w = torch.arange(1, v.numel() + 1, device=y.device, dtype=torch.int64) % 1000003 + 1
    return int((v * w).sum().item())


def config4_headline(torch, efg, args, world, rank, local, hbm_peak, barrier):
    """Config 4 row-sharded over the job's GPUs: device time of K steps, the local matvec
    alone, verification of the gathered y, and the host-buffer e2e loop."""
    b, c = efg.shard_rows(ROWS4, world, rank)
    rb = COLS4 // 32 * 18
    shard_bytes = c * rb
    copies = max(1, -(-2 * L2_BYTES // max(shard_bytes, 1)))  # rotating shards > 2x L2
    W0 = config4_shard(efg, torch, b, c)
    Ws = [W0] + [W0.clone() for _ in range(copies - 1)]
    x = torch.randn(COLS4, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda")
    y = torch.empty(ROWS4, device="cuda")
    comm = efg.Comm.from_torch() if world > 1 else efg.Comm(efg.Comm.unique_id(), 1, 0)
    gather = "none (one rank)"
    ms_nccl = None
    registered = False
    W_reg = None  # the host copy of W registered for the one-GPU e2e loop
    try:
        if world > 1:
            # the same step with y not registered: the slices go through ncclAllGather (for
            # comparison; device time of CUDA graphs of the calls)
            y_n = torch.empty(ROWS4, device="cuda")
            ms_nccl = time_calls(torch, lambda i: efg.matvec_sharded(Q4_0, y_n, Ws[i % copies], x, ROWS4, COLS4, comm),
                                 args.steps, args.warmup, barrier, world)
            del y_n
            try:
                comm.register(y)
                registered = True
                gather = "in-kernel: every CTA stores its rows into each peer's y over NVLink (efg_comm_register)"
            except efg.EdgeForgeError as e:  # every rank gets the same outcome
                gather = f"ncclAllGather in place (registration failed: {e})"

        def step(i):
            efg.matvec_sharded(Q4_0, y, Ws[i % copies], x, ROWS4, COLS4, comm)

        # W warm-up steps as plain calls, then the graphs are captured and replayed once
        # untimed (a graph's first launch uploads it to the device)
        g_full, g_rem, chunk = graphs_of(torch, step, args.steps, args.warmup)
        g_full.replay()
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        ms = replay_timed(torch, g_full, g_rem, chunk, args.steps, barrier, world, clocks)
        del g_full, g_rem

        # the local matvec alone (this rank's rows, no exchange): the dominant kernel
        yl = y[b:b + c]

        def local_step(i):
            efg.matvec(Q4_0, yl, Ws[i % copies], x, c, COLS4)

        lf, lr, lc = graphs_of(torch, local_step, args.steps, args.warmup)
        lf.replay()
        ms_local = replay_timed(torch, lf, lr, lc, args.steps, barrier, world)
        del lf, lr
        efg.set_q4_mma(False)  # the same local matvec on the CUDA-core kernel, for comparison
        try:
            ms_local_cc = time_calls(torch, local_step, args.steps, args.warmup, barrier, world) * args.steps
        finally:
            efg.set_q4_mma(True)

        # verification: this rank's slice of the gathered y equals its own local matvec bit for
        # bit, and every rank holds the same y
        y.fill_(float("nan"))
        efg.matvec_sharded(Q4_0, y, Ws[0], x, ROWS4, COLS4, comm)
        mine = torch.empty(max(c, 1), device="cuda")
        efg.matvec(Q4_0, mine, Ws[0], x, c, COLS4)
        torch.cuda.synchronize()
        ok = bool(torch.equal(y[b:b + c], mine[:c])) and not bool(torch.isnan(y).any())
        dg = y_digest(torch, y)
        if world > 1:
            t = torch.tensor([1 if ok else 0, dg, -dg], device="cuda", dtype=torch.int64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            ok = bool(t[0].item() == 1) and int(t[1].item()) == -int(t[2].item()) == dg
        # e2e: x from page-locked host memory in, the C-ABI call, y back in page-locked memory,
        # every step. One GPU: efg_host_matvec, the reference-facing host-buffer call, on W
        # registered once as a model load does (the matrix is 604 MB, far above L2); its
        # kernel stores y into the page-locked buffer as rows finish. Several GPUs: the
        # sharded call with explicit copies.
        x_h = x.cpu().pin_memory()
        y_h = torch.empty(ROWS4).pin_memory()
        x_d = torch.empty_like(x)
        cur = torch.cuda.current_stream()
        if world == 1:
            W_reg = Ws[0].cpu().numpy()
            efg.host_register_weights(W_reg)
            x_hn, y_hn = x_h.numpy(), y_h.numpy()

            def e2e_step(i):
                efg.host_matvec(Q4_0, W_reg, x_hn, ROWS4, y=y_hn)
        else:
            def e2e_step(i):
                x_d.copy_(x_h, non_blocking=True)
                efg.matvec_sharded(Q4_0, y, Ws[i % copies], x_d, ROWS4, COLS4, comm)
                y_h.copy_(y, non_blocking=True)
                cur.synchronize()

        for i in range(args.warmup):
            e2e_step(i)
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i)
        el = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([el], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            el = float(t.item())
        else:  # the host call's y is the device call's y, bit for bit
            ok = ok and bool(np.array_equal(y_h.numpy(), mine[:c].cpu().numpy()))
        assert efg.device_error() == 0
    finally:
        if W_reg is not None:
            efg.host_unregister_weights(W_reg)
        if registered:
            comm.deregister(y)
        comm.close()
    total = algo_bytes(Q4_0, ROWS4, COLS4)
    local_bytes = shard_bytes + 4 * COLS4 + 4 * c
    return {"ms": ms, "ms_local": ms_local, "el_e2e": el, "total": total, "local_bytes": local_bytes,
            "ms_nccl": ms_nccl, "ms_local_cc": ms_local_cc,
            "rows_per_rank": c, "copies": copies, "verified": ok, "gather": gather, "clocks": clocks.summary(),
            "W_host": W_reg if (world == 1 and not args.no_cpu_baseline) else None,
            "x_host": x.cpu().numpy()}


def config1_extra(torch, efg, hbm_peak, steps=2000, warmup=60):
    """Config 1: the Q8_0 matvec at lm_head shape (32000 x 2048), 6 rotating W copies (418 MB),
    device time of CUDA graphs of C-ABI launches; e2e through efg_host_matvec (page-locked x in
    and y out every call, W registered resident once, like a model load)."""
    Ws = make_weights(efg, torch, Q8_0, ROWS, COLS, N_COPIES, seed=1)
    x = torch.randn(COLS, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    y = torch.empty(ROWS, device="cuda")

    def step(i):
        efg.matvec(Q8_0, y, Ws[i % N_COPIES], x, ROWS, COLS)

    g_full, g_rem, chunk = graphs_of(torch, step, steps, warmup)
    g_full.replay()
    ms = replay_timed(torch, g_full, g_rem, chunk, steps, torch.cuda.synchronize, 1) / steps
    del g_full, g_rem
    nbytes = algo_bytes(Q8_0, ROWS, COLS)
    x_h = torch.empty(COLS, dtype=torch.float32).pin_memory().numpy()
    y_h = torch.empty(ROWS, dtype=torch.float32).pin_memory().numpy()
    x_h[:] = x.cpu().numpy()
    Whs = [Ws[0].cpu().numpy() for _ in range(N_COPIES)]
    for w in Whs:
        efg.host_register_weights(w)
    for i in range(10):
        efg.host_matvec(Q8_0, Whs[i % N_COPIES], x_h, ROWS, y=y_h)
    t0 = time.perf_counter()
    n = 500
    for i in range(n):
        efg.host_matvec(Q8_0, Whs[i % N_COPIES], x_h, ROWS, y=y_h)
    el = (time.perf_counter() - t0) / n
    efg.host_release_weights()
    assert efg.device_error() == 0
    return {"us_per_launch": round(ms * 1e3, 3), "gbs": round(nbytes / ms / 1e6, 1),
            "frac_of_hbm": round(nbytes / ms / 1e6 / hbm_peak, 4), "bytes_per_launch": nbytes, "copies": N_COPIES,
            "e2e_us_per_call": round(el * 1e6, 2), "e2e_gbs": round(nbytes / el / 1e9, 1),
            "e2e_api": "efg_host_matvec (page-locked x, y; W registered)"}


def config0_extra(torch, efg, hbm_peak, x_seed=2, launches=1280):
    """Config 0: the Q4_0 matvec at TinyLlama gate_proj shape (5632 x 2048), 64 rotating copies
    (415 MB), launched back to back in CUDA graphs (weight prefetch on, PDL)."""
    rows, cols, copies = 5632, 2048, 64
    W4 = make_weights(efg, torch, Q4_0, rows, cols, copies, seed=3)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(x_seed), device="cuda")
    y4 = torch.empty(rows, device="cuda")

    def step(i):
        efg.matvec(Q4_0, y4, W4[i % copies], x, rows, cols)

    g, gr, c = graphs_of(torch, step, launches, 64, chunk=640)
    g.replay()
    ms = replay_timed(torch, g, gr, c, launches, torch.cuda.synchronize, 1) / launches
    del g, gr

    def step_hot(i):  # one copy: W stays in L2 (the hot-cache number)
        efg.matvec(Q4_0, y4, W4[0], x, rows, cols)

    g, gr, c = graphs_of(torch, step_hot, launches, 64, chunk=640)
    g.replay()
    ms_hot = replay_timed(torch, g, gr, c, launches, torch.cuda.synchronize, 1) / launches
    del g, gr
    efg.set_q4_mma(False)  # the same launches on the CUDA-core kernel, for comparison
    try:
        g, gr, c = graphs_of(torch, step, launches, 64, chunk=640)
        g.replay()
        ms_cc = replay_timed(torch, g, gr, c, launches, torch.cuda.synchronize, 1) / launches
        del g, gr
    finally:
        efg.set_q4_mma(True)
    # Independent matvecs (no data dependence between them) on several streams at once, each
    # stream a CUDA graph of its own chain over its own share of the weight copies: the
    # kernel's throughput when it is not waiting on the launch before it (multi-sequence /
    # multi-model serving).
    main = torch.cuda.current_stream()

    def independent(n_streams):
        per, share = launches // n_streams, copies // n_streams
        ys = [torch.empty(rows, device="cuda") for _ in range(n_streams)]
        streams = [torch.cuda.Stream() for _ in range(n_streams)]
        graphs = []
        for k, st in enumerate(streams):
            def fn(i, k=k):
                efg.matvec(Q4_0, ys[k], W4[k * share + i % share], x, rows, cols)
            for i in range(8):
                fn(i)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(st), torch.cuda.graph(g, stream=st):
                for i in range(per):
                    fn(i)
            graphs.append(g)
        torch.cuda.synchronize()

        def run_all():
            ev0 = torch.cuda.Event()
            ev0.record(main)
            ends = []
            for st, g in zip(streams, graphs):
                st.wait_event(ev0)
                with torch.cuda.stream(st):
                    g.replay()
                e = torch.cuda.Event()
                e.record(st)
                ends.append(e)
            for e in ends:
                main.wait_event(e)

        run_all()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(main)
        run_all()
        s1.record(main)
        torch.cuda.synchronize()
        del graphs
        return s0.elapsed_time(s1) / (per * n_streams), per * n_streams

    ind = {n: independent(n) for n in (4, 8)}
    del W4
    nb = algo_bytes(Q4_0, rows, cols)
    return {"gbs": round(nb / ms / 1e6, 1), "frac_of_hbm": round(nb / ms / 1e6 / hbm_peak, 4),
            "measure": "dependent chain: each launch waits for the one before it (as in a decode step)",
            **{f"independent_{n}_streams": {"gbs": round(nb / m / 1e6, 1), "frac_of_hbm": round(nb / m / 1e6 / hbm_peak, 4),
                                             "us_per_launch": round(m * 1e3, 3), "launches": k}
               for n, (m, k) in ind.items()},
            "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": nb, "copies": copies,
            "hot_cache_us_per_launch": round(ms_hot * 1e3, 3),
            "kernel": "small-matrix integer tensor-core kernel (weights fetched ahead, next launch co-resident)",
            "us_per_launch_cuda_cores": round(ms_cc * 1e3, 3),
            "frac_of_hbm_cuda_cores": round(nb / ms_cc / 1e6 / hbm_peak, 4)}


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

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # Extras run first; besides their own figures they bring the GPU to its working clocks
    # before the headline's timed region.
    extra = {}
    if args.no_extras:
        args.no_sharded = True
    if world == 1 and not args.no_extras:
        extra["config1_q8_0_matvec_32000x2048"] = config1_extra(torch, efg, hbm_peak)
        extra["config0_q4_0_matvec_5632x2048"] = config0_extra(torch, efg, hbm_peak)
        if not args.no_decode:
            extra["config2_decode_tinyllama"] = decode_extra(hbm_peak, with_cpu=not args.no_cpu_baseline)
        if not args.no_gemm:
            extra["config3_gemm_q4_0"] = gemm_extra(torch, efg, bf16_peak)
            extra["config1_quantize_round_trip"] = quant_extra(torch, efg, hbm_peak)
    if not args.no_sharded:
        extra["lm_head_sharded_argmax_32000x2048"] = lm_head_extra(torch, efg, world, rank, barrier)

    h = config4_headline(torch, efg, args, world, rank, local, hbm_peak, barrier)
    ms_step = h["ms"] / args.steps
    value = h["total"] * args.steps / (h["ms"] / 1e3) / 1e9
    ms_local = h["ms_local"] / args.steps
    achieved = h["local_bytes"] / (ms_local / 1e3) / 1e9  # the local matvec kernel, per launch
    e2e = h["total"] * args.steps / h["el_e2e"] / 1e9

    # DRAM bytes per launch of this kernel from the committed ncu capture summary
    traffic = None
    tpath = ROOT / "profiles" / "matvec_q4_0_config4.json"
    if tpath.exists():
        tr = json.loads(tpath.read_text())
        traffic = tr.get("dram_bytes_per_launch_scaled", {}).get(str(h["rows_per_rank"]))

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and (ROOT / "oracle" / "_ref" / "libefref.so").exists():
            gbs_c, thr, n_c, el_c = cpu_reference_matvec(Q4_0, [h["W_host"].reshape(ROWS4, -1)], h["x_host"],
                                                         ROWS4, COLS4, seconds=args.cpu_seconds)
            cpu = dict(value=round(gbs_c, 3), unit="GB/s", kind="reference", **cpu_info(thr),
                       sample=f"{n_c} matvecs ({el_c:.1f} s) of the whole 604 MB config-4 matrix by the reference "
                              f"AVX2 kernel + ThreadPool({thr})")
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (Q4_0 weights)", "data": "synthetic (seeded N(0,0.02) W, N(0,1) x)",
            "config": {"workload": "config4_q4_0_matvec_131072x8192", "rows": ROWS4, "cols": COLS4,
                       "rows_per_rank": h["rows_per_rank"], "copies_per_rank": h["copies"],
                       "l2": f"inputs larger than L2: {h['copies']} rotating copies of each rank's shard "
                             f"({h['copies'] * h['rows_per_rank'] * COLS4 // 32 * 18 / 1e6:.0f} MB)",
                       "launch": "CUDA graphs of C-ABI calls, weight prefetch on (PDL)",
                       "gather": h["gather"],
                       "parallelism": f"row-sharded x{world}" if world > 1 else "single GPU"},
            "verified": h["verified"],
            "sharded_step_us": {"this_run": round(ms_step * 1e3, 3), "local_matvec_alone": round(ms_local * 1e3, 3),
                                "local_matvec_alone_cuda_cores": round(h["ms_local_cc"] / args.steps * 1e3, 3),
                                "with_ncclAllGather": round(h["ms_nccl"] * 1e3, 3) if h["ms_nccl"] else None},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": h["local_bytes"],
                         "kernel": "local Q4_0 matvec (integer tensor-core MMA), this rank's rows",
                         "kernel_us": round(ms_local * 1e3, 3)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * COLS4,
                    "d2h_bytes_per_step": 4 * ROWS4,
                    "api": ("efg_host_matvec (C ABI, host pointers): x copied in from page-locked memory, the kernel "
                            "storing y into page-locked memory, W registered once" if world == 1 else
                            "efg_matvec_sharded (C ABI) with x copied in from and y read back to page-locked host "
                            "memory every step")},
            "gpu_launches": args.steps,
            "clocks": h["clocks"],
            "extra": extra,
        }
        emit(line)
    if world > 1:
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


def lm_head_extra(torch, efg, world, rank, barrier, steps=200, warmup=10, rows=32000, cols=2048):
    """The decode step's last operation with lm_head (Q8_0 32000 x 2048) row-sharded over the
    job's GPUs: this rank's logits with the final RMSNorm fused, then the argmax over all
    ranks (efg_lm_head_argmax_sharded). Device time per call (CUDA graphs, max over ranks;
    strong scaling), at N > 1 with a buffer registered on the communicator (the pairs travel
    by peer stores inside the argmax launch) and, for comparison, through NCCL. Verified: the
    token on every rank equals the argmax of all ranks' logits gathered afterwards."""
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
    try:
        def step(i):
            efg.lm_head_argmax_sharded(Q8_0, logits, tok, shard, x, nw, 1e-5, rows, cols, comm)

        ms_nccl = None
        reg = None
        if world > 1:
            ms_nccl = time_calls(torch, step, steps, warmup, barrier, world)
            reg = torch.zeros(64, device="cuda")
            comm.register(reg)
        ms = time_calls(torch, step, steps, warmup, barrier, world)
        tok.fill_(-1)
        step(0)
        torch.cuda.synchronize()
        if world > 1 and rows % world == 0:
            full = torch.empty(rows, device="cuda")
            torch.distributed.all_gather_into_tensor(full, logits[:c].contiguous())
        elif world > 1:
            parts = [torch.empty(efg.shard_rows(rows, world, r)[1], device="cuda") for r in range(world)]
            torch.distributed.all_gather(parts, logits[:c].contiguous())
            full = torch.cat(parts)
        else:
            full = logits[:c]
        want = efg.argmax(full)
        torch.cuda.synchronize()
        ok = int(tok.item()) == int(want.item())
        if world > 1:
            t = torch.tensor([1 if ok else 0], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            ok = bool(t.item() == 1)
        assert efg.device_error() == 0
        if reg is not None:
            comm.deregister(reg)
    finally:
        comm.close()
    return {"us_per_call": round(ms * 1e3, 3), "ranks": world, "rows_per_rank": c, "token": int(tok.item()),
            "verified": ok, "scaling": "strong",
            "exchange": "peer stores in the argmax launch" if world > 1 else "none (one rank)",
            "us_per_call_nccl": round(ms_nccl * 1e3, 3) if ms_nccl is not None else None}


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
    torch.cuda.empty_cache()  # the FP32 source of the weights is freed (less device memory under ncu)
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
    ap.add_argument("--no-sharded", action="store_true", help="skip the row-sharded lm_head extra")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-3 GEMM measurement")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the headline (configs 0-3 and the lm_head extra skipped; for the ncu launch list)")
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
