#!/usr/bin/env python3
"""Benchmark of the B200 per-layer kernels (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c5|c1|c2|c3|c4|g1|g2|v1|...] [--graph auto|on|off]

A step is one decoder layer's elementwise chain over one batch (runner.LayerChain):
fused residual-add+RMSNorm, fused q/k RMSNorm+RoPE, fused residual-add+RMSNorm,
SwiGLU -- BF16 storage, FP32 math -- on inputs resident in HBM. The default
workload is config c5: the Qwen3-1.7B chain (hidden 2048, FFN 6144, 16/8 heads of
128) over 2 097 152 tokens, row-sharded in contiguous blocks across the N GPUs with
no collective ("scaling": "strong"; N = 1 holds all of it, ~116 GB). `value` is
tokens/s over all GPUs (the slowest rank's CUDA-event time); `per_rank` has every
rank's per-kernel GB/s; the roofline object reports the dominant kernel's achieved
HBM GB/s from live CUDA events. At N = 1 the line also carries `other_shapes`: the
c2 chain (64 x 1024 tokens) with both SwiGLU call forms, the L2-resident c1 and c3
(decode at random positions, CUDA graph) and the c4 SnakeBeta stages, each with its
own per-kernel table and roofline. --config c2 runs the 65536-token batch per GPU
("weak").

--config g1/g2 time the decode step's fused linear path (GEMVs with RMSNorm prologue
and residual / SwiGLU epilogues) through 28 layers; --config v1 times the vocoder's
12 BigVGAN ResUnits on tcgen05 tensor cores (roofline: TF32 tensor throughput).

--impl reference times the reference's CPU implementation of the same chain
(the oracle restatement of the absent qwen-asr C, built at the reference's
optimisation tier with OpenMP over all host cores) on a bounded sample of rows.
Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "local-ai-server_b200"))

METRIC = "achieved HBM GB/s (% of peak) and rows/sec per fused kernel at 1/2/4/8 B200"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks() -> tuple[float, str]:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def load_traffic() -> dict:
    """Per-launch DRAM bytes from the committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of one GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------- CPU side
def cpu_chain_rate(cfg, rows: int, min_seconds: float, steps: int | None = None,
                   warmup: int = 1, threads: int | None = None) -> dict:
    """The reference's FP32 chain on host cores (oracle/_build/liblai_cpuref.so).

    Returns rows/s. Either `steps` timed passes, or passes until `min_seconds`.
    threads: OpenMP threads (default: every core this process may run on).
    """
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("liblai_cpuref.so")
    lib.oracle_set_threads(threads or len(os.sched_getaffinity(0)))  # whatever OMP_* says
    rng = np.random.default_rng(5)
    D, I, hd = cfg.dim, cfg.inter, cfg.head_dim
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    x, da, df, y = f(rows, D), f(rows, D), f(rows, D), np.empty((rows, D), np.float32)
    q, k, gu = f(rows, cfg.n_q * hd), f(rows, cfg.n_kv * hd), f(rows, 2 * I)
    w_in = (1 + 0.02 * f(D)).astype(np.float32)
    w_post = (1 + 0.02 * f(D)).astype(np.float32)
    wq = (1 + 0.02 * f(hd)).astype(np.float32)
    wk = (1 + 0.02 * f(hd)).astype(np.float32)
    pos = np.arange(rows) % cfg.pos_period
    ct, st = oracle.compute_rope_neox(np.arange(cfg.pos_period), hd, cfg.theta)
    c_rows, s_rows = np.ascontiguousarray(ct[pos]), np.ascontiguousarray(st[pos])
    P = oracle.ptr
    args = [P(x), P(da), P(df), P(y), P(q), P(k), P(gu), P(w_in), P(w_post), P(wq), P(wk),
            P(c_rows), P(s_rows), rows, D, cfg.n_q, cfg.n_kv, hd, I, cfg.eps]
    for _ in range(warmup):
        lib.oracle_layer_chain_f32(*args)
    n, t0 = 0, time.perf_counter()
    while True:
        lib.oracle_layer_chain_f32(*args)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
            break
    return {"rows_per_s": rows * n / el, "threads": lib.oracle_num_threads(), "passes": n,
            "seconds": el}


def cpu_decode_rate(cfg, min_seconds: float) -> dict:
    """One layer's decode linear path on host cores (oracle/_build/liblai_cpuref.so: the
    restated linear_bf16 and elementwise ops, OpenMP), M = cfg.m tokens per pass."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("liblai_cpuref.so")
    lib.oracle_set_threads(len(os.sched_getaffinity(0)))
    rng = np.random.default_rng(8)
    D, I, M = cfg.dim, cfg.inter, cfg.m
    qkv_n = cfg.q_dim + 2 * cfg.kv_dim
    wb = lambda n, k: oracle.f32_to_bf16_bits((rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32))  # noqa: E731
    Wqkv, Wo, Wgu, Wd = wb(qkv_n, D), wb(D, cfg.q_dim), wb(2 * I, D), wb(D, I)
    x = rng.standard_normal((M, D), dtype=np.float32)
    attn = rng.standard_normal((M, cfg.q_dim), dtype=np.float32)
    w_in = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    w_post = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)

    def step():
        xn = oracle.rms_norm(x, w_in, cfg.eps, lib)
        oracle.linear_bf16(xn, Wqkv, lib)
        o = oracle.linear_bf16(attn, Wo, lib)
        x2 = oracle.add_inplace(x, o, lib)
        gu = oracle.linear_bf16(oracle.rms_norm(x2, w_post, cfg.eps, lib), Wgu, lib)
        act = oracle.swiglu_multiply(gu, I, lib)
        oracle.add_inplace(x2, oracle.linear_bf16(act, Wd, lib), lib)

    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    # one layer per pass (its weights stay cache-warm, favouring the CPU); a decode
    # step runs cfg.layers of them
    return {"rows_per_s": M * n / el / cfg.layers, "threads": lib.oracle_num_threads(),
            "passes": n, "seconds": el}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_snake_rate(stages, batch: int, min_seconds: float, steps: int | None = None,
                   warmup: int = 1, build: str = "avx2") -> dict:
    """The reference's own voc_snake_beta (oracle/_ref, built from src/tts_vocoder_ops.c as
    shipped: AVX2 fast sin) on host cores: channel ranges of each stage run on a thread
    pool (ctypes releases the GIL). Returns channel-rows/s over one sweep of `stages`."""
    import concurrent.futures as cf

    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load(f"libvoc_ref_{build}.so")
    nthreads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(6)
    data = []
    for c, t in stages:
        x = rng.standard_normal((batch * c, t), dtype=np.float32)
        ea = np.exp(0.1 * rng.standard_normal(c)).astype(np.float32)
        ieb = (1 / np.exp(0.1 * rng.standard_normal(c))).astype(np.float32)
        data.append((x, ea, ieb, c, t))
    F = ctypes.POINTER(ctypes.c_float)

    jobs = []  # (x row pointer, ea pointer, ieb pointer, channels, T): one per (item, chunk)
    for x, ea, ieb, c, t in data:
        per = max(1, c // max(1, nthreads // batch))
        for b_ in range(batch):
            for c0 in range(0, c, per):
                n = min(per, c - c0)
                row = x[b_ * c + c0]
                jobs.append((row.ctypes.data_as(F), ea[c0:].ctypes.data_as(F),
                             ieb[c0:].ctypes.data_as(F), n, t))
    rows = sum(batch * c for _, _, _, c, _ in data)
    with cf.ThreadPoolExecutor(nthreads) as ex:
        def sweep():
            list(ex.map(lambda j: lib.voc_snake_beta(*j), jobs))
        for _ in range(warmup):
            sweep()
        n, t0 = 0, time.perf_counter()
        while True:
            sweep()
            n += 1
            el = time.perf_counter() - t0
            if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
                break
    return {"rows_per_s": rows * n / el, "threads": nthreads, "passes": n, "seconds": el,
            "rows": rows}


def cpu_resunit_rate(stages, batch: int, min_seconds: float, sample_t: int = 4000,
                     steps: int | None = None, warmup: int = 1) -> dict:
    """The reference's ResUnit (run_resunit, src/tts_vocoder.c:540-583) on host cores as
    its USE_BLAS build runs it: voc_snake_beta from the reference's own AVX2 build
    (oracle/_ref) over channel ranges on a thread pool, and voc_conv1d_causal's SGEMM
    formulation (src/tts_vocoder_ops.c:83-125: left padding, then im2col + one SGEMM
    when the column buffer holds <= 1e7 floats at the stage's FULL length, else one
    SGEMM per tap) through numpy's OpenBLAS on all host cores. Each stage runs its three
    units on `sample_t` time rows of one batch item; the measured per-row rate of each
    stage is scaled to the whole step (batch x T rows per stage)."""
    import concurrent.futures as cf

    import numpy as np
    from threadpoolctl import threadpool_limits
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    import runner
    snake = oracle.load("libvoc_ref_avx2.so").voc_snake_beta
    F = ctypes.POINTER(ctypes.c_float)
    nthreads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(8)

    def f32(a):
        return np.ascontiguousarray(a, dtype=np.float32)

    data = []
    for c, t_full in stages:
        units = []
        for d in runner.RESUNIT_DILATIONS:
            units.append({"ea1": f32(np.exp(rng.normal(0, 0.1, c))),
                          "ieb1": f32(1 / np.exp(rng.normal(0, 0.1, c))),
                          "w1": f32(rng.standard_normal((c, c * 7)) / np.sqrt(7 * c)),
                          "b1": f32(rng.normal(0, 0.1, (c, 1))),
                          "ea2": f32(np.exp(rng.normal(0, 0.1, c))),
                          "ieb2": f32(1 / np.exp(rng.normal(0, 0.1, c))),
                          "w2": f32(rng.standard_normal((c, c)) / np.sqrt(c)),
                          "b2": f32(rng.normal(0, 0.1, (c, 1))), "d": d})
        for u in units:  # per-tap weight slices, extracted once like the reference's w_slice
            u["w1_taps"] = [f32(u["w1"].reshape(c, c, 7)[:, :, k]) for k in range(7)]
        data.append((c, t_full, units, f32(rng.standard_normal((c, sample_t)))))

    with cf.ThreadPoolExecutor(nthreads) as pool, threadpool_limits(nthreads):
        def snake_mt(x, ea, ieb):
            c, t = x.shape
            per = max(1, -(-c // nthreads))
            list(pool.map(lambda c0: snake(x[c0].ctypes.data_as(F), ea[c0:].ctypes.data_as(F),
                                           ieb[c0:].ctypes.data_as(F), min(per, c - c0), t),
                          range(0, c, per)))

        def conv7(x, u, im2col):
            c, t = x.shape
            pad = 6 * u["d"]
            padded = np.zeros((c, t + pad), np.float32)
            padded[:, pad:] = x
            if im2col:
                cols = np.empty((c, 7, t), np.float32)
                for k in range(7):
                    cols[:, k, :] = padded[:, k * u["d"]:k * u["d"] + t]
                out = u["w1"] @ cols.reshape(c * 7, t)
            else:
                out = u["w1_taps"][0] @ padded[:, :t]
                for k in range(1, 7):
                    out += u["w1_taps"][k] @ padded[:, k * u["d"]:k * u["d"] + t]
            out += u["b1"]
            return out

        def stage_seconds(c, t_full, units, x0):
            im2col = c * 7 * t_full <= 10_000_000
            x = x0.copy()
            t0 = time.perf_counter()
            for u in units:
                r = x.copy()
                snake_mt(x, u["ea1"], u["ieb1"])
                h = conv7(x, u, im2col)
                snake_mt(h, u["ea2"], u["ieb2"])
                x = u["w2"] @ h
                x += u["b2"]
                x += r
            return time.perf_counter() - t0

        for _ in range(warmup):
            for st in data:
                stage_seconds(*st)
        n, secs = 0, [0.0] * len(data)
        t_start = time.perf_counter()
        while True:
            for i, st in enumerate(data):
                secs[i] += stage_seconds(*st)
            n += 1
            el = time.perf_counter() - t_start
            if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
                break
    step_s = sum(batch * t_full * (secs[i] / n) / sample_t
                 for i, (c, t_full, _, _) in enumerate(data))
    rows = sum(batch * t for _, t in stages)
    return {"rows_per_s": rows / step_s, "step_seconds": step_s, "threads": nthreads,
            "passes": n, "seconds": el, "sample_t": sample_t,
            "per_stage_rows_per_s": {f"{c}x{t}": round(sample_t * n / secs[i], 1)
                                     for i, (c, t, _, _) in enumerate(data)}}


def tf32_peak_tflops(n: int = 8192, reps: int = 10) -> float:
    """cuBLAS FP32 GEMM with TF32 tensor cores (torch.matmul, allow_tf32), n^3, best of
    `reps`: the live denominator for the tensor-bound ResUnit roofline."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        c = a @ b
        best = float("inf")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(reps):
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        torch.cuda.empty_cache()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return 2.0 * n ** 3 / (best / 1000.0) / 1e12


def run_resunits(args) -> None:
    """--config v1: the vocoder's 12 BigVGAN ResUnits on tensor cores (runner.VocResUnits)."""
    import torch
    import torch.distributed as dist
    import runner

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    tf32 = tf32_peak_tflops()
    stages = [(c, t // args.t_div) for c, t in runner.RESUNIT_STAGES]
    work = runner.VocResUnits(stages=stages, passes=args.passes, seed=args.seed + 1000 * rank)
    launches = work.launches(None)
    for _ in range(args.warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    sampler = ClockSampler(phys[local] if local < len(phys) and phys[local] != "" else str(local))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    # v4's front is ~100 launches of a few microseconds: one CUDA graph per step
    total_ms, per = time_launches(launches, args.steps, args.config == "v4", work.kernel_names)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([total_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    assert int(work.err.item()) == 0, "a pipeline wait timed out in the ResUnit kernels"

    hbm_peak, hbm_kind = measured_peaks()
    rows_step = sum(work.rows_per_launch())
    value = rows_step * world * args.steps / (max_ms / 1000.0)
    per_kernel, dominant, dom_total = {}, None, -1.0
    flops, nbytes, rows_pl = work.flops_per_launch(), work.bytes_per_launch(), work.rows_per_launch()
    for j, name in enumerate(work.kernel_names):
        avg_ms = statistics.mean(per[j])
        tfs = flops[j] / (avg_ms / 1000.0) / 1e12
        per_kernel[name] = {"avg_us": round(avg_ms * 1000, 1), "tflops": round(tfs, 1),
                            "tensor_tflops_issued": round(tfs * args.passes, 1),
                            "frac_of_tf32_peak": round(tfs / tf32, 4),
                            "hbm_gbs": round(nbytes[j] / (avg_ms / 1000.0) / 1e9, 1),
                            "rows_per_s": round(rows_pl[j] / (avg_ms / 1000.0), 1),
                            "flops_per_launch": flops[j], "bytes_per_launch": nbytes[j]}
        if sum(per[j]) > dom_total:
            dominant, dom_total = name, sum(per[j])
    d = per_kernel[dominant]
    step_tflops = sum(flops) * args.steps / (total_ms / 1000.0) / 1e12
    roofline = {"bound": "tensor", "kernel": dominant, "achieved": d["tflops"], "peak": round(tf32, 1),
                "unit": "TFLOP/s", "frac": round(d["tflops"] / tf32, 4),
                "peak_source": "cuBLAS FP32 GEMM on TF32 tensor cores (8192^3, best of 10), "
                               "measured in this run",
                "achieved_is": "FP32 convolution flops as the reference counts them; with "
                               f"passes={args.passes} the tensor cores issue {args.passes}x that",
                "traffic": load_traffic().get(f"{dominant}@v1"),
                "algorithmic_bytes_per_launch": d["bytes_per_launch"],
                "hbm_gbs": d["hbm_gbs"], "hbm_frac": round(d["hbm_gbs"] / hbm_peak, 4),
                "step_tflops": round(step_tflops, 1), "step_frac": round(step_tflops / tf32, 4)}

    e2e = None
    if not args.no_e2e:
        # the public device API around host data: per stage, pinned host x -> device,
        # three ResUnits, device -> host, every step
        hosts = [x.cpu().pin_memory() for x in work.x]
        nb = sum(h.numel() * 4 for h in hosts)
        stream = torch.cuda.current_stream()

        def e2e_step():
            for i, f in enumerate(launches):
                work.x[i].copy_(hosts[i], non_blocking=True)
                f()
                hosts[i].copy_(work.x[i], non_blocking=True)
        e2e_step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        et = torch.tensor([a.elapsed_time(b)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": round(rows_step * world * args.e2e_steps / (float(et.item()) / 1000.0), 1),
               "unit": "rows/s", "h2d_bytes_per_step": nb, "d2h_bytes_per_step": nb,
               "dtype": "f32", "api": "lai_voc_resunits_f32 per stage with x copied from and "
                                       "back to pinned host memory inside the timed region"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r = cpu_resunit_rate(stages, runner.RESUNIT_BATCH, args.cpu_seconds)
        cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
               "kind": "port",
               "sample": f"{r['passes']} sweeps of the 4 stages x 3 units on {r['sample_t']} "
                         f"time rows of one item ({r['seconds']:.1f} s), scaled per stage to "
                         f"batch {runner.RESUNIT_BATCH}: the reference's USE_BLAS ResUnit "
                         "(its AVX2 voc_snake_beta + SGEMM convolutions through numpy's "
                         f"OpenBLAS), host {cpu_model()}",
               "per_stage_rows_per_s": r["per_stage_rows_per_s"]}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded counter-based N(0,1) on device; conv weights N(0,1)/sqrt(fan_in))",
        "config": {"workload": "vocoder BigVGAN ResUnits (snake1, dilated causal conv k=7, "
                               "snake2, conv k=1, residual) x 3 per block, 4 blocks, FP32 "
                               "channels-last on tcgen05 tensor cores",
                   "config": "v1", "stages": stages, "batch": runner.RESUNIT_BATCH,
                   "dilations": list(runner.RESUNIT_DILATIONS), "passes": args.passes,
                   "precision": "3xTF32 split, F32 within 1e-5 per unit" if args.passes == 3
                                else "TF32 (1e-2)",
                   "rows": "time rows (batch x T) per stage through its 3 units",
                   "parallelism": f"replicas x{world}, no collective",
                   "l2": f"inputs larger than L2 ({sum(nbytes) / 1e9:.2f} GB moved per step)"},
        "tflops": round(step_tflops, 1),
        "per_kernel": per_kernel, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * len(launches) * (1 + 2 * len(runner.RESUNIT_DILATIONS)),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def cpu_attention_rate(seqs: int, n_heads: int, n_kv: int, max_seq: int, min_seconds: float,
                       steps: int | None = None, warmup: int = 1) -> dict:
    """Decode attention on host cores: the restated qwen_causal_attention for one query
    token per sequence (oracle/_build/liblai_cpuref.so: float sums, the reference's
    optimisation tier, OpenMP over (sequence, head)) on `seqs` sequences with positions
    uniform in [0, max_seq). Returns sequences/s."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("liblai_cpuref.so")
    lib.oracle_set_threads(len(os.sched_getaffinity(0)))
    rng = np.random.default_rng(12)
    kv_dim = n_kv * 128
    q = rng.standard_normal((seqs, n_heads * 128), dtype=np.float32)
    kc = rng.standard_normal((seqs, max_seq, kv_dim), dtype=np.float32)
    vc = rng.standard_normal((seqs, max_seq, kv_dim), dtype=np.float32)
    pos = rng.integers(0, max_seq, seqs).astype(np.int32)
    for _ in range(warmup):
        oracle.decode_attention(q, kc, vc, pos, n_heads, n_kv, 128, lib=lib)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.decode_attention(q, kc, vc, pos, n_heads, n_kv, 128, lib=lib)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
            break
    return {"rows_per_s": seqs * n / el, "threads": lib.oracle_num_threads(), "passes": n,
            "seconds": el, "seqs": seqs}


def cpu_convnext_rate(stages, batch: int, min_seconds: float, sample_t: int = 500,
                      steps: int | None = None, warmup: int = 1) -> dict:
    """The reference's ConvNeXt block (run_convnext, src/tts_vocoder.c:463-533) on host cores
    as its USE_BLAS build runs it: its own compiled voc_conv1d_causal (depthwise branch),
    voc_layer_norm_channels and voc_gelu (oracle/_ref, single-threaded C as in the
    reference) and the two pointwise convolutions as SGEMMs through numpy's OpenBLAS on
    all host cores. `sample_t` time rows of one item per stage, scaled to the step."""
    import numpy as np
    from threadpoolctl import threadpool_limits
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("libvoc_ref_avx2.so")
    P = oracle.ptr
    nthreads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(4)
    f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
    data = []
    for c, t_full in stages:
        prm = {"dw_w": f(rng.standard_normal((c, 1, 7)) / np.sqrt(7)), "dw_b": f(rng.normal(0, .01, c)),
               "nw": f(1 + rng.normal(0, .1, c)), "nb": f(rng.normal(0, .1, c)),
               "w1": f(rng.standard_normal((4 * c, c)) / np.sqrt(c)), "b1": f(rng.normal(0, .01, (4 * c, 1))),
               "w2": f(rng.standard_normal((c, 4 * c)) / np.sqrt(4 * c)), "b2": f(rng.normal(0, .01, (c, 1))),
               "g": f(rng.normal(0, .1, (c, 1)))}
        data.append((c, t_full, prm, f(rng.standard_normal((c, sample_t)))))

    def stage_seconds(c, t_full, p, x0):
        t = x0.shape[1]
        x = x0.copy()
        dw = np.empty_like(x)
        scratch = np.empty(c * (t + 6) + 16, np.float32)
        t0 = time.perf_counter()
        lib.voc_conv1d_causal(P(dw), P(x), P(p["dw_w"]), P(p["dw_b"]), c, c, t, 7, 1, c, P(scratch))
        lib.voc_layer_norm_channels(P(dw), P(p["nw"]), P(p["nb"]), c, t, 1e-6)
        h = p["w1"] @ dw
        h += p["b1"]
        lib.voc_gelu(P(h), h.size)
        y = p["w2"] @ h
        y += p["b2"]
        y *= p["g"]
        x += y
        return time.perf_counter() - t0

    with threadpool_limits(nthreads):
        for _ in range(warmup):
            for st in data:
                stage_seconds(*st)
        n, secs = 0, [0.0] * len(data)
        t_start = time.perf_counter()
        while True:
            for i, st in enumerate(data):
                secs[i] += stage_seconds(*st)
            n += 1
            el = time.perf_counter() - t_start
            if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
                break
    step_s = sum(batch * t_full * (secs[i] / n) / sample_t for i, (c, t_full, _, _) in enumerate(data))
    return {"rows_per_s": sum(batch * t for _, t in stages) / step_s, "step_seconds": step_s,
            "threads": nthreads, "passes": n, "seconds": el, "sample_t": sample_t}


def cpu_decoder_rate(t0: int, batch: int, min_seconds: float, t0_sample: int = 40,
                     steps: int | None = None, warmup: int = 1, full: bool = False) -> dict:
    """The BigVGAN decoder's 4 blocks on host cores as the reference's USE_BLAS build runs
    them (src/tts_vocoder.c:709-728): its own compiled AVX2 voc_snake_beta over channel
    ranges on a thread pool; voc_conv_transpose1d as its SGEMM + col2im formulation
    (src/tts_vocoder_ops.c:169-194) and the ResUnits as in cpu_resunit_rate, the SGEMMs
    through numpy's OpenBLAS on all host cores. Runs from t0_sample input rows; every op is
    linear in T, so the step time is scaled by t0 / t0_sample. Returns audio samples/s.
    full: start from the pre-transformer's output [1024, t0 / 4] instead - 2 upsample stages
    (transposed conv k = s = 2 as SGEMM + col2im, ConvNeXt as cpu_convnext_rate runs it),
    the init conv 1024 -> 1536 (per-tap SGEMMs), then the blocks, then the final SnakeBeta ->
    conv 96 -> 1 -> clamp (the reference's compiled voc_snake_beta and voc_conv1d_causal)."""
    import concurrent.futures as cf

    import numpy as np
    from threadpoolctl import threadpool_limits
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    import runner
    snake = oracle.load("libvoc_ref_avx2.so").voc_snake_beta
    F = ctypes.POINTER(ctypes.c_float)
    nthreads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(10)
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    blocks = []
    for b, r in enumerate(runner.BIGVGAN_RATES):
        c_in, c_out = runner.BIGVGAN_CHANNELS[b], runner.BIGVGAN_CHANNELS[b + 1]
        units = []
        for d in runner.RESUNIT_DILATIONS:
            units.append({"ea1": f(np.exp(rng.normal(0, .1, c_out))), "ieb1": f(np.exp(-rng.normal(0, .1, c_out))),
                          "w1t": [f(rng.standard_normal((c_out, c_out)) / np.sqrt(7 * c_out)) for _ in range(7)],
                          "b1": f(rng.normal(0, .01, (c_out, 1))),
                          "ea2": f(np.exp(rng.normal(0, .1, c_out))), "ieb2": f(np.exp(-rng.normal(0, .1, c_out))),
                          "w2": f(0.1 * rng.standard_normal((c_out, c_out)) / np.sqrt(c_out)),
                          "b2": f(rng.normal(0, .01, (c_out, 1))), "d": d})
        blocks.append({"ea": f(np.exp(rng.normal(0, .1, c_in))), "ieb": f(np.exp(-rng.normal(0, .1, c_in))),
                       "wt": f((rng.standard_normal((c_in, c_out * 2 * r)) / np.sqrt(2 * c_in)).T),
                       "b": f(rng.normal(0, .01, (c_out, 1))), "r": r, "c_out": c_out,
                       "units": units})
    x0 = f(rng.standard_normal((runner.BIGVGAN_CHANNELS[0], t0_sample)))
    ref = oracle.load("libvoc_ref_avx2.so")
    Pt = oracle.ptr
    if full:
        C = 1024
        x0 = f(rng.standard_normal((C, t0_sample // 4)))
        ups = [{"wt": f((rng.standard_normal((C, C * 2)) / np.sqrt(C)).T), "b": f(rng.normal(0, .01, (C, 1))),
                "dw_w": f(rng.standard_normal((C, 1, 7)) / np.sqrt(7)), "dw_b": f(rng.normal(0, .01, C)),
                "nw": f(1 + rng.normal(0, .1, C)), "nb": f(rng.normal(0, .1, C)),
                "w1": f(rng.standard_normal((4 * C, C)) / np.sqrt(C)), "b1": f(rng.normal(0, .01, (4 * C, 1))),
                "w2": f(rng.standard_normal((C, 4 * C)) / np.sqrt(4 * C)), "b2": f(rng.normal(0, .01, (C, 1))),
                "g": f(rng.normal(0, .1, (C, 1)))} for _ in range(2)]
        init_taps = [f(rng.standard_normal((1536, C)) / np.sqrt(7 * C)) for _ in range(7)]
        init_b = f(rng.normal(0, .01, (1536, 1)))
        fin = {"ea": f(np.exp(rng.normal(0, .1, 96))), "ieb": f(np.exp(-rng.normal(0, .1, 96))),
               "w": f(rng.standard_normal((1, 96, 7)) / np.sqrt(672)), "b": f(rng.normal(0, .01, 1))}

    with cf.ThreadPoolExecutor(nthreads) as pool, threadpool_limits(nthreads):
        def snake_mt(x, ea, ieb):
            c, t = x.shape
            per = max(1, -(-c // nthreads))
            list(pool.map(lambda c0: snake(x[c0].ctypes.data_as(F), ea[c0:].ctypes.data_as(F),
                                           ieb[c0:].ctypes.data_as(F), min(per, c - c0), t),
                          range(0, c, per)))

        def front(x):
            for u in ups:  # transposed conv k = s = 2 (no overlap), then ConvNeXt
                t = x.shape[1]
                cols = (u["wt"] @ x).reshape(1024, 2, t)
                y = np.empty((1024, 2 * t), np.float32)
                y[:, 0::2], y[:, 1::2] = cols[:, 0, :], cols[:, 1, :]
                y += u["b"]
                dw = np.empty_like(y)
                scr = np.empty(1024 * (2 * t + 6) + 16, np.float32)
                ref.voc_conv1d_causal(Pt(dw), Pt(y), Pt(u["dw_w"]), Pt(u["dw_b"]), 1024, 1024, 2 * t,
                                      7, 1, 1024, Pt(scr))
                ref.voc_layer_norm_channels(Pt(dw), Pt(u["nw"]), Pt(u["nb"]), 1024, 2 * t, 1e-6)
                h = u["w1"] @ dw
                h += u["b1"]
                ref.voc_gelu(Pt(h), h.size)
                z = u["w2"] @ h
                z += u["b2"]
                z *= u["g"]
                x = y + z
            t = x.shape[1]
            pad = np.zeros((1024, t + 6), np.float32)
            pad[:, 6:] = x
            out = init_taps[0] @ pad[:, :t]
            for k in range(1, 7):
                out += init_taps[k] @ pad[:, k:k + t]
            out += init_b
            return out

        def final(x):
            snake_mt(x, fin["ea"], fin["ieb"])
            t = x.shape[1]
            y = np.empty((1, t), np.float32)
            scr = np.empty(96 * (t + 6) + 96 * 7 * t, np.float32)
            ref.voc_conv1d_causal(Pt(y), Pt(x), Pt(fin["w"]), Pt(fin["b"]), 96, 1, t, 7, 1, 1,
                                  Pt(scr))
            np.clip(y, -1.0, 1.0, out=y)
            return y

        def decoder():
            x = front(x0.copy()) if full else x0.copy()
            for blk in blocks:
                snake_mt(x, blk["ea"], blk["ieb"])
                r, c_out, t = blk["r"], blk["c_out"], x.shape[1]
                cols = (blk["wt"] @ x).reshape(c_out, 2 * r, t)  # W^T X, then col2im
                y = np.zeros((c_out, (t - 1) * r), np.float32)
                for ki in range(2 * r):
                    if ki < r:
                        y[:, ki::r] += cols[:, ki, 1:]
                    else:
                        y[:, ki - r::r] += cols[:, ki, :t - 1]
                y += blk["b"]
                x = y
                for u in blk["units"]:
                    res = x.copy()
                    snake_mt(x, u["ea1"], u["ieb1"])
                    pad = np.zeros((c_out, x.shape[1] + 6 * u["d"]), np.float32)
                    pad[:, 6 * u["d"]:] = x
                    tt = x.shape[1]
                    h = u["w1t"][0] @ pad[:, :tt]
                    for k in range(1, 7):
                        h += u["w1t"][k] @ pad[:, k * u["d"]:k * u["d"] + tt]
                    h += u["b1"]
                    snake_mt(h, u["ea2"], u["ieb2"])
                    x = u["w2"] @ h
                    x += u["b2"]
                    x += res
            return final(x) if full else x

        for _ in range(warmup):
            decoder()
        n, t_start = 0, time.perf_counter()
        while True:
            out = decoder()
            n += 1
            el = time.perf_counter() - t_start
            if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
                break
    step_s = (el / n) * (t0 / t0_sample) * batch
    t_final = t0
    for r in runner.BIGVGAN_RATES:
        t_final = (t_final - 1) * r
    return {"rows_per_s": batch * t_final / step_s, "step_seconds": step_s, "threads": nthreads,
            "passes": n, "seconds": el, "t0_sample": t0_sample, "samples_sample": out.shape[1]}


def cpu_front_seconds(t_frames: int, min_seconds: float = 1.0, steps: int | None = None) -> dict:
    """tts_vocoder_run stages 1-3 (RVQ decode, pre_conv, the 8-layer pre-transformer,
    src/tts_vocoder.c:589-640) on host cores as the reference's USE_BLAS build runs them: every
    linear (the 16 RVQ projections, input/q/k/v/o/gate/up/down/output projections) and the
    pre_conv taps as SGEMMs through numpy's OpenBLAS on all cores; RMSNorm, NeoX RoPE, causal
    attention, SwiGLU and the residual adds from the oracle's timed C build (float sums,
    OpenMP). Runs the full t_frames (attention is T^2). Returns seconds per run."""
    import numpy as np
    from threadpoolctl import threadpool_limits
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    import runner
    lib = oracle.load("liblai_cpuref.so")
    nthreads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(21)
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32)  # noqa: E731
    T, H, A, I = t_frames, runner.XFMR_HIDDEN, runner.XFMR_ATTN, runner.XFMR_INTER
    books = f(rng.standard_normal((runner.RVQ_CODEBOOKS, runner.RVQ_SIZE, runner.RVQ_DIM)))
    proj = [f(rng.standard_normal((runner.RVQ_OUT, runner.RVQ_DIM)) / 64)
            for _ in range(runner.RVQ_CODEBOOKS)]
    codes = rng.integers(0, runner.RVQ_SIZE, (T, runner.RVQ_CODEBOOKS))
    pre_taps = [f(rng.standard_normal((1024, 512)) / np.sqrt(1536)) for _ in range(3)]
    pre_b = f(rng.normal(0, .01, (1024, 1)))
    lin_w = lambda n, k: f(rng.standard_normal((n, k)) / np.sqrt(k))  # noqa: E731
    in_w, in_b, out_w, out_b = lin_w(H, 1024), f(rng.normal(0, .01, H)), lin_w(1024, H), f(
        rng.normal(0, .01, 1024))
    layers = [{"n1": f(1 + rng.normal(0, .1, H)), "wq": lin_w(A, H), "wk": lin_w(A, H),
               "wv": lin_w(A, H), "wo": lin_w(H, A), "g1": f(rng.normal(0, .1, H)),
               "n2": f(1 + rng.normal(0, .1, H)), "wg": lin_w(I, H), "wu": lin_w(I, H),
               "wd": lin_w(H, I), "g2": f(rng.normal(0, .1, H))}
              for _ in range(runner.XFMR_LAYERS)]
    fnorm = f(1 + rng.normal(0, .1, H))
    cos_t, sin_t = oracle.compute_rope_neox(np.arange(T, dtype=np.int32), runner.XFMR_HD,
                                            runner.XFMR_THETA, lib=lib)

    def run():
        rvq = np.zeros((runner.RVQ_OUT, T), np.float32)  # [512, T] as the reference
        for cb in range(runner.RVQ_CODEBOOKS):
            rvq += proj[cb] @ books[cb][codes[:, cb]].T
        pad = np.zeros((512, T + 2), np.float32)
        pad[:, 2:] = rvq
        pre = pre_taps[0] @ pad[:, :T]
        for k in range(1, 3):
            pre += pre_taps[k] @ pad[:, k:k + T]
        pre += pre_b
        x = f(pre.T) @ in_w.T + in_b  # the reference transposes to [T, 1024] first
        for L in layers:
            xn = oracle.rms_norm(x, L["n1"], 1e-5, lib=lib)
            q = oracle.apply_rope_neox(xn @ L["wq"].T, cos_t, sin_t, 16, 64, lib=lib)
            k = oracle.apply_rope_neox(xn @ L["wk"].T, cos_t, sin_t, 16, 64, lib=lib)
            a = oracle.causal_attention(q, k, xn @ L["wv"].T, 16, 16, 64, lib=lib)
            x = oracle.add_inplace(x, (a @ L["wo"].T) * L["g1"], lib=lib)
            xn = oracle.rms_norm(x, L["n2"], 1e-5, lib=lib)
            ffn = oracle.swiglu_separate(xn @ L["wg"].T, xn @ L["wu"].T, lib=lib)
            x = oracle.add_inplace(x, (ffn @ L["wd"].T) * L["g2"], lib=lib)
        x = oracle.rms_norm(x, fnorm, 1e-5, lib=lib)
        return f((x @ out_w.T + out_b).T)  # back to [1024, T]

    with threadpool_limits(nthreads):
        run()
        n, t0 = 0, time.perf_counter()
        while True:
            run()
            n += 1
            el = time.perf_counter() - t0
            if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
                break
    return {"seconds": el / n, "passes": n, "threads": nthreads}


def cpu_sampling_rate(rows: int, vocab: int, top_k: int, temperature: float, penalty: float,
                      hist: int, min_seconds: float, steps: int | None = None) -> dict:
    """The reference's own tts_apply_repetition_penalty + tts_sample_topk (oracle/_ref, built
    from src/tts_sampling.c at its server tier) over `rows` rows, one thread as the
    reference calls them. Returns rows/s."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("libtts_sampling_ref.so")
    rng = np.random.default_rng(3)
    logits = (2 * rng.standard_normal((rows, vocab))).astype(np.float32)
    history = rng.integers(0, vocab, (rows, hist)).astype(np.int32)
    P = oracle.ptr
    n, t0 = 0, time.perf_counter()
    while True:
        for r in range(rows):
            lib.tts_apply_repetition_penalty(P(logits[r]), vocab, P(history[r], oracle._I32), hist,
                                             penalty)
            lib.tts_sample_topk(P(logits[r]), vocab, temperature, top_k)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= min_seconds):
            break
    return {"rows_per_s": rows * n / el, "threads": 1, "passes": n, "seconds": el}


def cpu_tts_frame_rate(min_seconds: float, frames: int | None = None) -> dict:
    """run_decode_loop's frame (config d1) on the host cores: the same steps as runner.TtsFrame
    restated with the oracle's C functions in their timed build (liblai_cpuref.so: -O2 -mavx2
    -ffast-math, OpenMP over output rows, float sums) -- RMSNorm, the BF16 linear, per-head
    q/k norm + RoPE, cache attention, SwiGLU, repetition penalty, top-k -- with distinct
    synthetic weights per layer, so the host streams the same 1.7 GB of BF16 weights per frame
    as the device. The code predictor runs each row once against a 16-row cache, as on the
    device (the reference's recompute of all rows per sub-code does more work). Returns
    frames/s."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    import runner
    lib = oracle.load("liblai_cpuref.so")
    c = runner.TtsConfig()
    H, qd, kvd, hd = c.hidden, c.n_q * c.head_dim, c.n_kv * c.head_dim, c.head_dim
    rng = np.random.default_rng(3)
    pool = rng.standard_normal(1 << 22, dtype=np.float32)
    offs = iter(rng.integers(0, 1 << 21, 4096))

    def w(n, k, scale=None):  # distinct arrays (same bytes streamed), values tiled from a pool
        x = np.resize(pool[next(offs):], (n, k)) * np.float32(scale or k ** -0.5)
        return (x.view(np.uint32) >> 16).astype(np.uint16)

    def nrm(n):
        return (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)

    def layer(inter):
        return {"wqkv": w(qd + 2 * kvd, H), "wo": w(H, qd), "wgu": w(2 * inter, H),
                "wd": w(H, inter), "in": nrm(H), "post": nrm(H), "qn": nrm(hd), "kn": nrm(hd)}

    talker = [layer(c.inter) for _ in range(c.layers)]
    cp = [layer(c.cp_inter) for _ in range(c.cp_layers)]
    head, embed = w(c.talker_vocab, H), w(c.talker_vocab, H, 0.5)
    cp_heads = [w(c.codec_vocab, H) for _ in range(c.groups - 1)]
    cp_embed = [w(c.codec_vocab, H, 0.5) for _ in range(c.groups - 1)]
    fnorm, cnorm = nrm(H), nrm(H)
    max_seq = 256
    ang = np.arange(max_seq)[:, None] * (1.0 / c.theta ** (np.arange(0, hd, 2) / hd))[None]
    cos_t = np.concatenate([np.cos(ang), np.cos(ang)], 1).astype(np.float32)
    sin_t = np.concatenate([np.sin(ang), np.sin(ang)], 1).astype(np.float32)
    kc = np.zeros((c.layers, 1, max_seq, kvd), np.float32)
    vc = np.zeros_like(kc)
    ckc = np.zeros((c.cp_layers, 1, c.groups, kvd), np.float32)
    cvc = np.zeros_like(ckc)

    def run_layers(x, layers, kcs, vcs, pos, inter):
        p = np.array([pos], np.int32)
        for i, L in enumerate(layers):
            qkv = oracle.linear_bf16(oracle.rms_norm(x, L["in"], c.eps, lib), L["wqkv"], lib)
            q, k = oracle.qk_norm_rope(qkv[:, :qd], qkv[:, qd:qd + kvd], L["qn"], L["kn"], cos_t,
                                       sin_t, p, c.n_q, c.n_kv, hd, c.eps, bf16=False, lib=lib)
            kcs[i, 0, pos], vcs[i, 0, pos] = k[0], qkv[0, qd + kvd:]
            a = oracle.decode_attention(q, kcs[i], vcs[i], p, c.n_q, c.n_kv, hd, lib=lib)
            x = oracle.add_inplace(x, oracle.linear_bf16(a, L["wo"], lib), lib)
            gu = oracle.linear_bf16(oracle.rms_norm(x, L["post"], c.eps, lib), L["wgu"], lib)
            x = oracle.add_inplace(
                x, oracle.linear_bf16(oracle.swiglu_multiply(gu, inter, lib), L["wd"], lib), lib)
        return x

    codec_sum = (0.5 * rng.standard_normal((1, H))).astype(np.float32)
    hist = []
    n, pos, t0 = 0, 0, time.perf_counter()
    while True:
        x = run_layers(codec_sum, talker, kc, vc, pos, c.inter)
        hidden = oracle.rms_norm(x, fnorm, c.eps, lib)
        lg = oracle.linear_bf16(hidden, head, lib)
        keep = lg[0, c.eos]
        lg[0, c.suppress_start:] = -1.0e9
        lg[0, c.eos] = keep
        lg = oracle.repetition_penalty(lg, np.array(hist, np.int32), c.penalty, lib)
        cb0 = oracle.sample_topk(lg, c.temperature, c.top_k, rng.random(), lib)[0]
        hist.append(cb0)
        run_layers(hidden, cp, ckc, cvc, 0, c.cp_inter)
        e = oracle.gather_bf16_to_f32(embed, np.array([cb0], np.int32), lib)
        codec_sum = e.copy()
        for j in range(c.groups - 1):
            y = run_layers(e, cp, ckc, cvc, j + 1, c.cp_inter)
            lgj = oracle.linear_bf16(oracle.rms_norm(y, cnorm, c.eps, lib), cp_heads[j], lib)
            sub = oracle.sample_topk(lgj, c.temperature, c.top_k, rng.random(), lib)[0]
            e = oracle.gather_bf16_to_f32(cp_embed[j], np.array([sub], np.int32), lib)
            codec_sum = oracle.add_inplace(codec_sum, e, lib)
        n, pos = n + 1, pos + 1
        el = time.perf_counter() - t0
        if (frames is not None and n >= frames) or (frames is None and el >= min_seconds):
            break
    return {"rows_per_s": n / el, "frames": n, "seconds": el,
            "threads": len(os.sched_getaffinity(0))}


def _e2e_copy_loop(work, launches, steps, pairs, world, dist):
    """Time `steps` steps of: copy every (device, pinned host) input in, the step's launches,
    copy outputs back. pairs: (inputs [(dev, host)], outputs [(host, dev)])."""
    import torch
    ins, outs = pairs
    stream = torch.cuda.current_stream()

    def step():
        for dev, host in ins:
            dev.copy_(host, non_blocking=True)
        for f in launches:
            f()
        for host, dev in outs:
            host.copy_(dev, non_blocking=True)
    step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    et = torch.tensor([a.elapsed_time(b)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    h2d = sum(h.numel() * h.element_size() for _, h in ins)
    d2h = sum(h.numel() * h.element_size() for h, _ in outs)
    return float(et.item()), h2d, d2h


def run_single(args) -> None:
    """--config a3 / n1 / s3: one workload object (runner.DecodeAttention, VocConvNeXt,
    SampleBatch), per-launch CUDA events, roofline against HBM (a3, s3) or the live
    cuBLAS TF32 GEMM (n1), e2e through the same entry with host copies, CPU baseline."""
    import torch
    import torch.distributed as dist
    import runner

    world, rank, local = env_int("WORLD_SIZE", 1), env_int("RANK", 0), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    seed = args.seed + 1000 * rank
    tensor = args.config in ("n1", "v2", "v3", "v4")
    tf32 = tf32_peak_tflops() if tensor else None
    if args.config == "a3":
        work = runner.DecodeAttention(seqs=args.rows or 256, seed=seed)
    elif args.config == "n1":
        work = runner.VocConvNeXt(stages=[(1024, 1000 // args.t_div), (1024, 2000 // args.t_div)],
                                  passes=args.passes, seed=seed)
    elif args.config == "v2":
        work = runner.VocDecoder(t0=2000 // args.t_div, passes=args.passes, seed=seed)
    elif args.config == "v3":
        work = runner.VocFullDecoder(t_frames=500 // args.t_div, passes=args.passes, seed=seed)
    elif args.config == "v4":
        work = runner.VocCodesToAudio(t_frames=500 // args.t_div, passes=args.passes, seed=seed)
    elif args.config == "d1":
        work = runner.TtsDecode(frames=args.warmup + args.steps + args.e2e_steps + 2, seed=seed)
    else:
        work = runner.SampleBatch(seed=seed)
    launches = work.launches(None)
    for _ in range(args.warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    sampler = ClockSampler(phys[local] if local < len(phys) and phys[local] != "" else str(local))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    total_ms, per = time_launches(launches, args.steps, False, work.kernel_names)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([total_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    if hasattr(work, "err"):
        assert int(work.err.item()) == 0, "a device error flag was set"
    peak, peak_kind = measured_peaks()
    nbytes, rows_pl = work.bytes_per_launch(), work.rows_per_launch()
    flops = work.flops_per_launch() if tensor else [0.0] * len(launches)
    per_kernel, dominant, dom_total = {}, None, -1.0
    for j, name in enumerate(work.kernel_names):
        avg_ms = statistics.mean(per[j])
        k = {"avg_us": round(avg_ms * 1000, 2),
             "gbs": round(nbytes[j] / (avg_ms / 1000.0) / 1e9, 1),
             "frac_of_hbm_peak": round(nbytes[j] / (avg_ms / 1000.0) / 1e9 / peak, 4),
             "rows_per_s": round(rows_pl[j] / (avg_ms / 1000.0), 1), "bytes_per_launch": nbytes[j]}
        if tensor:
            k["tflops"] = round(flops[j] / (avg_ms / 1000.0) / 1e12, 1)
            k["tensor_tflops_issued"] = round(k["tflops"] * args.passes, 1)
            k["frac_of_tf32_peak"] = round(k["tflops"] / tf32, 4)
            k["flops_per_launch"] = flops[j]
        per_kernel[name] = k
        if sum(per[j]) > dom_total:
            dominant, dom_total = name, sum(per[j])
    d = per_kernel[dominant]
    if tensor:
        roofline = {"bound": "tensor", "kernel": dominant, "achieved": d["tflops"],
                    "peak": round(tf32, 1), "unit": "TFLOP/s", "frac": d["frac_of_tf32_peak"],
                    "peak_source": "cuBLAS FP32 GEMM on TF32 tensor cores (8192^3, best of 10), "
                                   "measured in this run",
                    "achieved_is": "F32 pointwise-convolution flops; with passes=3 the tensor "
                                   "cores issue 3x that"}
    else:
        roofline = {"bound": "hbm", "kernel": dominant, "achieved": d["gbs"], "peak": peak,
                    "unit": "GB/s", "frac": d["frac_of_hbm_peak"],
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}
    roofline.update({"traffic": load_traffic().get(f"{dominant}@{args.config}"),
                     "algorithmic_bytes_per_launch": d["bytes_per_launch"]})
    rows_step = getattr(work, "rows_step", sum(rows_pl))
    value = rows_step * world * args.steps / (max_ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        if args.config == "a3":
            ins = [(work.q, pin(work.q)), (work.k_new, pin(work.k_new)),
                   (work.v_new, pin(work.v_new)), (work.pos, pin(work.pos))]
            outs = [(pin(work.out), work.out)]
            api = ("lai_decode_attention_f32 with q/k/v/pos copied in from pinned host memory and "
                   "the output back each step; the cache stays on the device")
        elif args.config == "v2":
            ins = [(work.x0, pin(work.x0))]
            outs = [(pin(work.outs[-1]), work.outs[-1])]
            api = ("lai_voc_bigvgan_block_f32 x 4 with the decoder input copied in from and the "
                   "audio-rate output back to pinned host memory each step")
        elif args.config == "v3":
            ins = [(work.x_in, pin(work.x_in))]
            outs = [(pin(work.audio), work.audio)]
            api = ("the 10 vocoder-decoder calls with the pre-transformer output copied in from and "
                   "the audio copied back to pinned host memory each step")
        elif args.config == "v4":
            ins = [(work.codes, pin(work.codes))]
            outs = [(pin(work.audio), work.audio)]
            launches = [lambda: work.run(graph=True)]
            api = ("VocCodesToAudio.run(graph=True): the whole tts_vocoder_run as one CUDA graph "
                   "of library calls (RVQ gather + GEMM, pre_conv, 8 pre-transformer layers, "
                   "the decoder's 10 calls) with the int64 codes copied in from and the audio "
                   "copied back to pinned host memory each step")
        elif args.config == "d1":
            tf = work.tf
            ins = [(tf.u_frame, pin(tf.draws[:1])), (tf.trail_frame, pin(tf.trailing[:1]))]
            outs = [(pin(tf.codes_frame), tf.codes_frame)]
            launches = [lambda: tf.frame(graph=True, staged=True)]
            api = ("one frame per step with its 16 sampling draws and trailing text embedding "
                   "copied in from pinned host memory and its 16 codes copied back (the host "
                   "needs cb0 every frame for the EOS check, src/tts_native.c:1100-1103)")
        elif args.config == "n1":
            ins = [(x, pin(x)) for x in work.x]
            outs = [(pin(x), x) for x in work.x]
            api = "lai_voc_convnext_f32 per stage with x copied in from and back to pinned host memory"
        else:
            ins = [(work.logits, pin(work.logits))]
            outs = [(pin(work.out), work.out)]
            api = "lai_sample_topk_f32 with logits copied in from pinned host memory, tokens back"
        ms, h2d, d2h = _e2e_copy_loop(work, launches, args.e2e_steps, (ins, outs), world, dist)
        e2e = {"value": round(rows_step * world * args.e2e_steps / (ms / 1000.0), 1),
               "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "dtype": "f32", "api": api}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        if args.config == "a3":
            r = cpu_attention_rate(16, work.n_heads, work.n_kv, work.max_seq, args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['passes']} passes over {r['seqs']} sequences at uniform random "
                             f"positions < {work.max_seq} ({r['seconds']:.1f} s): the restated "
                             "qwen_causal_attention (seq_q = 1), float sums, OpenMP over "
                             f"(sequence, head), host {cpu_model()}"}
        elif args.config == "v2":
            r = cpu_decoder_rate(work.t0, work.batch, args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['passes']} runs of the whole decoder from {r['t0_sample']} input "
                             f"rows ({r['samples_sample']} output samples, {r['seconds']:.1f} s), "
                             f"scaled to t0 = {work.t0}: the reference's USE_BLAS path (its AVX2 "
                             "voc_snake_beta, transposed conv as SGEMM + col2im, ResUnits as "
                             f"SGEMMs through numpy's OpenBLAS), host {cpu_model()}"}
        elif args.config == "v3":
            r = cpu_decoder_rate(work.t_dec, work.batch, args.cpu_seconds, full=True)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['passes']} runs of the whole path from {r['t0_sample'] // 4} "
                             f"frames ({r['samples_sample']} samples, {r['seconds']:.1f} s), "
                             f"scaled to {work.t_frames} frames: the reference's USE_BLAS path "
                             "(its compiled SnakeBeta, depthwise conv, LayerNorm, GELU and final "
                             f"conv + OpenBLAS SGEMMs), host {cpu_model()}"}
        elif args.config == "v4":
            fr = cpu_front_seconds(work.t_frames, min_seconds=min(2.0, args.cpu_seconds / 4))
            r = cpu_decoder_rate(work.dec.t_dec, 1, args.cpu_seconds, full=True)
            step_s = fr["seconds"] + r["step_seconds"]
            cpu = {"value": round(work.rows_step / step_s, 1), "unit": "rows/s",
                   "cores": r["threads"], "kind": "port",
                   "sample": f"the front (RVQ decode, pre_conv, 8-layer pre-transformer) at the "
                             f"full {work.t_frames} frames, {fr['passes']} runs "
                             f"({fr['seconds'] * 1000:.0f} ms each: OpenBLAS SGEMM linears, the "
                             "oracle's timed C build for norms, RoPE, attention, SwiGLU), plus "
                             f"the decoder path as config v3 times it ({r['passes']} runs from "
                             f"{r['t0_sample'] // 4} frames scaled to {work.t_frames}: "
                             f"{r['step_seconds'] * 1000:.0f} ms), host {cpu_model()}"}
        elif args.config == "d1":
            r = cpu_tts_frame_rate(args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 3), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['frames']} frames ({r['seconds']:.1f} s) of the same frame "
                             "restated with the oracle's timed C build (BF16 linears, norms, "
                             "RoPE, cache attention, SwiGLU, penalty, top-k; OpenMP over output "
                             f"rows), distinct weights per layer, host {cpu_model()}"}
        elif args.config == "n1":
            r = cpu_convnext_rate(work.stages, work.batch, args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['passes']} sweeps of both stages on {r['sample_t']} time rows of "
                             f"one item ({r['seconds']:.1f} s), scaled per stage to batch "
                             f"{work.batch}: the reference's compiled depthwise conv, channel "
                             "LayerNorm and GELU + OpenBLAS SGEMM pointwise convs, host "
                             f"{cpu_model()}"}
        else:
            r = cpu_sampling_rate(work.rows, work.vocab, work.top_k, work.temperature,
                                  work.penalty, work.history.shape[1], args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": 1,
                   "kind": "reference",
                   "sample": f"{r['passes']} passes over {work.rows} rows ({r['seconds']:.1f} s) of "
                             "the reference's own tts_apply_repetition_penalty + "
                             "tts_sample_topk (built from src/tts_sampling.c), one thread as "
                             f"the reference calls them, host {cpu_model()}"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    desc = {
        "a3": {"workload": "TTS talker decode attention: cache append + attention over keys "
                           "0..pos, one token per sequence, F32 KV cache",
               "sequences": getattr(work, "seqs", None), "heads": [16, 8, 128], "max_seq": 4096,
               "keys_per_step": getattr(work, "keys", None), "rows": "sequences (one token each)"},
        "n1": {"workload": "vocoder ConvNeXt upsample blocks (depthwise conv k=7 + channel "
                           "LayerNorm, pointwise 4x MLP with GELU on tcgen05, layer scale, "
                           "residual), FP32 channels-last",
               "stages": getattr(work, "stages", None), "batch": getattr(work, "batch", None),
               "passes": args.passes, "rows": "time rows (batch x T) per stage"},
        "v2": {"workload": "vocoder BigVGAN decoder after its init conv: 4 blocks of SnakeBeta, "
                           "transposed conv (2r, stride r) and 3 ResUnits on tcgen05, FP32 "
                           "channels-last, at the reference's length progression",
               "t0": getattr(work, "t0", None), "batch": getattr(work, "batch", None),
               "stages": getattr(work, "shapes", None), "passes": args.passes,
               "rows": "audio samples (24 kHz) out of the last block per step"},
        "v3": {"workload": "tts_vocoder_run from the pre-transformer output to audio: 2 x "
                           "(transposed conv + ConvNeXt), init conv, 4 BigVGAN blocks, final "
                           "SnakeBeta + conv + clamp; FP32 channels-last on tcgen05",
               "frames": getattr(work, "t_frames", None), "batch": getattr(work, "batch", None),
               "audio_samples": getattr(work, "t_final", None), "passes": args.passes,
               "rows": "audio samples (24 kHz) per step"},
        "v4": {"workload": "the whole tts_vocoder_run, codec codes to audio: RVQ decode (16 "
                           "codebooks, one gather + one GEMM), pre_conv k=3, 8-layer "
                           "pre-transformer (fused q|k|v and gate|up GEMMs, causal attention "
                           "with RoPE, LayerScale residual epilogues), then the v3 decoder "
                           "path; FP32 channels-last, linears and convs on tcgen05 (3xTF32)",
               "frames": getattr(work, "t_frames", None), "batch": 1,
               "audio_samples": getattr(work, "rows_step", None), "passes": args.passes,
               "rows": "audio samples (24 kHz) per step"},
        "d1": {"workload": "run_decode_loop frames of Qwen3-TTS 0.6B: talker step (28 layers, "
                           "fused GEMVs, q/k norm + RoPE, KV-cache attention, codec head), "
                           "cb0 suppression + penalty + top-k, 15 code-predictor sub-codes (5 "
                           "layers, 16-row cache, lm_head, top-k, embedding feedback); BF16 "
                           "weights, F32 activations; one CUDA graph per frame",
               "layers": [28, 5], "hidden": 1024, "ffn": 3072, "codes_per_frame": 16,
               "weight_bytes_per_frame": work.tf.weight_bytes_per_frame()
               if args.config == "d1" else None,
               "rows": "frames (16 codec codes = 80 ms of audio each)"},
        "s3": {"workload": "talker token sampling: repetition penalty + top-k 50 at temperature "
                           "0.9 over codec logits (vocab 3072), 64-token histories",
               "rows": "decode rows (one token drawn each)", "batch": getattr(work, "rows", None)},
    }[args.config]
    desc.update({"config": args.config, "parallelism": f"replicas x{world}, no collective",
                 "l2": (f"inputs larger than L2 ({sum(nbytes) / 1e9:.2f} GB per step)"
                        if sum(nbytes) > 126e6 else
                        f"L2-resident working set ({sum(nbytes) / 1e6:.1f} MB per step)")})
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded counter-based N(0,1) on device)", "config": desc,
        "per_kernel": per_kernel, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * {"n1": 3 * len(launches), "v2": 8 * len(launches),
                                      "v3": 2 + 2 * 3 + 2 + 4 * 8 + 1,
                                      # front: gather, 3 convs x (split + GEMM), 8 x (2 norms,
                                      # attention, SwiGLU, 4 x (split + GEMM)), norm + conv
                                      "v4": 1 + 6 + 8 * 12 + 3 + 2 + 2 * 3 + 2 + 4 * 8 + 1,
                                      "d1": work.tf.launches_per_frame()
                                      if args.config == "d1" else 0}.get(args.config,
                                                                         len(launches)),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_reference(args) -> None:
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    import runner
    common = {"metric": METRIC, "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
              "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
              "data": "synthetic"}
    # each step is a bounded sample sized so that warm-up + timed steps take about
    # args.ref_budget seconds in total, whatever K and W the caller passes
    per_step_s = args.ref_budget / (args.steps + args.warmup)
    if args.config == "c4":
        # every stage (rows/s depends on the stage mix), items scaled to the budget
        probe = cpu_snake_rate(runner.SNAKE_STAGES, 1, 0.0, steps=1, warmup=0)
        batch = int(max(1, min(runner.SNAKE_BATCH, per_step_s / probe["seconds"])))
        r = cpu_snake_rate(runner.SNAKE_STAGES, batch, 0.0, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"],
              "kind": "reference",
              "sample": f"all stages x batch {batch} (of {runner.SNAKE_BATCH}) per step; the "
                        f"reference's voc_snake_beta (AVX2 build) on {r['threads']} threads, "
                        f"host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["seconds"] / r["passes"], scaling="weak",
                    dtype="f32", config={"workload": "vocoder SnakeBeta stages", "config": "c4",
                                         "stages": runner.SNAKE_STAGES, "batch": batch})
    elif args.config == "v1":
        # all 4 stages x 3 units per step on sample_t time rows, sized to the budget
        probe = cpu_resunit_rate(runner.RESUNIT_STAGES, runner.RESUNIT_BATCH, 0.0, sample_t=256,
                                 steps=1, warmup=0)
        sample_t = int(max(256, min(16000, 256 * per_step_s / max(probe["seconds"], 1e-3))))
        r = cpu_resunit_rate(runner.RESUNIT_STAGES, runner.RESUNIT_BATCH, 0.0,
                             sample_t=sample_t, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"{sample_t} time rows of one item per stage per step, scaled per stage "
                        f"to batch {runner.RESUNIT_BATCH}; the reference's USE_BLAS ResUnit "
                        "(AVX2 voc_snake_beta from its source + SGEMM convolutions through "
                        f"numpy's OpenBLAS) on {r['threads']} threads, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["step_seconds"], scaling="weak", dtype="f32",
                    config={"workload": "vocoder BigVGAN ResUnits", "config": "v1",
                            "stages": runner.RESUNIT_STAGES, "batch": runner.RESUNIT_BATCH,
                            "dilations": list(runner.RESUNIT_DILATIONS)})
    elif args.config == "a3":
        r = cpu_attention_rate(16, 16, 8, 4096, 0.0, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"16 sequences at uniform random positions < 4096 per step: the "
                        f"restated qwen_causal_attention (seq_q = 1), OpenMP, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["seconds"] / r["passes"], scaling="weak", dtype="f32",
                    config={"workload": "TTS talker decode attention", "config": "a3",
                            "sequences": 16, "heads": [16, 8, 128], "max_seq": 4096})
    elif args.config == "v2":
        r = cpu_decoder_rate(2000, 1, 0.0, t0_sample=40, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"the whole decoder from 40 input rows per step ({r['samples_sample']} "
                        "output samples), scaled to t0 = 2000; the reference's USE_BLAS path "
                        f"(AVX2 voc_snake_beta + OpenBLAS SGEMMs), host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["step_seconds"], scaling="weak", dtype="f32",
                    config={"workload": "vocoder BigVGAN decoder (4 blocks)", "config": "v2",
                            "t0": 2000, "batch": 1})
    elif args.config == "v3":
        r = cpu_decoder_rate(2000, 1, 0.0, t0_sample=40, steps=args.steps, warmup=args.warmup,
                             full=True)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"the whole path from 10 frames per step ({r['samples_sample']} output "
                        "samples), scaled to 500 frames; the reference's USE_BLAS path (its "
                        "compiled SnakeBeta, depthwise conv, LayerNorm, GELU and final conv + "
                        f"OpenBLAS SGEMMs), host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["step_seconds"], scaling="weak", dtype="f32",
                    config={"workload": "tts_vocoder_run from the pre-transformer output to audio",
                            "config": "v3", "frames": 500, "batch": 1})
    elif args.config == "v4":
        fr = cpu_front_seconds(500, steps=1)
        r = cpu_decoder_rate(2000, 1, 0.0, t0_sample=40, steps=args.steps, warmup=args.warmup,
                             full=True)
        step_s = fr["seconds"] + r["step_seconds"]
        value = r["rows_per_s"] * r["step_seconds"] / step_s
        cb = {"value": value, "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"the front at the full 500 frames ({fr['seconds'] * 1000:.0f} ms: "
                        "OpenBLAS SGEMM linears + the oracle's timed C build for norms, RoPE, "
                        "attention, SwiGLU) plus the decoder path from 10 frames per step "
                        "scaled to 500 frames (the reference's USE_BLAS path, its compiled "
                        f"SnakeBeta, depthwise conv, LayerNorm, GELU, final conv), host {cpu_model()}"}
        line = dict(common, value=value, unit="rows/s", ms_per_step=1000.0 * step_s,
                    scaling="weak", dtype="f32",
                    config={"workload": "the whole tts_vocoder_run, codec codes to audio",
                            "config": "v4", "frames": 500, "batch": 1})
    elif args.config == "d1":
        r = cpu_tts_frame_rate(0.0, frames=max(1, min(args.steps, int(args.ref_budget / 2))))
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"{r['frames']} frames of the run_decode_loop frame restated with the "
                        "oracle's timed C build (the reference's qwen_* sources are not "
                        f"vendored), host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 / r["rows_per_s"], scaling="weak", dtype="bf16 weights",
                    config={"workload": "run_decode_loop frames, Qwen3-TTS 0.6B", "config": "d1"})
    elif args.config == "n1":
        stages = [(1024, 1000), (1024, 2000)]
        r = cpu_convnext_rate(stages, 8, 0.0, sample_t=500, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"500 time rows of one item per stage per step, scaled to batch 8: the "
                        "reference's compiled depthwise conv, LayerNorm, GELU + OpenBLAS "
                        f"SGEMMs, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["step_seconds"], scaling="weak", dtype="f32",
                    config={"workload": "vocoder ConvNeXt blocks", "config": "n1",
                            "stages": stages, "batch": 8})
    elif args.config == "s3":
        r = cpu_sampling_rate(256, 3072, 50, 0.9, 1.05, 64, 0.0, steps=args.steps)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": 1, "kind": "reference",
              "sample": "256 rows per step through the reference's own tts_sample_topk + "
                        f"repetition penalty, one thread, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["seconds"] / r["passes"], scaling="weak", dtype="f32",
                    config={"workload": "talker token sampling", "config": "s3", "rows": 256,
                            "vocab": 3072, "top_k": 50})
    elif args.config in runner.DECODE_CONFIGS:
        cfg = runner.DECODE_CONFIGS[args.config]
        r = cpu_decode_rate(cfg, per_step_s * args.steps)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"{r['passes']} single-layer linear paths, rate divided by "
                        f"{cfg.layers} layers, FP32, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 / r["rows_per_s"], scaling="weak",
                    dtype="bf16 weights / f32 activations",
                    config={"workload": f"{cfg.name} decode linear path", "config": args.config,
                            "m": cfg.m, "dim": cfg.dim, "ffn": cfg.inter, "layers": cfg.layers})
    else:
        cfg = runner.CONFIGS[args.config]
        probe = cpu_chain_rate(cfg, min(cfg.tokens, 1024), 0.0, steps=2, warmup=1)
        rows = int(max(64, min(cfg.tokens, args.ref_rows, probe["rows_per_s"] * per_step_s)))
        r = cpu_chain_rate(cfg, rows, 0.0, steps=args.steps, warmup=args.warmup)
        cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
              "sample": f"{rows} of {cfg.tokens} tokens of {cfg.name} per step, FP32, "
                        f"OpenMP over rows, host {cpu_model()}"}
        line = dict(common, value=r["rows_per_s"], unit="rows/s",
                    ms_per_step=1000.0 * r["seconds"] / r["passes"],
                    scaling="weak" if args.config != "c5" else "strong", dtype="f32",
                    config={"workload": f"{cfg.name} layer elementwise chain",
                            "config": args.config, "rows_per_step": rows, "dim": cfg.dim,
                            "ffn": cfg.inter})
    line["cpu_baseline"] = cb
    line["e2e"] = {"value": line["value"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ e2e paths
def _pinned(shape, dtype, gen, fill="normal"):
    import torch
    t = torch.empty(shape, dtype=torch.float32).pin_memory() if dtype is None else \
        torch.empty(shape, dtype=dtype).pin_memory()
    if fill == "normal":
        src = torch.randn(shape, generator=gen)
        t.copy_(src if dtype is None else src.to(dtype))
    return t


def e2e_staged_bf16(cfg, rows: int, steps: int, warmup: int) -> dict:
    """The layer chain through the synchronous BF16 entry points on pinned host buffers.

    Per step: lai_staged_add_rmsnorm_bf16, lai_staged_qk_norm_rope_bf16,
    lai_staged_add_rmsnorm_bf16, lai_staged_swiglu_bf16 -- each copies its host inputs
    to the GPU and its outputs back (pipelined chunks) before returning.
    """
    import torch
    import lai
    lib = lai.load()
    D, I, hd, nq, nkv, P = cfg.dim, cfg.inter, cfg.head_dim, cfg.n_q, cfg.n_kv, cfg.pos_period
    g = torch.Generator().manual_seed(9)
    bf = torch.bfloat16
    x, da, df = _pinned((rows, D), bf, g), _pinned((rows, D), bf, g), _pinned((rows, D), bf, g)
    y = _pinned((rows, D), bf, g, fill=None)
    q, k = _pinned((rows, nq * hd), bf, g), _pinned((rows, nkv * hd), bf, g)
    gu, act = _pinned((rows, 2 * I), bf, g), _pinned((rows, I), bf, g, fill=None)
    w_in, w_post = _pinned((D,), None, g), _pinned((D,), None, g)
    wq, wk = _pinned((hd,), None, g), _pinned((hd,), None, g)
    pos = (torch.arange(rows, dtype=torch.int32) % P).pin_memory()
    inv = 1.0 / torch.pow(torch.tensor(cfg.theta, dtype=torch.float32),
                          torch.arange(0, hd, 2, dtype=torch.float32) / hd)
    ang = torch.arange(P, dtype=torch.float32)[:, None] * inv[None, :]
    cos_t = torch.cat([ang.cos(), ang.cos()], 1).contiguous().pin_memory()
    sin_t = torch.cat([ang.sin(), ang.sin()], 1).contiguous().pin_memory()
    V = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        st = [lib.lai_staged_add_rmsnorm_bf16(V(x), V(df), V(w_in), V(y), rows, D, cfg.eps),
              lib.lai_staged_qk_norm_rope_bf16(V(q), V(k), V(wq), V(wk), V(cos_t), V(sin_t), V(pos),
                                               P, rows, nq, nkv, hd, cfg.eps),
              lib.lai_staged_add_rmsnorm_bf16(V(x), V(da), V(w_post), V(y), rows, D, cfg.eps),
              lib.lai_staged_swiglu_bf16(V(act), V(gu), rows, I)]
        if any(st):
            raise RuntimeError(f"staged chain failed: {[lai.status_string(s) for s in st]}")

    b = 2
    h2d = rows * (2 * D * b + (nq + nkv) * hd * b + 4 + 2 * D * b + 2 * I * b) \
        + (2 * D + 2 * hd + 2 * P * hd) * 4
    d2h = rows * (2 * D * b + (nq + nkv) * hd * b + 2 * D * b + I * b)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    return {"seconds": time.perf_counter() - t0, "rows": rows, "steps": steps, "h2d": h2d,
            "d2h": d2h}


def e2e_dropin_f32(cfg, rows: int, steps: int, warmup: int) -> dict:
    """The reference-named FP32 drop-ins (qwen_*) on pinned host FP32 buffers.

    Per step, the layer's 9 calls in the reference's order; each copies its host
    inputs in and its outputs back before returning.
    """
    import numpy as np
    import torch
    import lai
    lib = lai.load()
    D, I, hd, nq, nkv = cfg.dim, cfg.inter, cfg.head_dim, cfg.n_q, cfg.n_kv
    g = torch.Generator().manual_seed(9)
    x, da, df = _pinned((rows, D), None, g), _pinned((rows, D), None, g), _pinned((rows, D), None, g)
    y = _pinned((rows, D), None, g, fill=None)
    q, k, gu = _pinned((rows, nq * hd), None, g), _pinned((rows, nkv * hd), None, g), \
        _pinned((rows, 2 * I), None, g)
    w_in, w_post, wq, wk = (_pinned((n,), None, g) for n in (D, D, hd, hd))
    pos = np.arange(rows) % cfg.pos_period
    inv = 1.0 / np.power(np.float32(cfg.theta), np.arange(0, hd, 2, dtype=np.float32) / hd)
    ang = pos[:, None].astype(np.float32) * inv[None, :].astype(np.float32)
    c_rows = torch.from_numpy(np.concatenate([np.cos(ang)] * 2, 1).astype(np.float32)).pin_memory()
    s_rows = torch.from_numpy(np.concatenate([np.sin(ang)] * 2, 1).astype(np.float32)).pin_memory()
    V = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    T = rows

    def step():
        lib.qwen_add_inplace(V(x), V(df), T * D)
        lib.qwen_rms_norm(V(y), V(x), V(w_in), T, D, cfg.eps)
        lib.qwen_rms_norm_per_head(V(q), V(wq), T, nq, hd, cfg.eps)
        lib.qwen_rms_norm_per_head(V(k), V(wk), T, nkv, hd, cfg.eps)
        lib.qwen_apply_rope_neox(V(q), V(c_rows), V(s_rows), T, nq, hd)
        lib.qwen_apply_rope_neox(V(k), V(c_rows), V(s_rows), T, nkv, hd)
        lib.qwen_add_inplace(V(x), V(da), T * D)
        lib.qwen_rms_norm(V(y), V(x), V(w_post), T, D, cfg.eps)
        lib.qwen_swiglu_multiply(V(gu), V(gu), T, I)

    f4 = 4
    h2d = T * (2 * D + D + nq * hd + nkv * hd + (nq * hd + 2 * hd) + (nkv * hd + 2 * hd)
               + 2 * D + D + 2 * I) * f4 + (2 * D + 2 * hd) * f4
    d2h = T * (D + D + nq * hd + nkv * hd + nq * hd + nkv * hd + D + D + I) * f4
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    el = time.perf_counter() - t0
    err = lib.lai_last_error()
    if err != 0:
        raise RuntimeError(f"drop-in chain failed: {lai.status_string(err)}")
    return {"seconds": el, "rows": rows, "steps": steps, "h2d": h2d, "d2h": d2h}


def e2e_snake_dropin(stages, batch: int, steps: int, warmup: int) -> dict:
    """voc_snake_beta (reference name, FP32) on pinned host buffers, one call per (item, stage)."""
    import torch
    import lai
    lib = lai.load()
    g = torch.Generator().manual_seed(12)
    bufs = [(_pinned((batch, c, t), None, g), _pinned((c,), None, g), _pinned((c,), None, g), c, t)
            for c, t in stages]
    V = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        for x, ea, ieb, c, t in bufs:
            for b_ in range(batch):
                lib.voc_snake_beta(ctypes.c_void_p(x.data_ptr() + b_ * c * t * 4), V(ea), V(ieb), c, t)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    if lib.lai_last_error() != 0:
        raise RuntimeError("voc_snake_beta drop-in failed")
    nbytes = sum(batch * c * t * 4 + 8 * c for _, _, _, c, t in bufs)
    return {"seconds": time.perf_counter() - t0, "steps": steps, "h2d": nbytes,
            "d2h": sum(batch * c * t * 4 for _, _, _, c, t in bufs)}


# ------------------------------------------------------------------ our path
def time_launches(launches, steps: int, graph: bool, names=None):
    """Time `steps` steps. Returns (total ms, per-launch lists of ms).

    Direct mode records a CUDA event after every launch on the launching stream.
    Graph mode (launch-bound configs) replays one captured graph per step for the
    total; for the per-launch times, every kernel name gets one graph holding all of
    that name's launches of a step (each layer's weights read once per replay),
    replayed until about `steps` launches, and its launches share the average."""
    import torch
    stream = torch.cuda.current_stream()
    nk = len(launches)
    if not graph:
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps * nk + 1)]
        evs[0].record(stream)
        i = 1
        for _ in range(steps):
            for f in launches:
                f()
                evs[i].record(stream)
                i += 1
        torch.cuda.synchronize()
        per = [[evs[s * nk + j].elapsed_time(evs[s * nk + j + 1]) for s in range(steps)]
               for j in range(nk)]
        return evs[0].elapsed_time(evs[-1]), per
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in launches:
            f()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    total = a.elapsed_time(b)
    names = list(names) if names is not None else [str(j) for j in range(nk)]
    groups: dict[str, list[int]] = {}
    for j, n in enumerate(names):
        groups.setdefault(n, []).append(j)
    per = [None] * nk
    for idx in groups.values():
        reps = max(1, 20 // len(idx))  # ~20 launches per replay
        gs = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gs):
            for _ in range(reps):
                for j in idx:
                    launches[j]()
        gs.replay()
        torch.cuda.synchronize()
        n_rep = max(1, steps * len(idx) // (reps * len(idx)) // 1)
        n_rep = max(1, min(n_rep, 2000))
        a.record(stream)
        for _ in range(n_rep):
            gs.replay()
        b.record(stream)
        torch.cuda.synchronize()
        avg = a.elapsed_time(b) / (n_rep * reps * len(idx))
        for j in idx:
            per[j] = [avg] * steps
    return total, per


def summarize_kernels(names, per, bpl, rows_pl, peak) -> tuple[dict, str]:
    """Per kernel name: mean CUDA-event time over its launches, algorithmic GB/s, fraction
    of `peak`, rows/s. Returns (table, name of the kernel with the largest total time)."""
    kernels = {}
    for j, name in enumerate(names):
        k = kernels.setdefault(name, {"ms": [], "bytes": bpl[j], "rows": rows_pl[j]})
        k["ms"] += per[j]
    table, dominant, dom_total = {}, None, -1.0
    for name, k in kernels.items():
        avg_ms = statistics.mean(k["ms"])
        gbs = k["bytes"] / (avg_ms / 1000.0) / 1e9
        table[name] = {"avg_us": round(avg_ms * 1000, 2),
                       "median_us": round(statistics.median(k["ms"]) * 1000, 2), "gbs": round(gbs, 1),
                       "frac_of_peak": round(gbs / peak, 4),
                       "rows_per_s": round(k["rows"] / (avg_ms / 1000.0), 1),
                       "bytes_per_launch": k["bytes"], "launches": len(k["ms"])}
        if sum(k["ms"]) > dom_total:
            dominant, dom_total = name, sum(k["ms"])
    return table, dominant


def roofline_of(table, dominant, peak, peak_kind, traffic_key) -> dict:
    d = table[dominant]
    return {"bound": "hbm", "kernel": dominant, "achieved": d["gbs"], "peak": peak,
            "unit": "GB/s", "frac": round(d["gbs"] / peak, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                           else "fallback 6650 GB/s",
            "traffic": load_traffic().get(traffic_key),
            "algorithmic_bytes_per_launch": d["bytes_per_launch"]}


def time_swiglu_forms(work, steps: int, warmup: int, peak: float) -> dict:
    """SwiGLU on a LayerChain's gate_up in both call forms, each launch restored from a
    pristine copy first (untimed): out of place into `act` (the chain's form) and in
    place, out == gate_up (the reference's qwen_swiglu_multiply(out, out, ...) form,
    src/tts_native.c:588, 665, 744). CUDA events bracket the call: the in-place form's
    whole wave schedule is inside them."""
    import torch
    import lai
    gu, inter = work.gate_up, work.cfg.inter
    pristine = gu.clone()
    stream = torch.cuda.current_stream()
    nbytes = work.cfg.bytes_per_token(work.elem)["swiglu"] * work.rows
    out = {}
    for form in ("out_of_place", "inplace"):
        evs = []
        for i in range(warmup + steps):
            gu.copy_(pristine)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            if form == "inplace":
                lai.swiglu_inplace(gu, inter)
            else:
                lai.swiglu(gu, inter, out=work.act)
            b.record(stream)
            if i >= warmup:
                evs.append((a, b))
        torch.cuda.synchronize()
        avg_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        gbs = nbytes / (avg_ms / 1000.0) / 1e9
        out[form] = {"avg_us": round(avg_ms * 1000, 2), "gbs": round(gbs, 1),
                     "frac_of_peak": round(gbs / peak, 4), "bytes_per_launch": nbytes,
                     "launches": len(evs)}
    del pristine
    out["inplace_over_out_of_place"] = round(out["inplace"]["avg_us"]
                                             / out["out_of_place"]["avg_us"], 4)
    return out


def measure_chain_extra(name: str, steps: int, warmup: int, seed: int, peak: float,
                        peak_kind: str, swiglu_forms: bool = False) -> dict:
    """One more named shape on this GPU (N = 1): its whole chain timed per launch (CUDA
    graph replay for the launch-bound L2-resident shapes), per-kernel GB/s, roofline."""
    import torch
    import runner
    cfg = runner.CONFIGS[name]
    rows = cfg.tokens
    work = runner.LayerChain(cfg, rows, row0=0, seed=seed)
    launches = work.launches(None)
    graph = rows <= 4096
    for _ in range(warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()
    total_ms, per = time_launches(launches, steps, graph, work.kernel_names)
    torch.cuda.synchronize()
    assert int(work.err.item()) == 0, f"an id or position was out of range in {name}"
    bpl = work.bytes_per_launch()
    table, dominant = summarize_kernels(work.kernel_names, per, bpl, [rows] * len(bpl), peak)
    step_bytes = sum(bpl)
    res = {"workload": f"{cfg.name} layer chain", "rows": rows, "dim": cfg.dim,
           "ffn": cfg.inter, "positions": f"{cfg.pos_mode} < {cfg.pos_period}",
           "value": round(rows * steps / (total_ms / 1000.0), 1), "unit": "rows/s",
           "ms_per_step": round(total_ms / steps, 4), "steps": steps,
           "timing": "CUDA graph replay" if graph else "direct launches",
           "l2": (f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step)"
                  if step_bytes > 126e6 else
                  f"L2-resident working set ({step_bytes / 1e6:.1f} MB per step): hot-cache, "
                  "launch-latency-bound numbers"),
           "per_kernel": table,
           "roofline": roofline_of(table, dominant, peak, peak_kind, f"{dominant}@{name}")}
    if swiglu_forms:
        res["swiglu_forms"] = time_swiglu_forms(work, min(steps, 20), 3, peak)
    del work, launches
    torch.cuda.empty_cache()
    return res


def time_after_l2_scrub(launches, names, bpl, steps: int, peak: float) -> dict:
    """Each launch timed alone (CUDA events on the launching stream around the launch only)
    after a read-only pass over 256 MiB, twice the L2: the pass evicts, and so writes back,
    the dirty lines the previous launch left, which a launch in a chain of in-place kernels
    otherwise pays for. The same cache state as ncu's default cache control."""
    import torch
    stream = torch.cuda.current_stream()
    scrub = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    out = {}
    for j, f in enumerate(launches):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            torch.sum(scrub, dim=0, out=sink)
            a.record(stream)
            f()
            b.record(stream)
        torch.cuda.synchronize()
        avg_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        gbs = bpl[j] / (avg_ms / 1000.0) / 1e9
        out[names[j]] = {"avg_us": round(avg_ms * 1000, 2), "gbs": round(gbs, 1),
                         "frac_of_peak": round(gbs / peak, 4)}
    del scrub
    return out


def measure_snake_extra(steps: int, warmup: int, seed: int, peak: float, peak_kind: str) -> dict:
    """Config c4 on this GPU (N = 1): SnakeBeta over the five BigVGAN stages x batch 8, one
    launch per stage, per-stage GB/s and its fraction of the measured HBM bandwidth."""
    import torch
    import runner
    work = runner.SnakeSweep(seed=seed)
    launches = work.launches(None)
    for _ in range(warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()
    total_ms, per = time_launches(launches, steps, False, work.kernel_names)
    bpl = work.bytes_per_launch()
    table, dominant = summarize_kernels(work.kernel_names, per, bpl, work.rows_per_launch(), peak)
    clean = time_after_l2_scrub(launches, work.kernel_names, bpl, steps, peak)
    res = {"workload": "vocoder SnakeBeta over the BigVGAN stages, FP32 in place",
           "stages": runner.SNAKE_STAGES, "batch": runner.SNAKE_BATCH,
           "value": round(sum(work.rows_per_launch()) * steps / (total_ms / 1000.0), 1),
           "unit": "channel rows/s", "ms_per_step": round(total_ms / steps, 4), "steps": steps,
           "sweep_gbs": round(sum(bpl) * steps / (total_ms / 1000.0) / 1e9, 1),
           "per_kernel": table,
           "roofline": roofline_of(table, dominant, peak, peak_kind, f"{dominant}@c4"),
           "min_stage_frac": min(v["frac_of_peak"] for v in table.values()),
           "per_kernel_clean_l2": clean,
           "min_stage_frac_clean_l2": min(v["frac_of_peak"] for v in clean.values())}
    del work, launches
    torch.cuda.empty_cache()
    return res


def measure_ops_extra(steps: int, warmup: int, seed: int, peak: float) -> dict:
    """The path's remaining entry points on their own at config-2 sizes (65 536 rows, hidden
    2048, FFN 6144), each launch timed with CUDA events: RMSNorm without the residual add
    (qwen_rms_norm), residual add (qwen_add_inplace) in BF16 and FP32, SiLU (qwen_silu) and
    SiLU*up with separate gate/up (swiglu_separate) in FP32, and the BF16 embedding gather from
    the 151 936-row text table, BF16 and widened to FP32. Algorithmic bytes per launch."""
    import torch
    import lai
    T, D, I, V = 65536, 2048, 6144, 151936
    f32, bf = torch.float32, torch.bfloat16
    dev = "cuda"

    def normal(shape, dt, k):
        t = torch.empty(shape, dtype=dt, device=dev)
        return lai.synth_normal(t, seed=seed + 500 + k)

    x, y = normal((T, D), bf, 1), normal((T, D), bf, 2)
    yo = torch.empty_like(x)
    w = 1 + 0.02 * normal((D,), f32, 3)
    xf, yf = normal((T, D), f32, 4), normal((T, D), f32, 5)
    g, u, o = normal((T * I // 4,), f32, 6), normal((T * I // 4,), f32, 7), torch.empty(T * I // 4, device=dev)
    table = normal((V, D), bf, 8)
    ids = torch.randint(0, V, (T,), dtype=torch.int32, device=dev)
    emb_bf = torch.empty((T, D), dtype=bf, device=dev)
    emb_f = torch.empty((T, D), dtype=f32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    P, S = lai._p, lambda: lai._s(None)  # noqa: E731
    n_act = T * I // 4
    ops = {
        "rmsnorm_bf16": (lambda: lai.call("lai_rmsnorm_bf16", P(yo), P(x), P(w), T, D, 1e-6, S()),
                         T * D * 2 * 2),
        "add_bf16": (lambda: lai.call("lai_add_bf16", P(x), P(y), T * D, S()), T * D * 2 * 3),
        "add_f32": (lambda: lai.call("lai_add_f32", P(xf), P(yf), T * D, S()), T * D * 4 * 3),
        "silu_f32": (lambda: lai.call("lai_silu_f32", P(g), n_act, S()), n_act * 4 * 2),
        "swiglu_separate_f32": (lambda: lai.call("lai_swiglu_separate_f32", P(o), P(g), P(u), n_act,
                                                 S()), n_act * 4 * 3),
        "embed_gather_bf16": (lambda: lai.call("lai_embed_gather_bf16", P(emb_bf), P(table), P(ids), T,
                                               D, V, P(err), S()), T * (2 * D * 2 + 4)),
        "embed_gather_bf16_to_f32": (lambda: lai.call("lai_embed_gather_bf16_to_f32", P(emb_f),
                                                      P(table), P(ids), T, D, V, P(err), S()),
                                     T * (2 * D + 4 * D + 4)),
    }
    out = {}
    for name, (f, nbytes) in ops.items():
        for _ in range(warmup):
            f()
        torch.cuda.synchronize()
        ms, _ = time_launches([f], steps, False)
        avg = ms / steps
        gbs = nbytes / (avg / 1000.0) / 1e9
        out[name] = {"avg_us": round(avg * 1000, 2), "gbs": round(gbs, 1),
                     "frac_of_peak": round(gbs / peak, 4), "bytes_per_launch": nbytes}
    assert int(err.item()) == 0
    del x, y, yo, xf, yf, g, u, o, table, emb_bf, emb_f
    torch.cuda.empty_cache()
    return {"workload": "the path's other entry points on their own, config-2 sizes",
            "rows": T, "dim": D, "ffn": I, "vocab": V, "steps": steps,
            "l2": "inputs larger than L2 for every op", "per_kernel": out}


def pcie_peaks(nbytes: int = 1 << 30, reps: int = 3) -> dict:
    """Pinned host <-> device copy rates of this GPU, measured in this run: H2D alone, D2H
    alone, and both directions at once on two streams (GB/s, best of `reps`)."""
    import torch
    h_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_a = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    d_b = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(fn):
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            best = min(best, time.perf_counter() - t0)
        return best

    def both():
        with torch.cuda.stream(s1):
            d_a.copy_(h_in, non_blocking=True)
        with torch.cuda.stream(s2):
            h_out.copy_(d_b, non_blocking=True)

    t_h2d = timed(lambda: d_a.copy_(h_in, non_blocking=True))
    t_d2h = timed(lambda: h_out.copy_(d_b, non_blocking=True))
    t_both = timed(both)
    del h_in, h_out, d_a, d_b
    torch.cuda.empty_cache()
    return {"h2d_gbs": round(nbytes / t_h2d / 1e9, 2), "d2h_gbs": round(nbytes / t_d2h / 1e9, 2),
            "duplex_gbs": round(2 * nbytes / t_both / 1e9, 2), "bytes": nbytes}


def pcie_fields(h2d: int, d2h: int, seconds_per_step: float, peaks: dict) -> dict:
    """Achieved bus rate of a host-buffer path and its fraction of the fastest the measured
    copy rates allow for the same bytes. With both directions busy each runs at half the
    measured duplex rate (below its solo rate), so the fastest schedule overlaps all of the
    smaller direction with the larger and moves the larger one's excess alone:
    min(H2D, D2H) / (duplex / 2) + the excess at that direction's solo rate."""
    if not peaks:
        return {}
    both = min(h2d, d2h)
    solo = (h2d - both) / (peaks["h2d_gbs"] * 1e9) + (d2h - both) / (peaks["d2h_gbs"] * 1e9)
    bound_s = both / (peaks["duplex_gbs"] * 1e9 / 2) + solo
    # never below a direction's own solo time (a duplex rate above twice a solo rate)
    bound_s = max(bound_s, h2d / (peaks["h2d_gbs"] * 1e9), d2h / (peaks["d2h_gbs"] * 1e9))
    return {"pcie_gbs": round((h2d + d2h) / seconds_per_step / 1e9, 2),
            "pcie_bound_ms": round(bound_s * 1000, 3),
            "pcie_frac": round(bound_s / seconds_per_step, 4)}


def cpu_chain_baseline(cfg, rows_all: int, rows_1t: int, seconds: float) -> dict:
    """The FP32 chain on the host: all cores and one thread, each the median of 3 runs of
    about seconds / 6 (the reference's vocoder_bench convention: tools/vocoder_bench.c:190,
    476)."""
    runs_all = [cpu_chain_rate(cfg, rows_all, seconds / 6) for _ in range(3)]
    runs_1t = [cpu_chain_rate(cfg, rows_1t, seconds / 6, threads=1) for _ in range(3)]
    med = lambda rs: statistics.median(r["rows_per_s"] for r in rs)  # noqa: E731
    return {"value": round(med(runs_all), 1), "value_1t": round(med(runs_1t), 1),
            "threads": runs_all[0]["threads"], "rows_all": rows_all, "rows_1t": rows_1t,
            "passes": sum(r["passes"] for r in runs_all),
            "passes_1t": sum(r["passes"] for r in runs_1t)}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    import runner

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    args.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    snake = args.config == "c4"
    decode = args.config in runner.DECODE_CONFIGS
    strong = args.config == "c5"
    if snake:
        work = runner.SnakeSweep(seed=args.seed + 1000 * rank)
        rows = sum(work.rows_per_launch())
        cfg = None
    elif decode:
        cfg = runner.DECODE_CONFIGS[args.config]
        can_chain = args.wfmt == "bf16" and cfg.m == 1 and args.gemv != "per-op"
        work = runner.DecodeLinear(cfg, seed=args.seed + 1000 * rank, wfmt=args.wfmt,
                                   chain=can_chain)
        rows = cfg.m
    else:
        cfg = runner.CONFIGS[args.config]
        if strong:
            row0, row1 = runner.shard_range(cfg.tokens, world, rank)
        else:
            per = args.rows or cfg.tokens
            row0, row1 = rank * per, (rank + 1) * per
        rows = row1 - row0
        work = runner.LayerChain(cfg, rows, row0=row0, seed=args.seed, dtype=args.dtype)
    graph = args.graph == "on" or (args.graph == "auto" and not snake and rows <= 4096)
    form_us = None
    if decode and work.chain is not None:
        # both forms of the step timed briefly (same weights); `auto` measures the faster below
        form_us = {}
        for form in ("per-op", "chain"):
            work.set_form(form)
            ls = work.launches(None)
            for _ in range(3):
                for f in ls:
                    f()
            torch.cuda.synchronize()
            ms, _ = time_launches(ls, 20, graph, list(work.kernel_names))
            form_us[form] = round(1000.0 * ms / 20, 2)
        work.set_form(args.gemv if args.gemv != "auto" else min(form_us, key=form_us.get))
    launches = work.launches(None)  # each launch goes to the current stream when called
    unfused_us = None
    ul = work.unfused_library_launches() if decode else None
    if ul:  # the same step as separate kernels around cuBLAS GEMMs, for comparison
        for _ in range(args.warmup):
            for f in ul:
                f()
        torch.cuda.synchronize()
        u_ms, _ = time_launches(ul, args.steps, graph, [str(j) for j in range(len(ul))])
        unfused_us = round(1000.0 * u_ms / args.steps, 2)

    for _ in range(args.warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()

    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = phys[local] if local < len(phys) and phys[local] != "" else str(local)
    sampler = ClockSampler(gpu_index)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)  # let the sampler attach before the timed region
    total_ms, per = time_launches(launches, args.steps, graph, work.kernel_names)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([total_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    if not snake and not decode:
        assert int(work.err.item()) == 0, "an id or position was out of range in the chain"

    peak, peak_kind = measured_peaks()
    total_rows = cfg.tokens if strong else rows * world
    value = total_rows * args.steps / (max_ms / 1000.0)
    bpl = work.bytes_per_launch()
    rows_pl = work.rows_per_launch() if (snake or decode) else [rows] * len(bpl)
    per_kernel, dominant = summarize_kernels(work.kernel_names, per, bpl, rows_pl, peak)

    # every rank's own step time and per-kernel GB/s (the slowest rank sets `value`)
    per_rank = None
    if world > 1:
        names = list(per_kernel)
        mine = torch.tensor([total_ms / args.steps, float(rows)]
                            + [per_kernel[n]["gbs"] for n in names],
                            device="cuda", dtype=torch.float64)
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [{"rank": r, "ms_per_step": round(float(v[0]), 4), "rows": int(v[1]),
                     "gbs": {n: round(float(v[2 + j]), 1) for j, n in enumerate(names)},
                     "frac_of_peak": {n: round(float(v[2 + j]) / peak, 4)
                                      for j, n in enumerate(names)}}
                    for r, v in enumerate(allr)]

    # each distinct kernel also timed alone: `steps` back-to-back launches of it (outside
    # the chain, so no neighbour's leftover L2 write-back is charged to it)
    isolated = {}
    if not args.no_isolate and not graph:
        seen = {}
        for j, name in enumerate(work.kernel_names):
            seen.setdefault(name, j)
        for name, j in seen.items():
            iso_ms, _ = time_launches([launches[j]], args.steps, False)
            avg_ms = iso_ms / args.steps
            isolated[name] = {"avg_us": round(avg_ms * 1000, 2),
                              "gbs": round(bpl[j] / (avg_ms / 1000.0) / 1e9, 1),
                              "frac_of_peak": round(bpl[j] / (avg_ms / 1000.0) / 1e9 / peak, 4)}
    step_bytes = sum(bpl)
    step_gbs = step_bytes * args.steps / (total_ms / 1000.0) / 1e9
    roofline = roofline_of(per_kernel, dominant, peak, peak_kind, f"{dominant}@{args.config}")
    roofline.update(step_gbs=round(step_gbs, 1), step_frac=round(step_gbs / peak, 4))
    if strong and roofline["traffic"] is not None:  # the committed figure is for all the tokens
        roofline["traffic"] = int(roofline["traffic"] * rows / cfg.tokens)

    def max_time(sec):
        et = torch.tensor([sec], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        return float(et.item())

    gemv_form = work.form if decode else None
    step_kernels = len(work.kernel_names)
    del work, launches  # free the device-resident workload before the other measurements
    torch.cuda.empty_cache()

    # the other named shapes, one GPU only (the scaling runs time the headline shape alone)
    extras = {}
    if world == 1 and not args.no_extras and args.config == "c5":
        ew = max(3, min(args.warmup, 10))
        es = max(args.steps, 20)
        extras["c2"] = measure_chain_extra("c2", es, ew, args.seed, peak, peak_kind,
                                           swiglu_forms=True)
        extras["c1"] = measure_chain_extra("c1", max(es, 200), ew, args.seed, peak, peak_kind)
        extras["c3"] = measure_chain_extra("c3", max(es, 200), ew, args.seed, peak, peak_kind)
        extras["c4"] = measure_snake_extra(es, ew, args.seed, peak, peak_kind)
        extras["ops"] = measure_ops_extra(es, ew, args.seed, peak)

    e2e = e2e_f32 = pcie = None
    if not args.no_e2e and not decode:
        pcie = pcie_peaks()
        if snake:
            r = e2e_snake_dropin(runner.SNAKE_STAGES, runner.SNAKE_BATCH, args.e2e_steps, 1)
            sec = max_time(r["seconds"])
            e2e = {"value": round(rows * world * r["steps"] / sec, 1),
                   "unit": "rows/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"], "dtype": "f32",
                   "api": "voc_snake_beta drop-in on pinned host buffers, one call per item and stage",
                   **pcie_fields(r["h2d"], r["d2h"], sec / r["steps"], pcie)}
        else:
            # every rank stages its own rows over its own PCIe link; beyond 4 ranks the rows
            # per rank shrink so the host's pinned memory stays bounded (~40 GB in all)
            share = max(1, world // 4)
            er = min(rows, max(1024, args.e2e_rows_bf16 // share))
            r = e2e_staged_bf16(cfg, er, args.e2e_steps, 1)
            sec = max_time(r["seconds"])
            e2e = {"value": round(er * world * r["steps"] / sec, 1),
                   "unit": "rows/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"], "rows_per_step": er, "dtype": "bf16",
                   "api": "lai_staged_{add_rmsnorm,qk_norm_rope,swiglu}_bf16 on pinned host "
                          "buffers, 4 synchronous calls/step",
                   **pcie_fields(r["h2d"], r["d2h"], sec / r["steps"], pcie)}
            fr = min(rows, max(1024, args.e2e_rows // share))
            r = e2e_dropin_f32(cfg, fr, args.e2e_steps, 1)
            sec = max_time(r["seconds"])
            e2e_f32 = {"value": round(fr * world * r["steps"] / sec, 1),
                       "unit": "rows/s", "h2d_bytes_per_step": r["h2d"],
                       "d2h_bytes_per_step": r["d2h"], "rows_per_step": fr, "dtype": "f32",
                       "api": "reference-named qwen_* drop-ins on pinned host FP32 buffers, "
                              "9 calls/step",
                       **pcie_fields(r["h2d"], r["d2h"], sec / r["steps"], pcie)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        if decode:
            r = cpu_decode_rate(cfg, args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": f"{r['passes']} single-layer linear paths ({r['seconds']:.1f} s, "
                             f"rate divided by {cfg.layers} layers): RMSNorm, linear_bf16 x4, "
                             f"SwiGLU, adds, FP32, host {cpu_model()}"}
        elif snake:
            r = cpu_snake_rate(runner.SNAKE_STAGES, args.cpu_batch, args.cpu_seconds)
            cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
                   "kind": "reference",
                   "sample": f"{r['passes']} sweeps of all stages x batch {args.cpu_batch} "
                             f"({r['seconds']:.1f} s) through the reference's voc_snake_beta "
                             f"(AVX2 build), host {cpu_model()}"}
        else:
            ra, r1 = min(rows, args.cpu_rows), min(rows, max(64, args.cpu_rows // 8))
            r = cpu_chain_baseline(cfg, ra, r1, args.cpu_seconds)
            cpu = {"value": r["value"], "unit": "rows/s", "cores": r["threads"],
                   "value_1t": r["value_1t"], "cores_1t": 1, "kind": "port",
                   "sample": f"the FP32 chain (the oracle's timed build: add+RMSNorm, per-head "
                             f"RMSNorm, RoPE, add+RMSNorm, SwiGLU): {ra} tokens on "
                             f"{r['threads']} threads ({r['passes']} passes) and {r1} tokens "
                             f"on 1 thread ({r['passes_1t']} passes), each the median of 3 "
                             f"runs, host {cpu_model()}"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    if decode:
        config = {"workload": f"{cfg.name}: the decode step's linear path through "
                              f"{cfg.layers} layers (per layer RMSNorm+QKV GEMV, O GEMV+residual, "
                              "RMSNorm+gate/up GEMV+SwiGLU, down GEMV+residual)",
                  "config": args.config, "m": cfg.m, "dim": cfg.dim, "ffn": cfg.inter,
                  "layers": cfg.layers, "weights": args.wfmt, "bytes_per_step": step_bytes,
                  "timing": "CUDA graph replay" if graph else "direct launches",
                  "unfused_library_us_per_step": unfused_us,
                  "gemv": ("one persistent GEMV-chain kernel per step" if gemv_form == "chain"
                           else "one fused-GEMV launch per projection"),
                  "gemv_forms_us_per_step": form_us,
                  "l2": f"weights larger than L2 ({step_bytes / 1e9:.2f} GB per step)"}
        launches_per_step = step_kernels
    elif snake:
        config = {"workload": "vocoder SnakeBeta over the BigVGAN stages, FP32 in place",
                  "config": "c4", "stages": runner.SNAKE_STAGES, "batch": runner.SNAKE_BATCH,
                  "rows": "channel rows (batch x channels) per sweep",
                  "parallelism": f"replicas x{world}, no collective",
                  "l2": f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step per GPU)"}
        launches_per_step = len(runner.SNAKE_STAGES)
    else:
        config = {"workload": f"{cfg.name} layer elementwise chain ("
                              + ", ".join(work_names := list(cfg.kernels())) + ")",
                  "config": args.config, "tokens": cfg.tokens if strong else rows * world,
                  "rows_per_gpu": rows, "dim": cfg.dim, "ffn": cfg.inter,
                  "heads": [cfg.n_q, cfg.n_kv, cfg.head_dim], "positions": cfg.pos_mode,
                  "parallelism": (f"row-sharded x{world} (contiguous blocks of the "
                                  f"{cfg.tokens} tokens), no collective" if strong else
                                  f"x{world} GPUs, each its own {rows} tokens, no collective"),
                  "timing": "CUDA graph replay" if graph else "direct launches",
                  "l2": (f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step per GPU)"
                         if step_bytes > 126e6 else
                         f"L2-resident working set ({step_bytes / 1e6:.1f} MB per step): hot-cache numbers")}
        launches_per_step = len(work_names) + (1 if (rows * cfg.inter) % 4 else 0)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": "f32" if snake else (f"{args.wfmt} weights / f32 activations" if decode
                                      else args.dtype),
        "data": "synthetic (seeded counter-based N(0,1) on device; norm weights 1+N(0,0.02))",
        "config": config,
        "hbm_gbs": round(step_gbs * (1 if strong else world), 1),
        "per_kernel": per_kernel, "per_kernel_isolated": isolated, "per_rank": per_rank,
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "e2e_dropin_f32": e2e_f32, "pcie_peaks": pcie, "other_shapes": extras or None,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 2000; 20 for v1, whose step is ~0.1 s)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5", "d1", "g1", "g2", "v1", "v2", "v3",
                                         "v4", "a3", "n1", "s3"],
                    default="c5")
    ap.add_argument("--t-div", type=int, default=1,
                    help="v1: divide every stage's length (small profiling cases)")
    ap.add_argument("--passes", type=int, choices=[1, 3], default=3,
                    help="v1: 3 = F32-faithful 3xTF32 products, 1 = plain TF32")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--gemv", choices=["auto", "chain", "per-op"], default="auto",
                    help="decode configs (BF16 weights, M = 1): the step as one persistent "
                         "GEMV-chain kernel or one fused-GEMV launch per projection; auto times "
                         "both briefly and measures the faster")
    ap.add_argument("--wfmt", choices=["bf16", "f16", "i8", "f32"], default="bf16",
                    help="g1/g2: decode weight format (the reference's GPU modes: BF16 as stored, "
                         "FP16, INT8 + per-row scale, F32)")
    ap.add_argument("--dtype", choices=["bf16", "f32"], default="bf16",
                    help="activation storage of the layer chain (f32: the drop-ins' type)")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU instead of the config's batch (small profiling cases)")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="CUDA-graph replay (auto: for launch-bound configs of <= 4096 rows)")
    ap.add_argument("--e2e-rows", type=int, default=16384, help="rows of the FP32 drop-in e2e")
    ap.add_argument("--e2e-rows-bf16", type=int, default=65536, help="rows of the BF16 e2e")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-isolate", action="store_true",
                    help="skip timing each kernel alone after the chain")
    ap.add_argument("--cpu-rows", type=int, default=8192,
                    help="tokens of the in-run CPU baseline sample (all cores; 1/8 of it on 1 thread)")
    ap.add_argument("--ref-rows", type=int, default=65536,
                    help="--impl reference: most tokens per step of the CPU sample")
    ap.add_argument("--cpu-batch", type=int, default=2,
                    help="SnakeBeta batch items in the CPU baseline sample (c4)")
    ap.add_argument("--ref-budget", type=float, default=90.0,
                    help="seconds the --impl reference run should take in total")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="c5: skip timing the other named shapes (c1, c2 + SwiGLU in place, c3, "
                         "c4) after the headline")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # timing rule: at least 3 untimed warm-up steps
    if args.steps is None:
        args.steps = {"v1": 20, "v2": 20, "v3": 20, "v4": 20, "n1": 50, "a3": 200,
                      "d1": 50}.get(
            args.config, 100 if args.config == "c5" else 2000)
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "v1":
        run_resunits(args)
    elif args.config in ("a3", "d1", "n1", "s3", "v2", "v3", "v4"):
        run_single(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
