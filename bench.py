#!/usr/bin/env python3
"""Benchmark of the B200 per-layer kernels (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c3|c5] [--e2e-rows R]

A step is one decoder layer's elementwise chain over one batch (runner.LayerChain):
fused residual-add+RMSNorm, fused q/k RMSNorm+RoPE, fused residual-add+RMSNorm,
SwiGLU -- BF16 storage, FP32 math -- on inputs resident in HBM. The default
workload is config c2 (Qwen3-ASR-1.7B layer ops, 64 x 1024 tokens, hidden 2048,
FFN 6144), per GPU: N GPUs each run their own 65536-token batch, no collective
("scaling": "weak"). --config c5 runs the 2M-token chain split across the N GPUs
instead ("strong"). `value` is tokens/s over all GPUs; the roofline object
reports the dominant kernel's achieved HBM GB/s from live CUDA events.

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
                   warmup: int = 1) -> dict:
    """The reference's FP32 chain on host cores (oracle/_build/liblai_cpuref.so).

    Returns rows/s. Either `steps` timed passes, or passes until `min_seconds`.
    """
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    lib = oracle.load("liblai_cpuref.so")
    lib.oracle_set_threads(len(os.sched_getaffinity(0)))  # all host cores, whatever OMP_* says
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


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> None:
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    import runner
    cfg = runner.CONFIGS[args.config]
    rows = min(cfg.tokens, args.cpu_rows)
    r = cpu_chain_rate(cfg, rows, 0.0, steps=args.steps, warmup=args.warmup)
    cb = {"value": r["rows_per_s"], "unit": "rows/s", "cores": r["threads"], "kind": "port",
          "sample": f"{rows} of {cfg.tokens} tokens of {cfg.name} per step, FP32, "
                    f"OpenMP over rows, host {cpu_model()} x {os.cpu_count()}"}
    line = {"metric": METRIC, "impl": "reference", "value": r["rows_per_s"], "unit": "rows/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * r["seconds"] / r["passes"], "higher_is_better": True,
            "scaling": "weak" if args.config != "c5" else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{cfg.name} layer elementwise chain", "config": args.config,
                       "rows_per_step": rows, "dim": cfg.dim, "ffn": cfg.inter},
            "cpu_baseline": cb,
            "e2e": {"value": r["rows_per_s"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
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


# ------------------------------------------------------------------ our path
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    import lai
    import runner

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    cfg = runner.CONFIGS[args.config]
    strong = args.config == "c5"
    if strong:
        row0, row1 = runner.shard_range(cfg.tokens, world, rank)
    else:
        per = args.rows or cfg.tokens
        row0, row1 = rank * per, (rank + 1) * per
    rows = row1 - row0
    chain = runner.LayerChain(cfg, rows, row0=row0, seed=args.seed)
    stream = torch.cuda.current_stream()
    launches = chain.launches(stream)
    nk = len(launches)

    for _ in range(args.warmup):
        for f in launches:
            f()
    torch.cuda.synchronize()

    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = phys[local] if local < len(phys) and phys[local] != "" else str(local)
    sampler = ClockSampler(gpu_index)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps * nk + 1)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)  # let the sampler attach before the timed region
    evs[0].record(stream)
    i = 1
    for _ in range(args.steps):
        for f in launches:
            f()
            evs[i].record(stream)
            i += 1
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    total_ms = evs[0].elapsed_time(evs[-1])
    per = [[] for _ in range(nk)]
    for s in range(args.steps):
        for j in range(nk):
            per[j].append(evs[s * nk + j].elapsed_time(evs[s * nk + j + 1]))
    t = torch.tensor([total_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    assert int(chain.err.item()) == 0, "position out of range in the chain"
    swiglu_tail = 1 if (rows * cfg.inter) % 4 else 0

    peak, peak_kind = measured_peaks()
    total_rows = cfg.tokens if strong else rows * world
    value = total_rows * args.steps / (max_ms / 1000.0)
    bpl = chain.bytes_per_launch()
    kernels = {}
    for j, name in enumerate(runner.LayerChain.KERNELS):
        k = kernels.setdefault(name, {"ms": [], "bytes": bpl[j]})
        k["ms"] += per[j]
    per_kernel, dominant, dom_total = {}, None, -1.0
    for name, k in kernels.items():
        avg_ms = statistics.mean(k["ms"])
        gbs = k["bytes"] / (avg_ms / 1000.0) / 1e9
        per_kernel[name] = {"avg_us": round(avg_ms * 1000, 2), "gbs": round(gbs, 1),
                            "frac_of_peak": round(gbs / peak, 4),
                            "rows_per_s": round(rows / (avg_ms / 1000.0), 1),
                            "bytes_per_launch": k["bytes"], "launches": len(k["ms"])}
        if sum(k["ms"]) > dom_total:
            dominant, dom_total = name, sum(k["ms"])
    step_bytes = cfg.step_bytes_per_token() * rows
    step_gbs = step_bytes * args.steps / (total_ms / 1000.0) / 1e9
    traffic = load_traffic().get(f"{dominant}@{args.config}")
    d = per_kernel[dominant]
    roofline = {"bound": "hbm", "kernel": dominant, "achieved": d["gbs"], "peak": peak,
                "unit": "GB/s", "frac": round(d["gbs"] / peak, 4), "peak_source": peak_kind,
                "traffic": traffic, "algorithmic_bytes_per_launch": d["bytes_per_launch"],
                "step_gbs": round(step_gbs, 1), "step_frac": round(step_gbs / peak, 4)}

    # e2e: the same chain on pinned host buffers through the C ABI's synchronous entries
    e2e = e2e_f32 = None
    if not args.no_e2e:
        def max_time(sec):
            et = torch.tensor([sec], device="cuda", dtype=torch.float64)
            if world > 1:
                dist.all_reduce(et, op=dist.ReduceOp.MAX)
            return float(et.item())
        del chain  # free the device-resident workload before the staged runs
        torch.cuda.empty_cache()
        r = e2e_staged_bf16(cfg, rows, args.e2e_steps, 1)
        e2e = {"value": round(rows * world * r["steps"] / max_time(r["seconds"]), 1),
               "unit": "rows/s", "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
               "rows_per_step": rows, "dtype": "bf16",
               "api": "lai_staged_{add_rmsnorm,qk_norm_rope,swiglu}_bf16 on pinned host buffers, "
                      "4 synchronous calls/step"}
        fr = min(rows, args.e2e_rows)
        r = e2e_dropin_f32(cfg, fr, args.e2e_steps, 1)
        e2e_f32 = {"value": round(fr * world * r["steps"] / max_time(r["seconds"]), 1),
                   "unit": "rows/s", "h2d_bytes_per_step": r["h2d"],
                   "d2h_bytes_per_step": r["d2h"], "rows_per_step": fr, "dtype": "f32",
                   "api": "reference-named qwen_* drop-ins on pinned host FP32 buffers, "
                          "9 calls/step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r = cpu_chain_rate(cfg, min(rows, args.cpu_rows), args.cpu_seconds)
        cpu = {"value": round(r["rows_per_s"], 1), "unit": "rows/s", "cores": r["threads"],
               "kind": "port",
               "sample": f"{min(rows, args.cpu_rows)} tokens x {r['passes']} passes "
                         f"({r['seconds']:.1f} s) of the FP32 chain, host {cpu_model()}"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded counter-based N(0,1) on device; norm weights 1+N(0,0.02))",
        "config": {"workload": f"{cfg.name} layer elementwise chain "
                               "(add+RMSNorm, qk-norm+RoPE, add+RMSNorm, SwiGLU)",
                   "config": args.config, "rows_per_gpu": rows, "dim": cfg.dim, "ffn": cfg.inter,
                   "heads": [cfg.n_q, cfg.n_kv, cfg.head_dim], "positions": cfg.pos_mode,
                   "parallelism": f"row-sharded x{world}, no collective",
                   "l2": f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step per GPU)"},
        "hbm_gbs": round(step_gbs * (world if not strong else 1), 1),
        "per_kernel": per_kernel, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "e2e_dropin_f32": e2e_f32,
        "gpu_launches": args.steps * (3 + 1 + swiglu_tail),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c5"], default="c2")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU instead of the config's batch (small profiling cases)")
    ap.add_argument("--e2e-rows", type=int, default=16384)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=8192)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # timing rule: at least 3 untimed warm-up steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
