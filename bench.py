#!/usr/bin/env python3
"""Benchmark of the qma B200 engine (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (single GPU; N > 1 runs one independent replica per GPU, weak
scaling): the configs[1] quantized GEMV microbench at the LM-head shape,
Q4_K 151936x2048 at batch 1 -- fp32 activation ~N(0,1) quantized to Q8_K on
the GPU, then the GEMV.  A step is one quantize + GEMV; the 175 MB weight
matrix exceeds L2 and L2 is also flushed (256 MB write) between timed steps.

--impl reference times the reference's own CPU matmul (nn.c:307-345, built
from its sources in oracle/_ref) on the host cores for the same shape.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for sub in ("qwen-mobile-agent_b200", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, sub))

METRIC = "Q4_K GEMV HBM GB/s vs peak (part of: qwen35moe decode tok/s (bs1, 1 GPU) & Q4_K GEMV HBM GB/s vs peak; EP tok/s @2/4/8)"
N_OUT, N_IN = 151936, 2048
Q4_K = 12


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(T=1):
    w = N_OUT * (N_IN // 256) * 144
    act = T * (N_IN * 4 + N_IN + (N_IN // 256) * 4 + (N_IN // 16) * 2)   # x read, Q8_K written+read
    out = T * N_OUT * 4
    return w + act + out, w


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- distributed --
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# -------------------------------------------------------------- CPU legs ---
def make_weight(seed=0):
    import oracle as O
    return O.synth_matrix("bench.lm_head", Q4_K, N_OUT, N_IN, seed=seed)


def cpu_reference_rate(W, x, seconds=10.0, min_steps=3, threads=None):
    """Reference CPU matmul (oracle/_ref, nn.c:307) GB/s over a bounded sample."""
    import oracle as O
    R = O.ref()
    th = threads or min(os.cpu_count() or 1, 16)
    R.qr_init(th)
    out = np.zeros((1, N_OUT), np.float32)
    R.qr_matmul(O._ptr(x), O._ptr(W), N_IN, N_OUT, 1, Q4_K, O._ptr(out), th)   # warm
    steps, t0 = 0, time.perf_counter()
    while True:
        R.qr_matmul(O._ptr(x), O._ptr(W), N_IN, N_OUT, 1, Q4_K, O._ptr(out), th)
        steps += 1
        el = time.perf_counter() - t0
        if steps >= min_steps and el >= seconds:
            break
    b, _ = algorithmic_bytes()
    return b * steps / el / 1e9, th, steps, el


def run_reference(args, world, rank):
    if rank != 0:
        return
    import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent at build time)"}))
        return
    W = make_weight()
    x = np.random.default_rng(0).standard_normal((1, N_IN)).astype(np.float32)
    th = min(os.cpu_count() or 1, 16)
    R = O.ref()
    R.qr_init(th)
    out = np.zeros((1, N_OUT), np.float32)
    for _ in range(args.warmup):
        R.qr_matmul(O._ptr(x), O._ptr(W), N_IN, N_OUT, 1, Q4_K, O._ptr(out), th)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        R.qr_matmul(O._ptr(x), O._ptr(W), N_IN, N_OUT, 1, Q4_K, O._ptr(out), th)
    el = time.perf_counter() - t0
    b, _ = algorithmic_bytes()
    v = b * args.steps / el / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4", "data": "synthetic",
        "config": {"workload": "configs[1] Q4_K GEMV 151936x2048 batch 1 (reference CPU matmul, nn.c:307)"},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": th, "kind": "reference",
                         "sample": f"{args.steps} steps of the full 151936x2048 matmul"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ----------------------------------------------------------------- GPU leg --
def run_ours(args, world, rank, local):
    import torch
    import qma_cuda as Q
    Q.init(local)
    dev = torch.device("cuda", local)
    W = make_weight()
    rng = np.random.default_rng(rank)
    x = rng.standard_normal((1, N_IN)).astype(np.float32)

    dW = torch.from_numpy(W).to(dev)
    dx = torch.from_numpy(x).to(dev)
    dq = torch.empty((1, N_IN), dtype=torch.int8, device=dev)
    dd = torch.empty((1, N_IN // 256), dtype=torch.float32, device=dev)
    ds = torch.empty((1, N_IN // 16), dtype=torch.int16, device=dev)
    out = torch.empty((1, N_OUT), dtype=torch.float32, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step():
        Q.call("qma_cuda_q8k_quant", Q.ptr(dx), 1, N_IN, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds), sp)
        Q.call("qma_cuda_matvec", Q4_K, Q.ptr(dW), N_IN, N_OUT, 1, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
               Q.ptr(out), sp)

    for _ in range(max(args.warmup, 3)):
        step()
        flush.zero_()
    torch.cuda.synchronize()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        # keep the GPU busy ~0.5 s before the timed region so the sampler sees it
        t_end = time.time() + 0.5
        while time.time() < t_end:
            step()
            flush.zero_()
        torch.cuda.synchronize()
        dist_barrier(world)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(stream)
            Q.call("qma_cuda_q8k_quant", Q.ptr(dx), 1, N_IN, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds), sp)
            ev[i][1].record(stream)
            Q.call("qma_cuda_matvec", Q4_K, Q.ptr(dW), N_IN, N_OUT, 1, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
                   Q.ptr(out), sp)
            ev[i][2].record(stream)
            flush.zero_()
        torch.cuda.synchronize()
        dist_barrier(world)
        torch.cuda.synchronize()
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    gemv_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    step_ms = dist_max(step_ms, world)

    # end to end through the C ABI with host buffers: H2D of x, quantize,
    # GEMV, D2H of the logits row, every step
    hx = torch.from_numpy(x).pin_memory()
    hout = torch.empty((1, N_OUT), dtype=torch.float32).pin_memory()
    for _ in range(3):
        dx.copy_(hx, non_blocking=True); step(); hout.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_ms = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0.record(stream)
        dx.copy_(hx, non_blocking=True)
        step()
        hout.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    e2e_ms = dist_max(e2e_ms, world)

    b, wbytes = algorithmic_bytes()
    value = world * b * args.steps / (step_ms / 1e3) / 1e9
    e2e_value = world * b * args.steps / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    achieved = b / (gemv_ms / args.steps / 1e3) / 1e9

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        import oracle as O
        if O.ref_available():
            v, th, n, el = cpu_reference_rate(W, x)
            cpu = {"value": round(v, 3), "unit": "GB/s", "cores": th, "kind": "reference",
                   "sample": f"{n} full 151936x2048 Q4_K matmuls in {el:.1f} s (reference nn.c:307, {th} pool threads)"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4",
        "data": "synthetic",
        "config": {"workload": "configs[1] Q4_K GEMV 151936x2048 (LM-head shape), batch 1; "
                               "weights N(0,0.02) quantized by the engine's Q4_K quantizer",
                   "l2": "weights 175 MB > L2; 256 MB L2 flush between timed steps",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_kind": peak_kind, "kernel": "gemv_kernel<FmtQ4K,1,32,1>",
                     "algorithmic_bytes_per_launch": b},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": N_IN * 4,
                "d2h_bytes_per_step": N_OUT * 4},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
