#!/usr/bin/env python3
"""Benchmark of the qma B200 engine; rank 0 prints one JSON line.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode|gemv|moe|ep]

decode (default; configs[3]): the full 40-layer random-init qwen35moe
(hidden 2048, 3 GDN + 1 gated attention x 10, 256 experts top-8 + shared,
vocab 151936, Q4_K projections and experts, Q6_K down, Q8_0 embeddings and
LM head) generated on the GPU; an 8192-token prompt of seeded uniform token
ids is prefilled (untimed), then K greedy decode steps at batch 1 are timed
with CUDA events on the engine's stream.  A step streams ~2 GB of weights
(> L2), so no L2 flush is needed.  `e2e` times the same steps through
qma_cuda_eval with the token from and the logits to host memory.

The default line also carries the configs[1] GEMV (`gemv`), the configs[4]
expert-parallel MoE blocks (`ep`) and the configs[4] batched decode of 64
sequences (`batch`, expert-parallel over the N GPUs at N > 1).

gemv: Q4_K 151936x2048 GEMV at batch 1 (quantize + GEMV).

batch: the `batch` leg alone (--prompt, --no-parity).

prefill: 512-token chunks of the full model after a 1024-token prompt.

gdn: one gated-delta-net layer, 1024 decode steps and a
4096-token chunked prefill.

moe: one MoE FFN layer (router, top-8 + shared expert, SwiGLU,
combine, residual) for one decode token through qma_cuda_moe_layer.

ep: the 40 MoE blocks with the 256 experts of every layer
sharded 256/N over the N GPUs, 64 tokens per GPU per step, rows and down
projections exchanged over NCCL (qma_cuda_ep_moe_layer); weak scaling.

For decode, gemv and moe, N > 1 runs one independent replica per GPU (weak
scaling, no collective): a batch-1 decode step does not shard.
--impl reference times the reference's own CPU code (oracle/_ref, built
from its sources) on the host cores for the same workload.
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

BASE_METRIC = "qwen35moe decode tok/s (bs1, 1 GPU) & Q4_K GEMV HBM GB/s vs peak; EP tok/s @2/4/8"
DECODE_METRIC = "qwen35moe decode tok/s (bs1, 1 GPU)"
GEMV_METRIC = "Q4_K GEMV HBM GB/s vs peak"
F32, Q8_0, Q4_K, Q6_K = 0, 8, 12, 14
N_VOCAB = 151936
PROMPT = 8192
N_CTX = 65536
SEED = 0
BATCH_SEQS, BATCH_PROMPT, BATCH_DECODE = 64, 2048, 128     # configs[4]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """SM clock and throttle reasons sampled every 10 ms through NVML while
    the timed region runs (reading only; nvidia-smi at 100 ms if NVML is
    missing)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu, self.samples, self.mx, self.stop = gpu_index, [], None, threading.Event()
        self.thread = None

    def _nvml(self):
        import pynvml as N
        N.nvmlInit()
        h = N.nvmlDeviceGetHandleByIndex(self.gpu)
        self.mx = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
        get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            N.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            self.samples.append((float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)), int(get_reasons(h))))
            time.sleep(0.01)
        N.nvmlShutdown()

    def _smi(self):
        fields = "clocks.sm,clocks.max.sm,clocks_event_reasons.active"
        proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                 "-i", str(self.gpu), "-lms", "100"],
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        threading.Thread(target=lambda: (self.stop.wait(), proc.terminate()), daemon=True).start()
        for line in proc.stdout:
            f = [x.strip() for x in line.split(",")]
            try:
                self.samples.append((float(f[0]), int(f[2], 16)))
                self.mx = float(f[1])
            except (ValueError, IndexError):
                pass

    def _run(self):
        try:
            self._nvml()
        except Exception:
            try:
                self._smi()
            except OSError:
                pass

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        time.sleep(0.05)
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self):
        sm = [c for c, _ in self.samples]
        reasons = sorted({nm for _, r in self.samples for nm, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.mx,
                "reasons": reasons, "samples": len(sm)}


# ------------------------------------------------------------- distributed --
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(v, world):
    """Max of v over the ranks (timings: the slowest rank decides)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# --------------------------------------------------------------- decode ----
def model_layout(lm_type):
    import qma_cuda as Q
    return Q.synth_layout(embd_type=lm_type, out_type=lm_type, down_type=Q6_K, proj_type=Q4_K)


def decode_bytes_per_token(arr, n, live_positions):
    """Algorithmic bytes one decode token moves: every non-expert tensor once
    (projections, norms, router, LM head), one token_embd row, 8 routed + 1
    shared expert per layer, GDN/conv state read+write, and the KV records the
    attention reads (q4 records of K and V for both KV heads)."""
    import qma_cuda as Q
    total = 0
    for i in range(n):
        t = arr[i]
        name = t.name.decode()
        if name == "token_embd.weight":
            total += Q.row_bytes(int(t.type), int(t.ne[0]))
        elif "_exps." in name:
            total += t.nbytes // int(t.ne[2]) * 8
        else:
            total += t.nbytes
    gdn_layers = 30
    total += gdn_layers * 2 * (32 * 128 * 128 * 4 + 8192 * 3 * 4)
    total += 10 * live_positions * 4 * 160
    return int(total)


MOE_TENSORS = ("post_attention_norm.weight", "ffn_gate_inp.weight", "ffn_gate_exps.weight",
               "ffn_up_exps.weight", "ffn_down_exps.weight", "ffn_gate_inp_shexp.weight",
               "ffn_gate_shexp.weight", "ffn_up_shexp.weight", "ffn_down_shexp.weight")
# DRAM bytes (read + write) one MoE block call moves, from the ncu capture of
# the moe workload summarised in profiles/moe_block_configs0.txt
MOE_TRAFFIC_PER_BLOCK = 20624128


def moe_block_bytes(arr, n, il=0):
    """Algorithmic bytes of one MoE block for one token: the router rows and
    norms, 8 routed experts' gate/up/down and the shared expert, the input
    read and the output written."""
    total = 2 * 2048 * 4
    for i in range(n):
        t = arr[i]
        name = t.name.decode()
        if not name.startswith(f"blk.{il}.") or name.split(".", 2)[2] not in MOE_TENSORS:
            continue
        total += t.nbytes // int(t.ne[2]) * 8 if "_exps." in name else t.nbytes
    return int(total)


def time_moe_blocks(weights, rounds, local):
    """Mean device time of one qma_cuda_moe_layer call (one token), cycling
    through the given layers' weights (CUDA events on the launching stream)."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    dev = torch.device("cuda", local)
    x2 = torch.randn((1, 2048), dtype=torch.float32, device=dev)
    out = torch.empty_like(x2)
    scratch = torch.empty(Q.lib().qma_cuda_moe_scratch_bytes(1), dtype=torch.uint8, device=dev)
    ms = torch.cuda.Stream(device=dev)
    sp = ms.cuda_stream

    def one(w):
        Q.call("qma_cuda_moe_layer", C.byref(w), Q.ptr(x2), 1, Q.ptr(out), None, None, Q.ptr(scratch),
               scratch.numel(), sp)

    torch.cuda.synchronize()
    for w in weights:
        one(w)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ms)
    for _ in range(rounds):
        for w in weights:
            one(w)
    e1.record(ms)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (rounds * len(weights))


def run_decode_ours(args, world, rank, local):
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    arr, n, size = model_layout(Q8_0)
    tp = C.cast(arr, C.POINTER(Q.Tensor))
    t0 = time.time()
    model = Q.Model(tp, n, seed=SEED, device=local)
    torch.cuda.synchronize()
    t_model = time.time() - t0
    st = Q.State(model, N_CTX)
    stream = torch.cuda.ExternalStream(Q.lib().qma_cuda_state_stream(st.h), device=local)
    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, N_VOCAB, args.prompt).astype(np.int32)
    torch.cuda.nvtx.range_push("prefill")
    t0 = time.time()
    logits = st.eval(prompt)
    t_prefill = time.time() - t0
    torch.cuda.nvtx.range_pop()
    tok = int(np.argmax(logits))
    toks, logits = st.decode_greedy(tok, max(args.warmup, 3))
    tok = int(np.argmax(logits))

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        dist_barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        e0.record(stream)
        toks, logits = st.decode_greedy(tok, args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        dist_barrier(world)
    ms_raw = dist_max(e0.elapsed_time(e1), world)
    tok = int(np.argmax(logits))
    nk_pos = st.n_pos

    # The live index is rebuilt every 128 positions (nn.c:2074-2088), which a
    # short timed window may miss: time one 128-step window that holds
    # exactly one rebuild and fold its extra cost, amortised over 128 steps,
    # into the reported step time.
    dist_barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    toks, logits = st.decode_greedy(int(np.argmax(logits)), HCM_EVERY)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_128 = dist_max(e0.elapsed_time(e1), world)
    tok = int(np.argmax(logits))
    rebuild_extra = max(0.0, ms_128 - HCM_EVERY * ms_raw / args.steps)
    ms = ms_raw + args.steps * rebuild_extra / HCM_EVERY
    kernels, sbytes = C.c_int(0), C.c_uint64(0)
    Q.call("qma_cuda_state_stats", st.h, C.byref(kernels), C.byref(sbytes))

    # end to end: one qma_cuda_eval per token, token H2D and logits D2H
    e2e_steps = min(args.steps, 64)
    e2e_ms = 0.0
    for _ in range(e2e_steps):
        e0.record(stream)
        logits = st.eval(np.array([tok], np.int32))
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms += e0.elapsed_time(e1)
        tok = int(np.argmax(logits))
    e2e_ms = dist_max(e2e_ms, world)

    # the dominant kernel pair (router + experts, the largest share of the
    # step): one MoE block per call through the C ABI, every layer in turn
    wts = []
    for il in range(40):
        w = Q.MoeWeights()
        Q.call("qma_cuda_model_moe_weights", model.h, il, C.byref(w))
        wts.append(w)
    moe_us = dist_max(time_moe_blocks(wts, 8, local), world)
    moe_b = moe_block_bytes(arr, n)
    ep = None if args.no_ep else run_ep_on_model(model, wts, args, world, rank, local)
    batch = None if args.no_batch else run_batch_on_model(model, wts, args, world, rank, local)

    value = world * args.steps / (ms / 1e3)
    e2e_value = world * e2e_steps / (e2e_ms / 1e3)
    live = min(nk_pos, 4 + 4096 + 2048) + 64
    bpt = decode_bytes_per_token(arr, n, live)
    peak, peak_kind = load_peaks()
    achieved = bpt * (args.steps / (ms / 1e3)) / 1e9
    st.close()
    model.close()
    gemv = None if args.no_gemv else gemv_measure(args, world, rank, local)
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_decode_baseline(seconds=20.0)
    line = {
        "metric": DECODE_METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4",
        "data": "synthetic: random-init weights (seeded N(0,0.02), engine quantizers) and uniform random prompt ids",
        "config": {"workload": "configs[3] full qwen35moe decode bs1: 40 layers (3 GDN + 1 attn) x10, "
                               "256 experts top-8 + shared, vocab 151936, Q4_K experts/projections, "
                               f"Q6_K down, Q8_0 embeddings + LM head; {args.prompt}-token prompt (prefill untimed), "
                               "then greedy decode; KV ring n_ctx 65536 with 4/2-bit tiers (sink 4, hot 4096)",
                   "model": "qwen35moe-random-init", "global_batch": 1, "seq_len": args.prompt,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "each step streams ~2 GB of weights (> 126 MB L2)",
                   "prefill_s": round(t_prefill, 2), "model_synth_s": round(t_model, 2),
                   "hcm_rebuild": {"every_steps": HCM_EVERY, "extra_ms": round(rebuild_extra, 4),
                                   "window_128_ms": round(ms_128, 3),
                                   "timed_steps_ms": round(ms_raw, 3),
                                   "note": "value and ms_per_step include the rebuild cost amortised over "
                                           "128 steps"},
                   "reference_arm": "the reference's CPU qma_eval decodes after a 16-token prompt (not 8192) "
                                    "with a Q6_K LM head (it has no Q8_0 kernels); both favour it",
                   "base_metric": BASE_METRIC},
        "roofline": {"bound": "hbm", "achieved": round(moe_b / (moe_us * 1e3), 1), "peak": peak, "unit": "GB/s",
                     "frac": round(moe_b / (moe_us * 1e3) / peak, 4), "traffic": MOE_TRAFFIC_PER_BLOCK,
                     "peak_kind": peak_kind,
                     "kernel": "MoE block: moe_router_kernel + moe_expert_kernel<FmtQ6K> via qma_cuda_moe_layer, "
                               "one token, the 40 layers' weights in turn",
                     "us_per_launch": round(moe_us, 2), "algorithmic_bytes_per_launch": moe_b},
        "step_roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(achieved / peak, 4), "kernel": "whole decode step (one CUDA graph)",
                          "algorithmic_bytes_per_step": bpt},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": N_VOCAB * 4},
        "gpu_launches": int(kernels.value) * args.steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "gemv": gemv,
        "ep": ep,
        "batch": batch,
    }
    print(json.dumps(line), flush=True)
    if ep is not None and not ep.get("ep_parity"):
        sys.exit("expert-parallel parity check failed: " + json.dumps(ep.get("parity_detail")))
    if batch is not None and not batch.get("parity"):
        sys.exit("batched decode parity check failed: " + json.dumps(batch.get("parity_detail")))


def host_blob_for_reference(threads):
    """The same random-init model for the reference, with Q6_K embeddings and
    LM head (the reference has no Q8_0 weight kernels, gguf.c:272-287)."""
    import ctypes as C
    import oracle as O
    qarr, n, size = model_layout(Q6_K)
    arr = C.cast(qarr, C.POINTER(O.Tensor))         # the same struct, the oracle's ctypes class
    blob = O.synth_blob(arr, n, size, seed=SEED, threads=threads)
    return arr, n, size, blob


def cpu_decode_baseline(seconds=20.0, threads=None, prompt_len=16):
    """The reference's qma_eval (oracle/_ref) decoding on the host cores over
    a bounded sample: a short prompt, then greedy steps for ~`seconds`."""
    import oracle as O
    if not O.ref_available():
        return None
    th = threads or min(os.cpu_count() or 1, 16)
    arr, n, size, blob = host_blob_for_reference(os.cpu_count() or 1)
    R = O.ref()
    R.qr_init(th)
    rm = R.qr_model_new(arr, n, O._ptr(blob), size)
    rs = R.qr_state_new(4096)
    logits = np.zeros(N_VOCAB, np.float32)
    prompt = np.random.default_rng(SEED).integers(0, N_VOCAB, prompt_len).astype(np.int32)
    R.qr_eval(rm, rs, O._ptr(prompt), prompt_len, O._ptr(logits), th, 0)
    steps, t0 = 0, time.perf_counter()
    while True:
        one = np.array([int(np.argmax(logits))], np.int32)
        R.qr_eval(rm, rs, O._ptr(one), 1, O._ptr(logits), th, 0)
        steps += 1
        el = time.perf_counter() - t0
        if steps >= 3 and el >= seconds:
            break
    R.qr_state_free(rs)
    R.qr_model_free(rm)
    return {"value": round(steps / el, 4), "unit": "tok/s", "cores": th, "kind": "reference",
            "sample": f"{steps} greedy decode tokens after a {prompt_len}-token prompt, {el:.1f} s, "
                      f"reference qma_eval (nn.c:2056) with {th} pool threads; Q6_K LM head "
                      f"(the reference has no Q8_0 kernels)"}


# --------------------------------------------- expert parallel on the model --
HCM_EVERY = 128          # HCM_REBUILD, nn.c:894-901
EP_SEQS = 64             # configs[4]: 64 concurrent sequences in total, 64 / N per GPU


def shard_weights(w, e0, n_local):
    """A copy of layer weights w whose routed expert tables start at expert
    e0 (the rank's shard): gate / up Q4_K experts and packed Q6_K down."""
    import qma_cuda as Q
    s = Q.MoeWeights()
    C_ = __import__("ctypes")
    C_.memmove(C_.byref(s), C_.byref(w), C_.sizeof(w))
    s.gate_exps = w.gate_exps + e0 * Q4K_EXPERT
    s.up_exps = w.up_exps + e0 * Q4K_EXPERT
    s.down_exps = w.down_exps + e0 * Q.packed_bytes(Q6_K, 2048, 512)
    return s


def ep_inputs(world):
    """configs[4]'s 64 sequences, one decode token each, split 64 / N per
    rank: rank r's tokens are rows r * 64/N .. of one seeded matrix."""
    return np.random.default_rng(SEED + 7).standard_normal((EP_SEQS, 2048)).astype(np.float32)


def run_ep_on_model(model, full_w, args, world, rank, local):
    """configs[4]'s expert-parallel MoE on the decode model's own weights:
    the 256 experts of each of the 40 layers sharded 256/N over the N ranks
    (rank r serves experts r*256/N ..), 64 sequences in total with 64/N
    decode tokens per GPU, NCCL dispatch and return (qma_cuda_ep_moe_layer).
    A step runs the 40 MoE blocks in sequence.

    Parity, before timing: each rank's first layer-0 call must equal, bit
    for bit, the one-GPU MoE block (qma_cuda_moe_layer, its grouped path)
    run on all 64 tokens, rank's slice, and its expert selection must equal
    the oracle's routing (nn.c:513-551 restated) of the same tokens; the
    result is the AND over ranks.  At N > 1, rank 0 also times the same 64
    tokens with every expert local (ep1) for the scaling comparison."""
    import ctypes as C
    import torch
    import oracle as O
    import qma_cuda as Q
    dev = torch.device("cuda", local)
    T = EP_SEQS // world
    e0, n_local = Q.ep_shard(rank, world)
    # configs[4]'s router prior: log Zipf(1.1) over a seeded per-layer expert
    # ranking, added to every router logit (a skewed expert load)
    bias_h = [O.zipf_router_bias(SEED, il) for il in range(len(full_w))]
    bias_d = [torch.from_numpy(b).to(dev) for b in bias_h]
    full_w = [shard_weights(w, 0, 0) for w in full_w]          # copies
    for w, b in zip(full_w, bias_d):
        w.router_bias = b.data_ptr()
    shard = [shard_weights(w, e0, n_local) for w in full_w]
    X = ep_inputs(world)
    mine = X[rank * T:(rank + 1) * T]
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    ep = Q.ExpertParallel(local, rank, world, T, ep_share_uid(world), timeout_ms=300000)

    # ---- parity ------------------------------------------------------------
    x0 = torch.from_numpy(mine).to(dev)
    y = torch.empty_like(x0)
    sel = torch.empty((T, 8), dtype=torch.int32, device=dev)
    ep.moe_layer(shard[0], x0, T, y, sel, None, sp)
    dX = torch.from_numpy(X).to(dev)
    Y = torch.empty_like(dX)
    SEL = torch.empty((EP_SEQS, 8), dtype=torch.int32, device=dev)
    nb = Q.lib().qma_cuda_moe_scratch_bytes(EP_SEQS)
    scratch = torch.empty(nb, dtype=torch.uint8, device=dev)
    Q.call("qma_cuda_moe_layer", C.byref(full_w[0]), Q.ptr(dX), EP_SEQS, Q.ptr(Y), Q.ptr(SEL), None,
           Q.ptr(scratch), nb, sp)
    torch.cuda.synchronize()
    got, want = y.cpu().numpy(), Y.cpu().numpy()[rank * T:(rank + 1) * T]
    gsel = sel.cpu().numpy()
    pn = np.frombuffer(ctypes_read(full_w[0].post_norm, 2048 * 4), np.float32)
    gi = np.frombuffer(ctypes_read(full_w[0].gate_inp, 256 * 2048 * 4), np.float32).reshape(256, 2048)
    osel, _ = O.moe_route(pn, gi, mine, bias=bias_h[0])
    cnt = np.bincount(SEL.cpu().numpy().ravel(), minlength=256)
    expert_load = {"layer": 0, "distinct_experts": int(np.count_nonzero(cnt)), "max_pairs_per_expert": int(cnt.max()),
                   "pairs": int(cnt.sum())}
    bit = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    sel_gpu = bool(np.array_equal(gsel, SEL.cpu().numpy()[rank * T:(rank + 1) * T]))
    sel_oracle = bool(np.array_equal(gsel, osel))
    ok_all = dist_min(float(bit and sel_gpu and sel_oracle), world) > 0.5
    detail = {"bit_equal_one_gpu": bit, "sel_equal_one_gpu": sel_gpu, "sel_equal_oracle": sel_oracle,
              "max_abs_diff": float(np.abs(got - want).max())}
    del dX, Y, SEL, scratch

    # ---- timing --------------------------------------------------------------
    def run(handle, layers, xin, tt, warm):
        buf = [torch.empty_like(xin), torch.empty_like(xin)]

        def step(src):
            buf[0].copy_(src, non_blocking=True)
            for il, w in enumerate(layers):
                handle.moe_layer(w, buf[il & 1], tt, buf[(il + 1) & 1], None, None, sp)
            return buf[len(layers) & 1]

        for _ in range(warm):
            step(xin)
        torch.cuda.synchronize()
        return step

    step = run(ep, shard, x0, T, max(args.warmup, 3))
    net = [0, 0]
    for il in range(EP_LAYERS):
        ep.moe_layer(shard[il], x0, T, y, None, None, sp)
        s_, r_, _ = ep.stats()
        net[0] += s_
        net[1] += r_
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_barrier(world)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        step(x0)
    ev1.record(stream)
    torch.cuda.synchronize()
    t_ms = dist_max(ev0.elapsed_time(ev1), world)
    # end to end: the step's tokens from pinned host memory, its output back
    hx = torch.from_numpy(mine).pin_memory()
    hout = torch.empty((T, 2048), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps // 4)
    dist_barrier(world)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(e2e_steps):
        hout.copy_(step(hx.to(dev, non_blocking=True)), non_blocking=True)
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist_max(ev0.elapsed_time(ev1), world)
    ep.close()

    ep1_value = None
    if world > 1:
        # rank 0 alone: the same 64 tokens, every expert local (ep1)
        dist_barrier(world)
        if rank == 0:
            ep1 = Q.ExpertParallel(local, 0, 1, EP_SEQS, lambda u: u, timeout_ms=300000)
            xa = torch.from_numpy(X).to(dev)
            step1 = run(ep1, full_w, xa, EP_SEQS, max(args.warmup, 3))
            ev0.record(stream)
            for _ in range(args.steps):
                step1(xa)
            ev1.record(stream)
            torch.cuda.synchronize()
            ep1_value = EP_SEQS * args.steps / (ev0.elapsed_time(ev1) / 1e3)
            ep1.close()
        dist_barrier(world)
    value = EP_SEQS * args.steps / (t_ms / 1e3)
    return {
        "metric": "EP tok/s @N (40 qwen35moe MoE blocks per step, experts sharded 256/N)",
        "tok_per_s": round(value, 1), "ms_per_step": round(t_ms / args.steps, 4), "n_ranks": world,
        "tokens_per_gpu": T, "sequences": EP_SEQS, "scaling": "strong (64 sequences in total)",
        "ep1_tok_per_s": round(ep1_value, 1) if ep1_value else (round(value, 1) if world == 1 else None),
        "e2e_tok_per_s": round(EP_SEQS * e2e_steps / (e2e_ms / 1e3), 1),
        "exchange": {"sent_bytes_per_step": net[0], "recv_bytes_per_step": net[1], "rank": rank,
                     "note": "rank 0's NCCL transfers, its own share included (over NVLink at N > 1)"},
        "ep_parity": ok_all, "parity_detail": detail,
        "router_prior": "log Zipf(s=1.1) over a seeded per-layer expert ranking, added to every router logit",
        "expert_load": expert_load,
        "collectives": "per layer: grouped NCCL send/recv of fixed blocks of 64/N rows per peer (dispatch) and of "
                       "their slot partials (return); no host synchronisation"
                       if not os.environ.get("QMA_CUDA_EP_COUNTED") else
                       "per layer: NCCL all-gather of the counts (read on the host), exact-size send/recv",
    }


def dist_gather_i64(vals, world):
    """vals (int64 [k], the same k on every rank) of every rank, in rank
    order (an NCCL all-gather through the process group)."""
    vals = np.ascontiguousarray(vals, np.int64)
    if world == 1:
        return [vals]
    import torch
    import torch.distributed as dist
    t = torch.from_numpy(vals)
    if dist.get_backend() == "nccl":
        t = t.cuda()
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.cpu().numpy() for o in out]


def logits_digest(rows):
    """One int64 per logits row: a hash of its exact bytes."""
    import hashlib
    return np.array([int.from_bytes(hashlib.blake2b(np.ascontiguousarray(r).tobytes(), digest_size=8).digest(),
                                    "little", signed=True) for r in rows], np.int64)


def run_batch_on_model(model, full_w, args, world, rank, local, prompt_len=None, check=True, max_steps=None):
    """configs[4] end to end: 64 concurrent sequences of the full model,
    each prefilled with its own 2048-token prompt (seeded ids, untimed), then
    decoded greedily in batched steps of one token per sequence
    (qma_cuda_batch_eval: host token ids in, greedy ids out) to 128 tokens
    each, the router biased by the log-Zipf(1.1) prior.  At N > 1 the 64
    sequences are split 64/N per GPU (attention and gated-delta state are
    per sequence) and every MoE block runs expert-parallel over the N GPUs
    (experts sharded 256/N, NCCL exchange per layer).

    Parity, before timing, on 64 sequences with 32-token prompts and three
    decode steps: at N > 1 every sequence's logits must equal, bit for bit,
    those of rank 0 decoding all 64 sequences alone on one GPU (local MoE
    blocks); at N = 1 a 64-row step must equal the same sequences stepped
    as four steps of 16 rows.  A mismatch makes the run exit non-zero."""
    import ctypes as C
    import torch
    import oracle as O
    import qma_cuda as Q
    dev = torch.device("cuda", local)
    n_here = BATCH_SEQS // world
    first = rank * n_here
    bias_d = [torch.from_numpy(O.zipf_router_bias(SEED, il)).to(dev) for il in range(len(full_w))]
    for il, b in enumerate(bias_d):
        Q.call("qma_cuda_model_set_router_bias", model.h, il, b.data_ptr())
    ep, shard = None, None
    if world > 1:
        e0, n_local = Q.ep_shard(rank, world)
        shard = []
        for w, b in zip(full_w, bias_d):
            s_ = shard_weights(w, e0, n_local)
            s_.router_bias = b.data_ptr()
            shard.append(s_)
        ep = Q.ExpertParallel(local, rank, world, n_here, ep_share_uid(world), timeout_ms=300000)

    def prompts(n_tok, seed):
        return [np.random.default_rng([seed, g]).integers(0, N_VOCAB, n_tok).astype(np.int32)
                for g in range(BATCH_SEQS)]

    def prefill(batch, pr, ids):
        sids = np.concatenate([np.full(len(pr[g]), i, np.int32) for i, g in enumerate(ids)])
        lo, g = batch.eval(sids, np.concatenate([pr[g] for g in ids]), logits=False, greedy=True)
        ends = np.cumsum([len(pr[g]) for g in ids]) - 1
        return g[ends].astype(np.int32)

    prompt_len = prompt_len or BATCH_PROMPT
    mine = list(range(first, first + n_here))
    sids = np.arange(n_here, dtype=np.int32)
    ok, detail = True, {"skipped": True}
    if check:
        # ---- parity ----------------------------------------------------------------
        P_TOK, P_STEPS = 32, 3
        pr = prompts(P_TOK, SEED + 11)
        b = Q.Batch(model, n_here, 4096)
        tok = prefill(b, pr, mine)
        if ep is not None:
            b.set_ep(ep, shard)
        digests = []
        for _ in range(P_STEPS):
            lo, g = b.eval(sids, tok)
            digests.append(logits_digest(lo))
            tok = g.astype(np.int32)
        b.close()
        got = np.concatenate([np.concatenate(dist_gather_i64(d, world)) for d in digests])
        detail = {}
        if rank == 0:
            ref = Q.Batch(model, BATCH_SEQS, 4096)
            tok = prefill(ref, pr, list(range(BATCH_SEQS)))
            allids = np.arange(BATCH_SEQS, dtype=np.int32)
            want = []
            for _ in range(P_STEPS):
                if world > 1:
                    lo, g = ref.eval(allids, tok)
                else:
                    lo = np.empty((BATCH_SEQS, N_VOCAB), np.float32)
                    g = np.empty(BATCH_SEQS, np.int32)
                    for q in range(0, BATCH_SEQS, 16):
                        l_, g_ = ref.eval(allids[q:q + 16], tok[q:q + 16])
                        lo[q:q + 16], g[q:q + 16] = l_, g_
                want.append(logits_digest(lo))
                tok = g.astype(np.int32)
            ref.close()
            want = np.concatenate(want)
            ok = bool(np.array_equal(got, want))
            detail = {"rows_compared": int(want.size), "rows_equal": int((got == want).sum()),
                      "reference": "rank 0 alone, all 64 sequences, local MoE blocks" if world > 1
                      else "the same sequences stepped 16 rows at a time"}
    ok = dist_min(float(ok), world) > 0.5

    # ---- timed: prompt_len-token prompts (2048), 128 decode tokens per sequence ----
    pr = prompts(prompt_len, SEED + 12)
    b = Q.Batch(model, n_here, prompt_len + 256)
    t0 = time.time()
    tok = prefill(b, pr, mine)
    t_prefill = dist_max(time.time() - t0, world)
    if ep is not None:
        b.set_ep(ep, shard)
    stream = torch.cuda.ExternalStream(Q.lib().qma_cuda_state_stream(Q.lib().qma_cuda_batch_seq(b.h, 0)),
                                       device=local)
    warm = max(args.warmup, 3)
    steps = max(1, BATCH_DECODE - warm)
    if max_steps:
        steps = max(1, min(steps, max_steps))
    for _ in range(warm):
        _, g = b.eval(sids, tok, logits=False)
        tok = g.astype(np.int32)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_barrier(world)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("capture")
    ev0.record(stream)
    for _ in range(steps):
        _, g = b.eval(sids, tok, logits=False)
        tok = g.astype(np.int32)
    ev1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    t_ms = dist_max(ev0.elapsed_time(ev1), world)
    n_pos = b.n_pos(0)
    b.close()
    if ep is not None:
        ep.close()
    for il in range(len(full_w)):
        Q.call("qma_cuda_model_set_router_bias", model.h, il, None)
    torch.cuda.synchronize()
    del bias_d
    value = BATCH_SEQS * steps / (t_ms / 1e3)
    return {
        "metric": "batched decode tok/s @N (configs[4]: 64 sequences, full model, EP over N GPUs)",
        "tok_per_s": round(value, 1), "ms_per_step": round(t_ms / steps, 3), "n_ranks": world,
        "sequences": BATCH_SEQS, "sequences_per_gpu": n_here, "prompt_tokens": prompt_len,
        "decode_tokens_per_sequence": warm + steps, "timed_steps": steps, "positions_at_end": n_pos,
        "prefill_s": round(t_prefill, 2),
        "moe": "expert-parallel, 256/N experts per GPU, NCCL exchange per layer" if world > 1
               else "local (all 256 experts on the GPU)",
        "api": "qma_cuda_batch_eval per step: token ids H2D, greedy ids D2H, host loop",
        "h2d_bytes_per_step": n_here * 8, "d2h_bytes_per_step": n_here * 4,
        "router_prior": "log Zipf(s=1.1) over a seeded per-layer expert ranking",
        "parity": ok, "parity_detail": detail,
    }


def ctypes_read(dptr, nbytes):
    """Bytes of device memory at the raw address dptr, copied to the host
    (the CUDA runtime's cudaMemcpy; the engine library loaded it)."""
    import ctypes as C
    rt = C.CDLL("libcudart.so.12")
    out = np.empty(nbytes, np.uint8)
    rc = rt.cudaMemcpy(C.c_void_p(out.ctypes.data), C.c_void_p(int(dptr)), C.c_size_t(nbytes), 2)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy device to host failed: {rc}")
    return out.tobytes()


def dist_min(v, world):
    return -dist_max(-v, world)


def run_decode_reference(args, world, rank):
    if rank != 0:
        return
    import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent at build time)"}))
        return
    th = min(os.cpu_count() or 1, 16)
    arr, n, size, blob = host_blob_for_reference(os.cpu_count() or 1)
    R = O.ref()
    R.qr_init(th)
    rm = R.qr_model_new(arr, n, O._ptr(blob), size)
    rs = R.qr_state_new(4096)
    logits = np.zeros(N_VOCAB, np.float32)
    prompt = np.random.default_rng(SEED).integers(0, N_VOCAB, 16).astype(np.int32)
    R.qr_eval(rm, rs, O._ptr(prompt), len(prompt), O._ptr(logits), th, 0)
    for _ in range(args.warmup):
        one = np.array([int(np.argmax(logits))], np.int32)
        R.qr_eval(rm, rs, O._ptr(one), 1, O._ptr(logits), th, 0)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one = np.array([int(np.argmax(logits))], np.int32)
        R.qr_eval(rm, rs, O._ptr(one), 1, O._ptr(logits), th, 0)
    el = time.perf_counter() - t0
    v = args.steps / el
    print(json.dumps({
        "impl": "reference", "metric": DECODE_METRIC, "value": round(v, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xq4", "data": "synthetic",
        "config": {"workload": "configs[3] qwen35moe decode bs1 on the reference's CPU qma_eval "
                               "(16-token prompt, Q6_K LM head: the reference has no Q8_0 kernels)",
                   "model": "qwen35moe-random-init", "global_batch": 1},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": th, "kind": "reference",
                         "sample": f"{args.steps} greedy decode steps after a 16-token prompt"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------ gemv ---
GN_OUT, GN_IN = 151936, 2048


def gemv_bytes(rows=GN_OUT, cols=GN_IN):
    w = rows * (cols // 256) * 144
    return w + cols * 4 + cols + (cols // 256) * 4 + (cols // 16) * 2 + rows * 4


def gemv_measure(args, world, rank, local):
    """configs[1]'s LM-head-shaped Q4_K GEMV (151936 x 2048, batch 1) in the
    decode run: the GB/s of its kernel and the fraction of the measured HBM
    peak (rank 0's figure; L2 flushed between timed launches)."""
    import argparse as A
    sub = A.Namespace(**vars(args))
    sub.rows, sub.cols, sub.steps, sub.warmup = GN_OUT, GN_IN, 20, 3
    return run_gemv_ours(sub, world, rank, local, as_dict=True)


def run_gemv_ours(args, world, rank, local, as_dict=False):
    import torch
    import qma_cuda as Q
    Q.init(local)
    GN_OUT, GN_IN = args.rows, args.cols
    dev = torch.device("cuda", local)
    # the weights from the engine's synthetic generator, on the device
    dW = torch.empty(GN_OUT * Q.row_bytes(Q4_K, GN_IN), dtype=torch.uint8, device=dev)
    Q.call("qma_cuda_synth_tensor", b"bench.lm_head", Q4_K, GN_OUT * GN_IN, 0, Q.ptr(dW), None)
    x = np.random.default_rng(rank).standard_normal((1, GN_IN)).astype(np.float32)
    dx = torch.from_numpy(x).to(dev)
    dq = torch.empty((1, GN_IN), dtype=torch.int8, device=dev)
    dd = torch.empty((1, GN_IN // 256), dtype=torch.float32, device=dev)
    ds = torch.empty((1, GN_IN // 16), dtype=torch.int16, device=dev)
    out = torch.empty((1, GN_OUT), dtype=torch.float32, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def quant():
        Q.call("qma_cuda_q8k_quant", Q.ptr(dx), 1, GN_IN, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds), sp)

    def gemv():
        Q.call("qma_cuda_matvec", Q4_K, Q.ptr(dW), GN_IN, GN_OUT, 1, Q.ptr(dq), Q.ptr(dd), Q.ptr(ds),
               Q.ptr(out), sp)

    for _ in range(max(args.warmup, 3)):
        quant(); gemv(); flush.zero_()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        t_end = time.time() + 0.5
        while time.time() < t_end:
            quant(); gemv(); flush.zero_()
        torch.cuda.synchronize()
        dist_barrier(world)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(stream); quant(); ev[i][1].record(stream); gemv(); ev[i][2].record(stream)
            flush.zero_()
        torch.cuda.synchronize()
        dist_barrier(world)
    step_ms = dist_max(sum(e[0].elapsed_time(e[2]) for e in ev), world)
    gemv_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    hx = torch.from_numpy(x).pin_memory()
    hout = torch.empty((1, GN_OUT), dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_ms = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0.record(stream)
        dx.copy_(hx, non_blocking=True); quant(); gemv(); hout.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    e2e_ms = dist_max(e2e_ms, world)
    b = gemv_bytes(GN_OUT, GN_IN)
    peak, peak_kind = load_peaks()
    achieved = b / (gemv_ms / args.steps / 1e3) / 1e9
    if as_dict:
        return {"metric": GEMV_METRIC, "shape": f"{GN_OUT}x{GN_IN} Q4_K, batch 1", "gbs": round(achieved, 1),
                "peak": peak, "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "us_per_launch": round(gemv_ms / args.steps * 1e3, 2), "algorithmic_bytes_per_launch": b,
                "kernel": "gemv_stream_kernel<FmtQ4K,1>", "l2": "256 MB L2 flush between timed launches",
                "steps": args.steps}
    if rank != 0:
        return
    print(json.dumps({
        "metric": GEMV_METRIC, "value": round(world * b * args.steps / (step_ms / 1e3) / 1e9, 2),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xq4", "data": "synthetic",
        "config": {"workload": f"{'configs[1] ' if (GN_OUT, GN_IN) == (151936, 2048) else ''}Q4_K GEMV {GN_OUT}x{GN_IN}, batch 1",
                   "l2": "256 MB L2 flush between timed steps", "base_metric": BASE_METRIC},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "gemv_stream_kernel<FmtQ4K,1> (per-SM row stream through 4 shared-memory stages)"
                               if GN_OUT * GN_IN // 256 * 144 > 148 * 160 * 1024
                               else "gemv_staged_kernel<FmtQ4K,32,1,2> (rows staged in shared memory)",
                     "algorithmic_bytes_per_launch": b},
        "e2e": {"value": round(world * b * args.steps / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": GN_IN * 4, "d2h_bytes_per_step": GN_OUT * 4},
        "gpu_launches": 2 * args.steps, "clocks": clk.summary(), "cpu_baseline": None,
    }), flush=True)



# ------------------------------------------------------------------- moe ---
MOE_METRIC = "MoE FFN layer GB/s (one decode token)"


def run_moe_ours(args, world, rank, local):
    """one MoE FFN layer for one token, weights generated on the
    GPU by the engine's synthetic generator (seed 0), activation ~N(0, 1);
    a 256 MB L2 flush between timed calls."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    dev = torch.device("cuda", local)
    arr, n, size = model_layout(Q8_0)
    idx = Q.tensor_index(arr, n)
    d = {}
    for name in MOE_TENSORS:
        t = arr[idx[f"blk.0.{name}"]]
        raw = torch.empty(int(t.nbytes), dtype=torch.uint8, device=dev)
        nel = int(t.ne[0]) * int(t.ne[1]) * int(t.ne[2])
        Q.call("qma_cuda_synth_tensor", t.name, int(t.type), nel, SEED, Q.ptr(raw), None)
        if "down" in name and int(t.type) != Q4_K:
            rows, n_in, nexp = int(t.ne[1]), int(t.ne[0]), int(t.ne[2])
            pb, gb = Q.packed_bytes(int(t.type), rows, n_in), Q.row_bytes(int(t.type), n_in) * rows
            packed = torch.empty(pb * nexp, dtype=torch.uint8, device=dev)
            for e in range(nexp):
                Q.call("qma_cuda_repack", int(t.type), raw.data_ptr() + e * gb, rows, n_in,
                       packed.data_ptr() + e * pb, None)
            raw = packed
        d[name] = raw
    w = Q.MoeWeights(*[d[k].data_ptr() for k in MOE_TENSORS], Q6_K, Q6_K)
    x = np.random.default_rng(SEED + rank).standard_normal((1, 2048)).astype(np.float32)
    dx = torch.from_numpy(x).to(dev)
    out = torch.empty_like(dx)
    scratch = torch.empty(Q.lib().qma_cuda_moe_scratch_bytes(1), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def moe():
        Q.call("qma_cuda_moe_layer", C.byref(w), Q.ptr(dx), 1, Q.ptr(out), None, None, Q.ptr(scratch),
               scratch.numel(), sp)

    for _ in range(max(args.warmup, 3)):
        moe(); flush.zero_()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        dist_barrier(world)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(stream); moe(); ev[i][1].record(stream)
            flush.zero_()
        torch.cuda.synchronize()
        dist_barrier(world)
    t_ms = dist_max(sum(e[0].elapsed_time(e[1]) for e in ev), world)
    hx = torch.from_numpy(x).pin_memory()
    hout = torch.empty((1, 2048), dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_ms = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0.record(stream)
        dx.copy_(hx, non_blocking=True); moe(); hout.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    e2e_ms = dist_max(e2e_ms, world)
    b = moe_block_bytes(arr, n)
    peak, peak_kind = load_peaks()
    achieved = b / (t_ms / args.steps / 1e3) / 1e9
    if rank != 0:
        return
    print(json.dumps({
        "metric": MOE_METRIC, "value": round(world * achieved, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4",
        "data": "synthetic",
        "config": {"workload": "configs[0] one qwen35moe MoE FFN layer (router 2048x256 fp32, top-8 + shared "
                               "expert, Q4_K gate/up, Q6_K down), one decode token",
                   "l2": "256 MB L2 flush between timed steps", "base_metric": BASE_METRIC},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": MOE_TRAFFIC_PER_BLOCK, "peak_kind": peak_kind,
                     "kernel": "MoE block: moe_router_kernel + moe_expert_kernel<FmtQ6K>",
                     "algorithmic_bytes_per_launch": b},
        "e2e": {"value": round(world * b * args.steps / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": 2048 * 4, "d2h_bytes_per_step": 2048 * 4},
        "gpu_launches": 2 * args.steps, "clocks": clk.summary(), "cpu_baseline": None,
    }), flush=True)


# -------------------------------------------------------- expert parallel --
EP_METRIC = "EP tok/s (qwen35moe MoE blocks, experts sharded 256/N)"
EP_T = 64                     # tokens per GPU per step: one decode step of 64 sequences
EP_LAYERS = 40
EP_LAUNCHES_PER_LAYER = 14    # router, plan, pack, lists, 2 x (gate/up, SwiGLU, down), recv plan, gather, unpack, combine
Q4K_EXPERT = 512 * (2048 // 256) * 144      # gate or up rows of one expert
Q6K_EXPERT_GGUF = 2048 * (512 // 256) * 210  # down rows of one expert, GGUF layout


def ep_share_uid(world):
    """The communicator id from rank 0 to every rank through the process
    group (qma_cuda.ExpertParallel's share_uid)."""
    def share(uid):
        obj = [uid]
        if world > 1:
            import torch.distributed as dist
            dist.broadcast_object_list(obj, src=0)
        return obj[0]
    return share


def ep_layer_weights(il, e0, n_local, dev):
    """Layer il's MoE weights on the device with only experts e0 ..
    e0 + n_local - 1 of the routed tables (the synthetic generator's bytes
    of the whole tensor, sliced; down projections repacked)."""
    import torch
    import qma_cuda as Q
    spec = [("post_attention_norm.weight", F32, 2048), ("ffn_gate_inp.weight", F32, 2048 * 256),
            ("ffn_gate_exps.weight", Q4_K, 2048 * 512 * 256), ("ffn_up_exps.weight", Q4_K, 2048 * 512 * 256),
            ("ffn_down_exps.weight", Q6_K, 512 * 2048 * 256), ("ffn_gate_inp_shexp.weight", F32, 2048),
            ("ffn_gate_shexp.weight", Q4_K, 2048 * 512), ("ffn_up_shexp.weight", Q4_K, 2048 * 512),
            ("ffn_down_shexp.weight", Q6_K, 512 * 2048)]
    nbytes = {F32: lambda n: 4 * n, Q4_K: lambda n: n // 256 * 144, Q6_K: lambda n: n // 256 * 210}
    pb = Q.packed_bytes(Q6_K, 2048, 512)
    d = {}
    for name, typ, nel in spec:
        raw = torch.empty(nbytes[typ](nel), dtype=torch.uint8, device=dev)
        Q.call("qma_cuda_synth_tensor", f"blk.{il}.{name}".encode(), typ, nel, SEED, Q.ptr(raw), None)
        if name in ("ffn_gate_exps.weight", "ffn_up_exps.weight"):
            raw = raw[e0 * Q4K_EXPERT:(e0 + n_local) * Q4K_EXPERT].clone()
        elif typ == Q6_K:
            ne = n_local if "_exps." in name else 1
            first = e0 if "_exps." in name else 0
            packed = torch.empty(pb * ne, dtype=torch.uint8, device=dev)
            for e in range(ne):
                Q.call("qma_cuda_repack", Q6_K, raw.data_ptr() + (first + e) * Q6K_EXPERT_GGUF, 2048, 512,
                       packed.data_ptr() + e * pb, None)
            raw = packed
        d[name] = raw
    w = Q.MoeWeights(*[d[k].data_ptr() for k in MOE_TENSORS], Q6_K, Q6_K)
    return w, d


def run_ep_ours(args, world, rank, local):
    """configs[4]'s expert-parallel MoE: the 40 MoE blocks of the random-init
    model, the 256 experts of every layer sharded 256/N over the N GPUs,
    EP_T tokens per GPU per step (one decode step of EP_T sequences; weak
    scaling), every layer's rows and down projections exchanged over NCCL.
    A step runs the 40 blocks in sequence on the same tokens, from the same
    input each step.  The weights of the 40 layers (21 GB / N per GPU) cycle
    through L2 between reuses."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    EP_T = args.tokens
    dev = torch.device("cuda", local)
    e0, n_local = Q.ep_shard(rank, world)
    layers = [ep_layer_weights(il, e0, n_local, dev) for il in range(EP_LAYERS)]
    torch.cuda.synchronize()

    ep = Q.ExpertParallel(local, rank, world, EP_T, ep_share_uid(world))
    x = np.random.default_rng(SEED + rank).standard_normal((EP_T, 2048)).astype(np.float32)
    x0 = torch.from_numpy(x).to(dev)
    buf = [torch.empty_like(x0), torch.empty_like(x0)]
    sel = torch.empty((EP_LAYERS, EP_T, 8), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step(src=None, keep_sel=False):
        buf[0].copy_(x0 if src is None else src, non_blocking=True)
        for il, (w, _) in enumerate(layers):
            ep.moe_layer(w, buf[il & 1], EP_T, buf[(il + 1) & 1], sel[il] if keep_sel else None, None, sp)
        return buf[EP_LAYERS & 1]

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # bytes: the shard's experts that some rank's token selected, per layer
    step(keep_sel=True)
    torch.cuda.synchronize()
    net = [0, 0]
    for il in range(EP_LAYERS):
        ep.moe_layer(layers[il][0], buf[0], EP_T, buf[1], None, None, sp)
        s_, r_, _ = ep.stats()
        net[0] += s_
        net[1] += r_
    all_sel = [sel]
    if world > 1:
        import torch.distributed as dist
        all_sel = [torch.empty_like(sel) for _ in range(world)]
        dist.all_gather(all_sel, sel)
    all_sel = torch.stack(all_sel).cpu().numpy()
    touched = sum(int(np.count_nonzero(np.bincount(all_sel[:, il].ravel(), minlength=256)[e0:e0 + n_local]))
                  for il in range(EP_LAYERS))
    expert_bytes = 2 * Q4K_EXPERT + Q6K_EXPERT_GGUF
    step_bytes = touched * expert_bytes + EP_LAYERS * (expert_bytes + 2048 * 256 * 4 + 2 * 2048 * 4) \
        + EP_LAYERS * 2 * EP_T * 2048 * 4
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        dist_barrier(world)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        dist_barrier(world)
    t_ms = dist_max(sum(e[0].elapsed_time(e[1]) for e in ev), world)
    # end to end: the step's tokens from pinned host memory, its output back
    hx = torch.from_numpy(x).pin_memory()
    hout = torch.empty((EP_T, 2048), dtype=torch.float32).pin_memory()
    e0_, e1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, args.steps // 4)
    dist_barrier(world)
    torch.cuda.synchronize()
    e0_.record(stream)
    for _ in range(e2e_steps):
        dx = hx.to(dev, non_blocking=True)
        hout.copy_(step(dx), non_blocking=True)
    e1_.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist_max(e0_.elapsed_time(e1_), world)
    ep.close()
    peak, peak_kind = load_peaks()
    achieved = step_bytes / (t_ms / args.steps / 1e3) / 1e9
    if rank != 0:
        return
    tok = world * EP_T
    print(json.dumps({
        "metric": EP_METRIC, "value": round(tok * args.steps / (t_ms / 1e3), 1), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4",
        "data": "synthetic",
        "config": {"workload": f"configs[4] expert-parallel MoE: the 40 MoE blocks of the random-init qwen35moe, "
                               f"256 experts sharded 256/{world} per GPU, {EP_T} tokens per GPU per step, "
                               f"NCCL point-to-point dispatch and return; router without the Zipf prior",
                   "parallelism": f"ep{world}", "tokens_per_gpu": EP_T,
                   "l2": "inputs larger than L2 (the 40 layers' weights cycle between reuses)",
                   "base_metric": BASE_METRIC},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "whole EP step on rank 0 (40 layers: touched shard experts, router, shared expert)",
                     "algorithmic_bytes_per_step": step_bytes},
        "nvlink": {"sent_bytes_per_step": net[0], "recv_bytes_per_step": net[1]},
        "e2e": {"value": round(tok * e2e_steps / (e2e_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": EP_T * 2048 * 4, "d2h_bytes_per_step": EP_T * 2048 * 4},
        "gpu_launches": EP_LAUNCHES_PER_LAYER * EP_LAYERS * args.steps, "clocks": clk.summary(),
        "cpu_baseline": None,
    }), flush=True)


# -------------------------------------------------------------------- gdn --
GDN_METRIC = "GDN layer decode us/step (configs[2])"
# algorithmic bytes of one gated-delta-net layer step: the stacked Q4_K
# in-projection (12352 x 2048), ssm_out (2048 x 4096), conv state r+w,
# recurrent state r+w, norms, the input and output vectors
GDN_STEP_BYTES = 12352 * 8 * 144 + 2048 * 16 * 144 + 2 * 8192 * 3 * 4 + 2 * 32 * 128 * 128 * 4 \
    + (2048 + 128 + 4 * 8192 + 64) * 4 + 2 * 2048 * 4


def run_gdn_ours(args, world, rank, local):
    """gated-delta-net layer 0 of the random-init model (Q4_K
    projections, zero state): 1024 single-token steps through
    qma_cuda_gdn_step (device time of each call, CUDA events on the state's
    stream), then a 4096-token prefill in 8 calls of 512 (the chunked
    gated-delta form) on a fresh state."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    dev = torch.device("cuda", local)
    arr, n, size = model_layout(Q8_0)
    model = Q.Model(C.cast(arr, C.POINTER(Q.Tensor)), n, seed=SEED, device=local)
    x = torch.from_numpy(np.random.default_rng(SEED + rank).standard_normal((4096, 2048)).astype(np.float32)).to(dev)
    out = torch.empty_like(x)

    def steps(st, n_steps, per):
        stream = torch.cuda.ExternalStream(Q.lib().qma_cuda_state_stream(st.h), device=local)
        evs = []
        for i in range(n_steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            Q.call("qma_cuda_gdn_step", st.h, 0, Q.ptr(x) + i * per * 8192, per, Q.ptr(out) + i * per * 8192, 1)
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs)

    def decode(st, n_steps):
        """n_steps single-token steps queued back to back (qma_cuda_gdn_decode)."""
        stream = torch.cuda.ExternalStream(Q.lib().qma_cuda_state_stream(st.h), device=local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        Q.call("qma_cuda_gdn_decode", st.h, 0, Q.ptr(x), n_steps, Q.ptr(out))
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    st = Q.State(model, 8192)
    decode(st, 16)                                     # warm-up
    st.close()
    st = Q.State(model, 8192)
    with ClockSampler(local) as clk:
        dist_barrier(world)
        dec_ms = dist_max(decode(st, 1024), world)
        dist_barrier(world)
    st.close()
    st = Q.State(model, 8192)
    pre_ms = dist_max(steps(st, 8, 512), world)
    st.close()
    model.close()
    if rank != 0:
        return
    peak, peak_kind = load_peaks()
    us = dec_ms * 1e3 / 1024
    achieved = GDN_STEP_BYTES / (us * 1e3)
    print(json.dumps({
        "metric": GDN_METRIC, "value": round(us, 3), "unit": "us/step", "n_gpus": world, "steps": 1024,
        "warmup": 16, "ms_per_step": round(dec_ms / 1024, 5), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xq4 projections, fp32 recurrence", "data": "synthetic",
        "config": {"workload": "configs[2] gated-delta-net layer 0: hidden 2048, 16 QK / 32 V heads of 128, "
                               "fp32 state 32x128x128 from zero, conv 4, Q4_K projections; 1024 decode steps, "
                               "then a 4096-token prefill in chunks of 512 (gated-delta chunks of 64)",
                   "per_step": "1024 single-token steps queued back to back by qma_cuda_gdn_decode (per "
                               "step: norm, in-projection + conv, recurrence + gated norm, ssm_out + "
                               "residual, and two 8 KB device copies), device time / 1024",
                   "base_metric": BASE_METRIC},
        "prefill": {"tokens": 4096, "ms": round(pre_ms, 3), "tok_per_s": round(4096 / (pre_ms / 1e3), 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "one decode step of the layer (5 kernels)",
                     "algorithmic_bytes_per_launch": GDN_STEP_BYTES},
        "e2e": {"value": round(us, 3), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 4 * 1024, "clocks": clk.summary(), "cpu_baseline": None,
    }), flush=True)


def run_batch_ours(args, world, rank, local):
    """configs[4] alone: the batched-decode leg of the default line on its
    own model (--prompt sets the prompt length; --steps caps the timed
    steps), printed as its own line."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    arr, n, size = model_layout(Q8_0)
    model = Q.Model(C.cast(arr, C.POINTER(Q.Tensor)), n, seed=SEED, device=local)
    wts = []
    for il in range(40):
        w = Q.MoeWeights()
        Q.call("qma_cuda_model_moe_weights", model.h, il, C.byref(w))
        wts.append(w)
    prompt = args.prompt if args.prompt != PROMPT else BATCH_PROMPT
    with ClockSampler(local) as clk:
        r = run_batch_on_model(model, wts, args, world, rank, local, prompt_len=prompt, check=not args.no_parity,
                               max_steps=args.steps)
    model.close()
    if rank != 0:
        return
    print(json.dumps({
        "metric": r["metric"], "value": r["tok_per_s"], "unit": "tok/s", "n_gpus": world, "steps": r["timed_steps"],
        "warmup": r["decode_tokens_per_sequence"] - r["timed_steps"], "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xq4",
        "data": "synthetic", "config": {"workload": "configs[4] batched decode", **{k: v for k, v in r.items()
                                                                                   if k not in ("metric",)}},
        "clocks": clk.summary(), "e2e": {"value": r["tok_per_s"], "unit": "tok/s",
                                         "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                                         "d2h_bytes_per_step": r["d2h_bytes_per_step"]},
    }), flush=True)
    if not r["parity"]:
        sys.exit("batched decode parity check failed")


def run_prefill_ours(args, world, rank, local):
    """Prefill throughput of the full model: a 1024-token prompt (untimed),
    W warm-up chunks, then K chunks of 512 tokens through qma_cuda_eval
    (last-token logits), timed with CUDA events on the state's stream inside
    an NVTX range "capture"."""
    import ctypes as C
    import torch
    import qma_cuda as Q
    Q.init(local)
    arr, n, size = model_layout(Q8_0)
    model = Q.Model(C.cast(arr, C.POINTER(Q.Tensor)), n, seed=SEED, device=local)
    K, W = max(1, args.steps), args.warmup
    st = Q.State(model, 1024 + 512 * (K + W) + 64)
    stream = torch.cuda.ExternalStream(Q.lib().qma_cuda_state_stream(st.h), device=local)
    rng = np.random.default_rng(SEED + rank)
    st.eval(rng.integers(0, N_VOCAB, 1024).astype(np.int32))
    for _ in range(W):
        st.eval(rng.integers(0, N_VOCAB, 512).astype(np.int32))
    chunks = [rng.integers(0, N_VOCAB, 512).astype(np.int32) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        dist_barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("capture")
        e0.record(stream)
        for c in chunks:
            st.eval(c)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        dist_barrier(world)
    ms = dist_max(e0.elapsed_time(e1), world)
    st.close()
    model.close()
    if rank != 0:
        return
    print(json.dumps({
        "metric": "qwen35moe prefill tok/s (512-token chunks)", "value": round(world * 512 * K / (ms / 1e3), 1),
        "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4", "data": "synthetic",
        "config": {"workload": "full model prefill: 512-token chunks after a 1024-token prompt, one state",
                   "replicas": world},
        "clocks": clk.summary(),
    }), flush=True)


# ------------------------------------------------------------------ main ---
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "moe", "ep", "gdn", "batch",
                                                             "prefill"])
    ap.add_argument("--no-parity", action="store_true", help="batch: skip the in-run parity check")
    ap.add_argument("--tokens", type=int, default=EP_T, help="ep: tokens per GPU per step (1..256)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-ep", action="store_true", help="decode: skip the expert-parallel leg")
    ap.add_argument("--no-gemv", action="store_true", help="decode: skip the configs[1] GEMV leg")
    ap.add_argument("--no-batch", action="store_true", help="decode: skip the configs[4] batched-decode leg")
    ap.add_argument("--rows", type=int, default=GN_OUT, help="gemv: output rows")
    ap.add_argument("--cols", type=int, default=GN_IN, help="gemv: input columns (multiple of 256)")
    ap.add_argument("--prompt", type=int, default=PROMPT,
                    help="decode: prompt tokens prefilled before the timed steps")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            if args.workload == "decode":
                run_decode_reference(args, world, rank)
            else:
                print(json.dumps({"impl": "reference", "unavailable": f"{args.workload} reference arm: use --workload decode"}))
        elif args.workload == "decode":
            run_decode_ours(args, world, rank, local)
        elif args.workload == "moe":
            run_moe_ours(args, world, rank, local)
        elif args.workload == "ep":
            run_ep_ours(args, world, rank, local)
        elif args.workload == "gdn":
            run_gdn_ours(args, world, rank, local)
        elif args.workload == "batch":
            run_batch_ours(args, world, rank, local)
        elif args.workload == "prefill":
            run_prefill_ours(args, world, rank, local)
        else:
            run_gemv_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
