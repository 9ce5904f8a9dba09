#!/usr/bin/env python
"""MoE-layer benchmark on B200 (DeepSeek-V2-Lite shape), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]

The layer: 64 routed experts (gate/up [1408, 2048], down [2048, 1408] bf16), 2 shared
experts, router [64, 2048] f32, softmax top-6, no renormalisation, scaling 1.0, with
weights N(0, 0.02) and activations N(0, 1) rounded to bf16 -- synthetic and seeded,
as no checkpoint exists on the box.  A step is one forward of the layer over a batch
of T tokens already resident in HBM.  L2 is flushed before every timed step, outside
its events (a 256 MiB write, then a 256 MiB read of another buffer), so each step
starts cold and clean and streams its experts from HBM.

One GPU (the default): the headline is the 128-token layer (weights seed 0, tokens
seed 0), HBM-bound.  The same line carries
  sweep      the decode sizes T in {1, 8, 32, 256} (tokens seed 1), HBM GB/s each
  prefill    16384 tokens (seed 2) whose expert load is skewed to Zipf(1.2) by a
             per-expert logit bias: tensor-bound, TFLOP/s against the measured
             dense bf16 burst peak (the launches are milliseconds long)
  ep_base    the expert-parallel per-rank workload (8192 tokens, weights and tokens
             seed 3) on this one GPU: the base of the weak-scaling series
  parity     sampled tokens of the headline batch against the CPU oracle
N > 1 GPUs (torchrun, one rank per GPU): expert parallelism, rank r holding routed
experts [r*64/N, (r+1)*64/N) and the shared experts; every rank forwards 8192 tokens
of its own per step (weights and tokens seed 3; random router, so near-uniform
routing), exchanging token rows and expert outputs with NCCL over NVLink.  Scaling is
weak (tokens per GPU fixed).  Every rank checks sampled tokens against the oracle
and the line reports the worst over ranks.

--impl ours (default): the CUDA path through liblitemind_b200.so.
  value      tokens/s over all ranks, device time from CUDA events per step
  e2e        tokens/s through lm_moe_forward_host from pinned host buffers
             (host->device copy of x, device->host copy of y, inside the timing)
  roofline   the dominant kernel: algorithmic bytes per launch / its mean device
             time, against MEASURED_PEAKS.json
  cpu_baseline  the reference's own CPU code (oracle/_ref, built from the
             reference's sources) on the host's cores, rank 0, N=1 only
--impl reference: the reference CPU path alone (rank 0), same metric and workload,
a bounded sample of the batch per step.

Other workloads: --workload prefill (the 16384-token Zipf batch as the headline),
stack (26 x (RMSNorm, MoE layer, residual) at 4096 tokens, seed 4), ffn (the dense
layer-0 feed-forward), load (the SafeTensors -> HBM loader).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "MoE-layer tokens/s (V2-Lite shape) + % HBM/TC roofline at 1/2/4/8 B200"
SEED_WEIGHTS = 0
SEED_HEADLINE = 0   # the 128-token headline batch
SEED_SWEEP = 1      # the decode sweep's batches
SEED_PREFILL = 2    # the prefill batch and its Zipf logit bias
SEED_EP = 3         # the expert-parallel workload: weights and every rank's tokens
HEADLINE_TOKENS = 128
SWEEP = (1, 8, 32, 256)
PREFILL_TOKENS = 16384
EP_TOKENS = 8192
PARITY_SAMPLES = 8
FLUSH_BYTES = 256 << 20


def kernels_per_forward(tokens: int, world: int, experts: int = 64, top_k: int = 6, sms: int = 148) -> int:
    """Our kernel launches in one forward (NCCL's own kernels not counted).
    One GPU: T <= 256 is the fused decode kernel alone; above that router
    logits, top-k, scan, placement and the two grouped GEMMs, plus a separate row
    gather unless the placement copies the rows itself (2 T >= 32 x SMs).  Expert parallel:
    the routing (fused route kernel for T <= 32, else four kernels), then with the
    fixed-capacity exchange (small batches) pack, sort, device schedule, two GEMMs
    and the combine, or with the host-planned exchange the row gather (when the
    placement does not copy), a sort and two GEMMs per chunk of local experts (plus
    the shared experts' two GEMMs when chunked) and the combine; when copy engines move
    the rows (the default on 2 ranks, LITEMIND_B200_EP_COPY), also one readiness signal
    for the rows and one per chunk, and per peer one wait for its rows and one per chunk."""
    gather = 0 if tokens > 32 and 2 * tokens >= 32 * sms else 1
    if world == 1:
        return 1 if tokens <= 256 else 6 + gather
    route = 1 if tokens <= 32 else 4
    local = experts // world
    fixed = world * tokens * min(top_k, local) <= 8192
    if fixed:
        return route + 6
    # Host-planned: per chunk of local experts a sort and two GEMMs; with more than one
    # chunk the shared experts get GEMMs of their own.
    chunks = max(1, min(int(os.environ.get("LITEMIND_B200_EP_CHUNKS", "2")), 8, local))
    copy_env = os.environ.get("LITEMIND_B200_EP_COPY")
    copy = world == 2 if copy_env is None else (int(copy_env) != 0 and world <= 8)
    signals = (1 + chunks + (world - 1) * (1 + chunks)) if copy else 0
    return route + gather + 3 * chunks + (2 if chunks > 1 else 0) + 1 + signals


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per rank per step (default: 128 on one GPU, 8192 per rank on several; 16384 "
                         "for prefill, 4096 for stack)")
    ap.add_argument("--workload", choices=["decode", "prefill", "stack", "ffn", "load"], default="decode",
                    help="decode: one MoE layer (the headline; expert parallel on several GPUs); prefill: one "
                         "layer at 16384 tokens with Zipf expert load (tensor-bound); stack: 26 x (RMSNorm, "
                         "MoE, residual); ffn: the dense layer-0 feed-forward; load: the SafeTensors -> HBM "
                         "loader")
    ap.add_argument("--layers", type=int, default=26, help="blocks in the stack workload")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill object of the one-GPU line")
    ap.add_argument("--no-ep-base", action="store_true", help="skip the one-GPU expert-parallel base")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--clock-window", type=float, default=1.5,
                    help="seconds of the forward loop run under the clock sampler before the timed steps")
    return ap.parse_args(argv)


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def committed_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu capture."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(workload)


# ── clocks ────────────────────────────────────────────────────────────────

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int, interval_ms: int = 200):
        self.device = device
        self.interval_ms = interval_ms
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.device), "-lms", str(self.interval_ms)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxes.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms),
                "window": f"nvidia-smi every {self.interval_ms} ms over the load window that ends with the timed "
                          "steps"}


# ── algorithmic work ──────────────────────────────────────────────────────

def layer_bytes(shape, touched_experts: int, T: int) -> int:
    """Algorithmic HBM bytes of one layer forward: touched experts, shared experts,
    router, x in (bf16), y out (f32)."""
    return (shape.expert_bytes * touched_experts + shape.shared_bytes + shape.router_bytes
            + T * shape.hidden * (2 + 4))


def layer_flops(shape, T: int) -> int:
    """Algorithmic FLOPs of one layer forward: router, top-k experts and shared experts."""
    per_token = 2 * shape.n_routed_experts * shape.hidden + 3 * 2 * shape.inter * shape.hidden * (
        shape.top_k + shape.n_shared_experts)
    return per_token * T


def gate_up_flops(shape, T: int) -> int:
    """Algorithmic FLOPs of one gate/up GEMM launch (gate and up rows of the top-k and shared experts)."""
    return 2 * (2 * shape.inter) * shape.hidden * (shape.top_k + shape.n_shared_experts) * T


def gate_up_bytes(shape, touched_experts: int, T: int) -> int:
    """Algorithmic bytes of one gate/up GEMM launch: gate and up of every touched
    expert and of the shared experts, plus the token activations."""
    return (2 * shape.inter * shape.hidden * 2) * (touched_experts + shape.n_shared_experts) + T * shape.hidden * 2


# ── reference CPU path ────────────────────────────────────────────────────

def cpu_reference_rate(weights, x_f32, seconds: float, min_reps: int = 1, max_reps: int = 1000, bias=None):
    """tokens/s of the reference's own MoE block (oracle/_ref) on all host threads."""
    from oracle.oracle import Reference, RouterConfig

    ref = Reference()
    threads = ref.hardware_threads()
    cfg = RouterConfig()
    T = x_f32.shape[0]
    ref.moe_layer(x_f32[:1], weights, cfg, 2, bias=bias, threads=threads)  # warm the pool, page in the weights
    reps, t0 = 0, time.perf_counter()
    while reps < min_reps or (time.perf_counter() - t0 < seconds and reps < max_reps):
        ref.moe_layer(x_f32, weights, cfg, 2, bias=bias, threads=threads)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": T * reps / dt, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{reps} x {T}-token batches of the same workload, {dt:.1f} s, reference "
                      f"gemm::/MoeRouter built from its sources ({ref.kernel_description()})"}


def run_reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    from litemind_b200 import synthetic as syn

    if args.workload == "load":
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no device loader (its WeightStore "
                                                              "maps shards and pages weights in on first touch)"}))
        return
    if args.workload == "ffn":
        g, u, d = dense_weights()
        xf = syn.bf16_to_f32(syn.tokens(syn.V2_LITE, args.tokens, seed=SEED_DENSE)).reshape(args.tokens, -1)
        per_step = max(args.cpu_seconds / max(args.steps, 1), 0.5)
        rates = [cpu_dense_rate(g, u, d, xf, per_step) for _ in range(args.steps)]
        value = statistics.median(r["value"] for r in rates)
        print(json.dumps({
            "impl": "reference", "metric": "dense feed-forward tokens/s (V2-Lite layer 0 shape)", "value": value,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * args.tokens / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "dense-ffn: DeepSeek-V2-Lite layer 0 feed-forward (hidden 2048, inter 10944)",
                       "tokens_per_rank": args.tokens},
            "cpu_baseline": {**rates[-1], "value": value},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    wl = layer_workload(args, world)
    W = syn.layer_weights(syn.V2_LITE, seed=wl["seed_weights"])
    # Each step is a bounded sample of the batch: the reference runs a token at a time.
    n = min(args.tokens, 128)
    x = syn.bf16_to_f32(syn.tokens(syn.V2_LITE, args.tokens, seed=wl["seed_tokens"]))
    x = x.reshape(args.tokens, -1)[:n]
    bias = syn.zipf_bias(syn.V2_LITE, seed=SEED_PREFILL) if wl["bias"] else None
    from oracle.oracle import Reference, RouterConfig

    ref = Reference()
    threads = ref.hardware_threads()
    for _ in range(max(args.warmup, 0)):
        ref.moe_layer(x[:1], W, RouterConfig(), 2, bias=bias, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.moe_layer(x, W, RouterConfig(), 2, bias=bias, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = n / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": wl["config"],
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"{args.steps} steps of the first {n} tokens of the {args.tokens}-token batch "
                                   f"on rank 0's host, one host for all {world} rank(s) "
                                   f"({ref.kernel_description()})"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def layer_workload(args, world: int) -> dict:
    """Seeds, bias and description of the layer workload both arms run."""
    if args.workload == "prefill":
        sw, st, bias = SEED_WEIGHTS, SEED_PREFILL, True
        name = "prefill: V2-Lite MoE layer, Zipf(1.2) expert load from a per-expert logit bias"
    elif world > 1:
        sw, st, bias = SEED_EP, SEED_EP, False
        name = ("expert-parallel: V2-Lite MoE layer, 64/N routed experts per GPU, NCCL all-to-all dispatch and "
                "return, random router (near-uniform routing)")
    else:
        sw, st, bias = SEED_WEIGHTS, (SEED_HEADLINE if args.tokens == HEADLINE_TOKENS else SEED_SWEEP), False
        name = "moe-layer: V2-Lite MoE layer on one GPU, HBM-bound batch"
    config = {"workload": name, "tokens_per_rank": args.tokens, "global_tokens": args.tokens * world,
              "seed_weights": sw, "seed_tokens": st,
              "experts": "64 routed top-6 + 2 shared, hidden 2048, inter 1408",
              "l2": "flushed before every timed step (256 MiB write, then 256 MiB read of a second buffer: cold, "
                    "clean L2), outside the step's events",
              "parallelism": "single GPU" if world == 1 else
              f"expert parallel: {64 // world} routed experts per GPU, NCCL all-to-all dispatch/combine"}
    if world > 1:
        config["tokens_seed_stream"] = "rank"
    return {"seed_weights": sw, "seed_tokens": st, "bias": bias, "config": config}


# ── our arm ───────────────────────────────────────────────────────────────

class L2Flush:
    """Evicts L2 between steps: writes one buffer larger than L2, then reads another,
    so the next step starts from a cold L2 that holds no dirty lines."""

    def __init__(self, torch, nbytes: int = FLUSH_BYTES):
        self.w = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        self.r = torch.zeros(nbytes // 8, dtype=torch.int64, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.r.sum()


def device_sms(torch) -> int:
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def stack_kernels_per_layer(tokens: int, world: int, sms: int = 148) -> int:
    """One block: the RMSNorm, then the layer's own launches; the router reads f32
    activations, so at >= 2048 tokens its logits take the split tiled kernel plus its
    reduction instead of one launch."""
    if world == 1 and tokens <= 128:
        return 1 + 1
    return 1 + kernels_per_forward(tokens, world, sms=sms) + (1 if tokens >= 2048 else 0)


def run_stack(args, rank: int, world: int, local_rank: int) -> int:
    """The layer stack: `layers` x (RMSNorm -> MoE -> residual) over T tokens per rank."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from litemind_b200 import synthetic as syn
    from litemind_b200.moe import MoeConfig, MoeLayer

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    shape, T, L = syn.V2_LITE, args.tokens, args.layers
    layer = MoeLayer(MoeConfig(num_layers=L, max_tokens=T), device=local_rank)
    if world > 1:
        uid = [MoeLayer.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        layer.ep_init(uid[0], rank, world)
    ones = np.ones(shape.hidden, np.float32)  # RMSNorm weights: ones, as tools/make_test_model.py writes them
    t_up = time.perf_counter()
    for l in range(L):
        layer.upload_layer(l, syn.layer_weights(shape, seed=4, layer=l), norm_weight=ones)
    upload_s = time.perf_counter() - t_up
    x0 = torch.from_numpy(syn.bf16_to_f32(syn.tokens(shape, T, seed=4, stream=rank)).reshape(T, -1)).cuda()
    hidden = x0.clone()
    flush = L2Flush(torch)

    def step():
        hidden.copy_(x0)
        for l in range(L):
            layer.block_forward(l, hidden)

    for _ in range(max(args.warmup, 3)):
        step()
    layer.sync()
    clocks = ClockSampler(local_rank)
    clocks.start()
    t_load = time.perf_counter()
    while load_window_open(t_load, args.clock_window, world, torch):
        step()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total = 0.0
    for _ in range(args.steps):
        flush()
        start.record()
        step()
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    clock_info = clocks.stop()
    ms = total / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    peaks = measured_peaks()
    flops = 138_674_176 * T * L * world
    hbm = (shape.expert_bytes * shape.n_routed_experts + shape.shared_bytes + shape.router_bytes) * L
    line = {
        "metric": METRIC, "value": T * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config4-stack: {L} x (RMSNorm, V2-Lite MoE layer, residual)", "tokens_per_rank": T,
                   "layers": L, "seed": 4, "norm_weights": "ones", "resident_weight_gb": hbm / 1e9 / world,
                   "upload_s": upload_s,
                   "parallelism": "single GPU" if world == 1 else f"expert parallel, {64 // world} experts per GPU"},
        # Timed inside seconds of back-to-back steps under the 1 kW cap: the sustained
        # GEMM figure is the denominator (the burst one is reported beside it).
        "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12 / world,
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": flops / (ms / 1e3) / 1e12 / world / peaks["bf16_tflops_sustained"],
                     "frac_of_burst": flops / (ms / 1e3) / 1e12 / world / peaks["bf16_tflops"],
                     "peak_source": f"{peaks['source']} (bf16_tflops_sustained)",
                     "hbm_frac": hbm / world / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], "traffic": None},
        "clocks": clock_info,
        "gpu_launches": stack_kernels_per_layer(T, world, device_sms(torch)) * L * args.steps,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


DENSE_INTER = 10944  # DeepSeek-V2-Lite's dense layer 0 (include/Config.hpp:59)
SEED_DENSE = 5


def dense_weights(seed: int = SEED_DENSE):
    from litemind_b200 import synthetic as syn

    H, I = syn.V2_LITE.hidden, DENSE_INTER
    return (syn.normal_bf16(seed, (0,), (I, H), 0.02), syn.normal_bf16(seed, (1,), (I, H), 0.02),
            syn.normal_bf16(seed, (2,), (H, I), 0.02))


def cpu_dense_rate(g, u, d, x_f32, seconds: float) -> dict:
    """tokens/s of the reference's dense feed-forward (Impl::feed_forward,
    src/DeepSeekRunner.cpp:228-240: gemm::matvec_bf16 gate and up, silu_multiply,
    matvec_bf16_accumulate down) on all host threads, one token at a time as the
    reference runs it."""
    import numpy as np

    from oracle.oracle import Reference

    ref = Reference()
    ref.threads = ref.hardware_threads()
    out = np.zeros(g.shape[1], np.float32)

    def one(x):
        h = ref.silu_multiply(ref.matvec_bf16(g, x), ref.matvec_bf16(u, x))
        ref.matvec_bf16_accumulate(d, h, out, 1.0)

    one(x_f32[0])  # page the weights in, start the pool
    n, t0 = 0, time.perf_counter()
    while n < 1 or time.perf_counter() - t0 < seconds:
        one(x_f32[n % x_f32.shape[0]])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
            "sample": f"{n} tokens one at a time, {dt:.1f} s, reference gemm:: built from its sources"}


def run_ffn(args, rank: int, world: int, local_rank: int) -> int:
    """The dense feed-forward (DeepSeek-V2-Lite layer 0, intermediate 10944) through
    lm_ffn_forward: gate/up with the SiLU epilogue, then down, on the grouped tcgen05
    GEMMs with one all-token segment.  With N > 1 every GPU runs its own replica
    (the dense layer is not sharded)."""
    import numpy as np

    import torch

    from litemind_b200 import synthetic as syn
    from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor

    torch.cuda.set_device(local_rank)
    H, I, T = syn.V2_LITE.hidden, DENSE_INTER, args.tokens
    g, u, d = dense_weights()
    layer = MoeLayer(MoeConfig(max_tokens=T), device=local_rank)
    layer.ffn_upload(0, g, u, d)
    x_bits = syn.tokens(syn.V2_LITE, T, seed=SEED_DENSE, stream=rank)
    x = bf16_tensor(x_bits)
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    flush = L2Flush(torch)
    for _ in range(max(args.warmup, 3)):
        layer.ffn_forward(0, x, y=y)
    layer.sync()
    clocks = ClockSampler(local_rank)
    clocks.start()
    t_load = time.perf_counter()
    while time.perf_counter() - t_load < args.clock_window:
        for _ in range(20):
            flush()
            layer.ffn_forward(0, x, y=y)
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total = 0.0
    for _ in range(args.steps):
        flush()
        start.record()
        layer.ffn_forward(0, x, y=y)
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    clock_info = clocks.stop()
    ms = total / args.steps
    # Per-kernel device times of the same steps.
    layer.profile(True)
    layer.profile_read(reset=True)
    for _ in range(args.steps):
        flush()
        layer.ffn_forward(0, x, y=y)
    prof = layer.profile_read(reset=True)
    layer.profile(False)
    # End to end: pinned host x in, y out, copies inside the timing.
    x_host = torch.from_numpy(x_bits.view(np.int16)).pin_memory()
    y_host = torch.empty((T, H), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((T, H), dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x_dev.copy_(x_host, non_blocking=True)
        layer.ffn_forward(0, x_dev.view(torch.bfloat16), y=y)
        y_host.copy_(y, non_blocking=True)
        torch.cuda.synchronize()
    e2e_ms = 1e3 * (time.perf_counter() - t0) / args.steps
    peaks = measured_peaks()
    weight_bytes = 3 * I * H * 2
    bytes_step = weight_bytes + T * H * (2 + 4)
    flops = 6 * I * H * T
    hbm_bound = flops / bytes_step < peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    gu_ms, gu_n = prof.get("gemm_gate_up", (0.0, 0))
    gu_avg = gu_ms / max(gu_n, 1)
    gu_bytes, gu_flops = 2 * I * H * 2 + T * H * 2 + T * I * 2, 4 * I * H * T
    if hbm_bound:
        k_achieved = gu_bytes / (gu_avg / 1e3) / 1e9 if gu_avg else 0.0
        roofline = {"bound": "hbm", "achieved": k_achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": k_achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} (hbm_gbs)",
                    "layer_achieved": bytes_step / (ms / 1e3) / 1e9,
                    "layer_frac": bytes_step / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
    else:
        k_achieved = gu_flops / (gu_avg / 1e3) / 1e12 if gu_avg else 0.0
        roofline = {"bound": "tensor", "achieved": k_achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": k_achieved / peaks["bf16_tflops"], "peak_source": f"{peaks['source']} (bf16_tflops)",
                    "layer_achieved": flops / (ms / 1e3) / 1e12,
                    "layer_frac": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"]}
    total_prof = sum(v[0] for v in prof.values())
    roofline.update({"kernel": "gemm_gate_up (tcgen05 grouped GEMM, one all-token segment, SiLU epilogue)",
                     "bytes_per_launch": gu_bytes, "flops_per_launch": gu_flops, "mean_launch_ms": gu_avg,
                     "traffic": None,
                     "share_of_step": {k: round(v[0] / total_prof, 4) for k, v in prof.items()} if total_prof else {}})
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        xf = syn.bf16_to_f32(x_bits).reshape(T, H)
        cpu = cpu_dense_rate(g, u, d, xf, args.cpu_seconds)
    line = {
        "metric": "dense feed-forward tokens/s (V2-Lite layer 0 shape)", "value": T * world / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "dense-ffn: DeepSeek-V2-Lite layer 0 feed-forward (hidden 2048, inter 10944)",
                   "tokens_per_rank": T, "seed": SEED_DENSE, "weights": "N(0, 0.02) bf16",
                   "l2": "flushed before every timed step (weights 134.5 MB also exceed L2)",
                   "parallelism": "single GPU" if world == 1 else "replicas (the dense layer is not sharded)"},
        "roofline": roofline, "cpu_baseline": cpu,
        "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4,
                "how": "pinned host x copied in, lm_ffn_forward, y copied out, synchronised, wall clock per step"},
        "clocks": clock_info, "gpu_launches": 3 * args.steps,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    layer.close()
    return 0


def run_load(args, rank: int, world: int, local_rank: int) -> int:
    """The SafeTensors -> HBM loader: one V2-Lite MoE layer (64 experts, shared experts,
    router, norm; DeepSeek tensor names) written to a shard in a temporary directory,
    then lm_moe_load_safetensors (mmap, header parse, name lookup, bf16 repack into the
    tile-major GEMM layout, host -> device copies) timed per call.  The shard was just
    written, so it is read from the page cache: this measures the loader, not the disk."""
    import numpy as np

    import shutil

    import torch

    from litemind_b200 import synthetic as syn
    from litemind_b200.checkpoint import layer_tensors, write_safetensors
    from litemind_b200.moe import MoeConfig, MoeLayer

    torch.cuda.set_device(local_rank)
    shape = syn.V2_LITE
    W = syn.layer_weights(shape, seed=SEED_WEIGHTS)
    tensors = layer_tensors(W, 0, shape.n_shared_experts)
    nbytes = sum(np.asarray(a).nbytes for _, a in tensors.values())
    tmp = tempfile.mkdtemp(prefix="lm_load_")
    try:
        path = os.path.join(tmp, "model-00001-of-00001.safetensors")
        write_safetensors(path, tensors)
        del tensors
        layer = MoeLayer(MoeConfig(max_tokens=32), device=local_rank)
        for _ in range(max(args.warmup, 1)):
            layer.load_safetensors(0, [path], checkpoint_layer=0)
        layer.sync()
        times = []
        for _ in range(args.steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            layer.load_safetensors(0, [path], checkpoint_layer=0)
            layer.sync()
            times.append(time.perf_counter() - t0)
        # The copy bound: a plain pinned host -> device copy of the same size.
        src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        dst.copy_(src)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        h2d = 3 * nbytes / (time.perf_counter() - t0) / 1e9
        layer.close()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    sec = statistics.median(times)
    gbs = nbytes / sec / 1e9
    line = {
        "metric": "SafeTensors -> HBM load GB/s (one V2-Lite MoE layer)", "value": gbs, "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "load: lm_moe_load_safetensors of one layer from a fresh shard in the page cache",
                   "tensor_bytes": nbytes, "tensors": 3 * shape.n_routed_experts + 6,
                   "parallelism": "single GPU"},
        "roofline": {"bound": "h2d", "achieved": gbs, "peak": h2d, "unit": "GB/s", "frac": gbs / h2d,
                     "peak_source": "pinned host -> device copy of the same bytes, measured in this run",
                     "traffic": None},
        "cpu_baseline": None,
        "cpu_baseline_note": "the reference has no device loader: WeightStore maps the shard and the CPU kernels "
                             "page weights in as they touch them",
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def sampled_parity(y, x_bits, W, rows, bias=None) -> dict:
    """Output parity of sampled tokens, checked after the timed region by the test
    suite's oracle checker (tests/parity.py)."""
    from tests.parity import sampled_oracle_parity

    return sampled_oracle_parity(y, x_bits, W, rows, bias=bias)


def kernel_roofline(prof: dict, ms_per_step: float, layer_b: int, gate_up_b: int, peaks: dict) -> dict:
    """The dominant kernel's roofline from the profiled per-launch device times.  A
    one-launch step is timed by the step's own events (the kernel is the step); a
    kernel of a several-launch step by its profiling events, capped at the step time."""
    total = sum(v[0] for v in prof.values())
    share = {k: round(v[0] / total, 4) for k, v in prof.items()} if total else {}
    if "decode_fused" in prof:
        k_bytes, name, mean = layer_b, ("moe_decode_kernel (fused routing, gathers, tcgen05 gate/up and down, "
                                        "weighted combine: the whole layer in one cooperative launch)"), ms_per_step
        how = "one launch per step: the step's CUDA events time the kernel"
    else:
        ms, n = prof.get("gemm_gate_up", (0.0, 0))
        k_bytes, name = gate_up_b, "gemm_gate_up (tcgen05 grouped GEMM, gate/up + SiLU epilogue)"
        mean = min(ms / max(n, 1), ms_per_step)
        how = "profiling events around the launch in the same steps, capped at the step time"
    achieved = k_bytes / (mean / 1e3) / 1e9 if mean > 0 else 0.0
    return {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} (hbm_gbs)",
            "bytes_per_launch": k_bytes, "mean_launch_ms": mean, "timing": how, "share_of_step": share}


# The fused kernel's per-CTA phase stamps (lm_moe_profile_trace), in kernel order.
TRACE_PHASES = ((0, "start"), (1, "logits_written"), (2, "logits_seen"), (10, "logits_in_smem"),
                (9, "topk_written"), (13, "topk_seen"), (11, "routed"), (12, "experts_scanned"),
                (3, "schedule_built"), (14, "rows_gathered"), (15, "producer_saw_rows"), (4, "gate_up_done"),
                (5, "producer_saw_h"), (6, "producer_done"), (8, "mma_done"), (7, "down_done"))


def phase_trace(layer, x, y, flush, torch, bias=None) -> dict | None:
    """One profiled forward of the fused kernel: per phase, the [min, median, max] over
    CTAs of its stamp in microseconds from the earliest CTA start (L2 flushed first)."""
    import numpy as np

    layer.profile(True)
    layer.profile_read(reset=True)
    flush()
    layer.forward(0, x, y=y, bias=bias)
    prof = layer.profile_read(reset=True)
    tr = layer.profile_trace().astype(np.int64) if "decode_fused" in prof else None
    layer.profile(False)
    layer.sync()
    if tr is None or tr.size == 0:
        return None
    t0 = tr[:, 0].min()
    out = {}
    for slot, name in TRACE_PHASES:
        col = tr[:, slot]
        if (col > 0).any():
            v = (col[col > 0] - t0) / 1000.0
            out[name] = [round(float(v.min()), 1), round(float(np.median(v)), 1), round(float(v.max()), 1)]
    return out


def load_window_open(t0: float, window: float, world: int, torch) -> bool:
    """True while the clock-sampling load window is open.  Under torchrun every forward is
    collective, so all ranks must run the same number of them: the ranks agree on the
    minimum of their votes instead of each reading its own clock."""
    go = time.perf_counter() - t0 < window
    if world > 1:
        import torch.distributed as dist

        device = "cuda" if dist.get_backend() == "nccl" else "cpu"
        vote = torch.tensor([1 if go else 0], dtype=torch.int32, device=device)
        dist.all_reduce(vote, op=dist.ReduceOp.MIN)
        go = bool(vote.item())
    return go


def time_steps(layer, x, y, flush, steps, torch, bias=None, slot=0):
    """Per-step CUDA-event time (ms) of layer.forward on layer slot `slot`, L2 flushed before each."""
    total = 0.0
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    for _ in range(steps):
        flush()
        start.record()
        layer.forward(slot, x, y=y, bias=bias)
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return total / steps


def measure_prefill(layer, W, flush, args, torch, peaks) -> dict:
    """The 16384-token Zipf(1.2) batch on one GPU: tensor-bound, against the burst peak."""
    import numpy as np

    from litemind_b200 import synthetic as syn
    from litemind_b200.moe import bf16_tensor

    shape, T = syn.V2_LITE, PREFILL_TOKENS
    x_bits = syn.tokens(shape, T, seed=SEED_PREFILL)
    x = bf16_tensor(x_bits)
    bias_np = syn.zipf_bias(shape, seed=SEED_PREFILL)
    bias = torch.from_numpy(bias_np).cuda()
    y = torch.empty((T, shape.hidden), dtype=torch.float32, device="cuda")
    for _ in range(max(args.warmup, 3)):
        layer.forward(0, x, y=y, bias=bias)
    layer.sync()
    dev = torch.cuda.current_device()
    # Burst: the steps right after the warm-up, as the dense bf16 peak's burst figure is
    # measured (a few milliseconds-long GEMMs); clocks sampled every 50 ms meanwhile.
    burst_clocks = ClockSampler(dev, interval_ms=50)
    burst_clocks.start()
    time.sleep(0.1)
    ms = time_steps(layer, x, y, flush, max(args.steps, 20), torch, bias=bias)
    burst_clock_info = burst_clocks.stop()
    # Per-kernel device times in the same regime (a few steps, profiling events).
    layer.profile(True)
    layer.profile_read(reset=True)
    for _ in range(5):
        flush()
        layer.forward(0, x, y=y, bias=bias)
    prof = layer.profile_read(reset=True)
    layer.profile(False)
    # Sustained: the same steps after seconds of back-to-back load (power-capped clocks).
    clocks = ClockSampler(dev)
    clocks.start()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < args.clock_window:
        for _ in range(2):
            flush()
            layer.forward(0, x, y=y, bias=bias)
        torch.cuda.synchronize()
    ms_sustained = time_steps(layer, x, y, flush, args.steps, torch, bias=bias)
    clock_info = clocks.stop()
    counts = [int(v) for v in layer.expert_counts()]
    lf = layer_flops(shape, T)
    gu_f = gate_up_flops(shape, T)
    gu_ms, gu_n = prof.get("gemm_gate_up", (0.0, 0))
    gu_avg = min(gu_ms / max(gu_n, 1), ms)
    dn_ms, dn_n = prof.get("gemm_down", (0.0, 0))
    dn_avg = min(dn_ms / max(dn_n, 1), ms)
    dn_f = 2 * shape.hidden * shape.inter * (shape.top_k + shape.n_shared_experts) * T
    total = sum(v[0] for v in prof.values())
    burst, sus = peaks["bf16_tflops"], peaks["bf16_tflops_sustained"]
    layer_tf = lf / (ms / 1e3) / 1e12
    sus_tf = lf / (ms_sustained / 1e3) / 1e12
    out = {
        "tokens": T, "seed_tokens": SEED_PREFILL, "seed_weights": SEED_WEIGHTS,
        "expert_load": "Zipf(1.2) from a per-expert logit bias b_e = -1.2 ln(rank_e) over a seeded permutation",
        "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
        "timing": "burst: the steps right after a 3-step warm-up (L2 flushed before each), as the burst bf16 "
                  "peak is measured; clocks sampled every 50 ms",
        "roofline": {"bound": "tensor", "achieved": layer_tf, "peak": burst, "unit": "TFLOP/s",
                     "frac": layer_tf / burst, "peak_source": f"{peaks['source']} (bf16_tflops, burst)",
                     "flops_per_step": lf},
        "burst_clocks": burst_clock_info,
        "sustained": {"ms_per_step": ms_sustained, "tokens_per_s": T / (ms_sustained / 1e3), "achieved": sus_tf,
                      "peak": sus, "frac": sus_tf / sus,
                      "peak_source": f"{peaks['source']} (bf16_tflops_sustained)",
                      "timing": f"after {args.clock_window} s of back-to-back steps (1 kW power cap)"},
        "kernels": {
            "gemm_gate_up": {"mean_ms": gu_avg, "tflops": gu_f / (gu_avg / 1e3) / 1e12 if gu_avg else 0.0,
                             "frac": gu_f / (gu_avg / 1e3) / 1e12 / burst if gu_avg else 0.0},
            "gemm_down": {"mean_ms": dn_avg, "tflops": dn_f / (dn_avg / 1e3) / 1e12 if dn_avg else 0.0,
                          "frac": dn_f / (dn_avg / 1e3) / 1e12 / burst if dn_avg else 0.0},
            "share_of_step": {k: round(v[0] / total, 4) for k, v in prof.items()} if total else {}},
        "expert_rows": counts, "clocks": clock_info,
        "kernel_timing": "profiling events around each launch in 5 steps right after the burst steps",
        "gpu_launches_per_step": kernels_per_forward(T, 1),
    }
    if not args.no_parity:
        rows = np.linspace(0, T - 1, PARITY_SAMPLES).astype(int)
        out["parity"] = sampled_parity(y.cpu().numpy(), x_bits, W, rows, bias=bias_np)
    return out


def measure_ep_base(layer, flush, args, torch) -> dict:
    """The expert-parallel per-rank workload (8192 tokens, seed 3) on this one GPU:
    what each rank of the N-GPU runs computes, with every expert local."""
    from litemind_b200 import synthetic as syn
    from litemind_b200.moe import bf16_tensor

    shape, T = syn.V2_LITE, EP_TOKENS
    x = bf16_tensor(syn.tokens(shape, T, seed=SEED_EP, stream=0))
    y = torch.empty((T, shape.hidden), dtype=torch.float32, device="cuda")
    for _ in range(3):
        layer.forward(1, x, y=y)
    layer.sync()
    ms = time_steps(layer, x, y, flush, max(5, args.steps // 2), torch, slot=1)
    # Sustained: after the same load window the N-GPU runs take before their timed steps
    # (power-capped clocks), the like-for-like base for them.
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < args.clock_window:
        for _ in range(2):
            flush()
            layer.forward(1, x, y=y)
        torch.cuda.synchronize()
    ms_sus = time_steps(layer, x, y, flush, max(5, args.steps // 2), torch, slot=1)
    clock_info = clocks.stop()
    return {"tokens": T, "seed": SEED_EP, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
            "timing": "burst: the steps right after a 3-step warm-up",
            "sustained": {"ms_per_step": ms_sus, "tokens_per_s": T / (ms_sus / 1e3), "clocks": clock_info,
                          "timing": f"after {args.clock_window} s of back-to-back steps, as the N-GPU lines are "
                                    "timed"},
            "note": "the expert-parallel runs' per-rank workload on one GPU (weights and rank-0 tokens of seed 3): "
                    "the base of the weak-scaling series (compare the N-GPU lines with `sustained`)"}


def main(argv=None) -> int:
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.tokens is None:
        args.tokens = {"decode": HEADLINE_TOKENS if world == 1 else EP_TOKENS, "prefill": PREFILL_TOKENS,
                       "stack": 4096, "ffn": 32, "load": 32}[args.workload]
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return 0
    if args.workload == "stack":
        return run_stack(args, rank, world, local_rank)
    if args.workload == "ffn":
        return run_ffn(args, rank, world, local_rank)
    if args.workload == "load":
        return run_load(args, rank, world, local_rank)
    return run_layer(args, rank, world, local_rank)


def run_layer(args, rank: int, world: int, local_rank: int) -> int:
    import numpy as np
    import torch
    import torch.distributed as dist

    from litemind_b200 import synthetic as syn
    from litemind_b200.moe import MoeConfig, MoeLayer, bf16_tensor

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    shape = syn.V2_LITE
    T = args.tokens
    wl = layer_workload(args, world)
    prefill = args.workload == "prefill"
    extras = world == 1 and not prefill  # sweep, prefill and ep_base ride on the one-GPU headline line
    W = syn.layer_weights(shape, seed=wl["seed_weights"])
    max_tokens = max([T] + (list(SWEEP) if extras and not args.no_sweep else [])
                     + ([PREFILL_TOKENS] if extras and not args.no_prefill else [])
                     + ([EP_TOKENS] if extras and not args.no_ep_base else []))
    n_slots = 2 if extras and not args.no_ep_base else 1
    layer = MoeLayer(MoeConfig(max_tokens=max_tokens, num_layers=n_slots), device=local_rank)
    if world > 1:
        uid = [MoeLayer.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        layer.ep_init(uid[0], rank, world)
    layer.upload_layer(0, W)
    x_bits = syn.tokens(shape, T, seed=wl["seed_tokens"], stream=rank)
    x = bf16_tensor(x_bits)
    bias_np = syn.zipf_bias(shape, seed=SEED_PREFILL) if wl["bias"] else None
    bias = torch.from_numpy(bias_np).cuda() if wl["bias"] else None
    y = torch.empty((T, shape.hidden), dtype=torch.float32, device="cuda")
    flush = L2Flush(torch)

    for _ in range(max(args.warmup, 3)):
        layer.forward(0, x, y=y, bias=bias)
    layer.sync()
    # Experts whose weights this GPU streams: the touched ones on one GPU; with
    # expert parallelism every local expert (all are hit at >= 32 tokens per rank).
    touched = int((layer.expert_counts() > 0).sum()) if world == 1 else shape.n_routed_experts // world

    # nvidia-smi samples every 200 ms and the timed steps take milliseconds, so the
    # sampler runs through a load window of the same forward loop that ends with
    # the timed region.
    clocks = ClockSampler(local_rank)
    clocks.start()
    t_load = time.perf_counter()
    while load_window_open(t_load, args.clock_window, world, torch):
        for _ in range(20 if T <= 1024 else 2):
            flush()
            layer.forward(0, x, y=y, bias=bias)
        torch.cuda.synchronize()

    # ── timed region: K steps, barrier + synchronize on both sides ──
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    ms = time_steps(layer, x, y, flush, args.steps, torch, bias=bias)
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    clock_info = clocks.stop()
    layer.sync()
    ms = max_over_ranks(ms)
    value = T * world / (ms / 1e3)
    y_host = y.cpu().numpy()

    # ── per-launch device times for the roofline (same workload, instrumented) ──
    layer.profile(True)
    layer.profile_read(reset=True)
    for _ in range(args.steps):
        flush()
        layer.forward(0, x, y=y, bias=bias)
    prof = layer.profile_read(reset=True)
    ep_timeline = layer.profile_ep_timeline() if world > 1 else None
    layer.profile(False)
    peaks = measured_peaks()
    lb = layer_bytes(shape, touched, T)
    roofline = kernel_roofline(prof, ms, lb, gate_up_bytes(shape, touched, T), peaks)
    roofline["traffic"] = committed_traffic(("decode_fused_T" if "decode_fused" in prof else "gemm_gate_up_T")
                                            + str(T))
    if ep_timeline is not None:
        roofline["ep_timeline_ms"] = ep_timeline
        roofline["note"] = ("chunked exchange: the gemm_gate_up slot spans the shared experts' and every chunk's "
                            "GEMMs, overlapped with the NCCL dispatch and return of other chunks")
    layer_roofline = {"bytes": lb, "achieved": lb / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": lb / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], "touched_experts": touched}
    if "decode_fused" in prof and world == 1:
        roofline["phase_trace_us"] = phase_trace(layer, x, y, flush, torch, bias=bias)
    if prefill or world > 1:
        # Tensor-bound batches: FLOPs against the dense bf16 burst peak (the launches
        # are milliseconds long), the sustained figure beside it.
        lf = layer_flops(shape, T)
        tf = lf / (ms / 1e3) / 1e12
        layer_roofline = {"flops": lf, "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                          "frac": tf / peaks["bf16_tflops"], "peak_source": f"{peaks['source']} (bf16_tflops, burst)",
                          "frac_of_sustained": tf / peaks["bf16_tflops_sustained"], "hbm_bytes": lb}
        if prefill:
            layer_roofline["expert_rows"] = [int(v) for v in layer.expert_counts()]
            gu_ms, gu_n = prof.get("gemm_gate_up", (0.0, 0))
            gu_avg = min(gu_ms / max(gu_n, 1), ms)
            gu_tf = gate_up_flops(shape, T) / (gu_avg / 1e3) / 1e12 if gu_avg > 0 else 0.0
            roofline.update({"bound": "tensor", "kernel": "gemm_gate_up (tcgen05 CTA-pair grouped GEMM, gate/up + "
                                                          "SiLU epilogue)",
                             "achieved": gu_tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": gu_tf / peaks["bf16_tflops"],
                             "peak_source": f"{peaks['source']} (bf16_tflops, burst)",
                             "flops_per_launch": gate_up_flops(shape, T), "bytes_per_launch": None,
                             "mean_launch_ms": gu_avg})
        else:
            # Expert parallel: the step is routing, two exchanges and the grouped GEMMs
            # overlapped in chunks; the per-rank step is the unit.
            roofline.update({"bound": "tensor", "kernel": "the expert-parallel step (per rank: routing, NCCL "
                                                          "dispatch/return overlapped with the tcgen05 grouped GEMMs, "
                                                          "combine)",
                             "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": tf / peaks["bf16_tflops"],
                             "peak_source": f"{peaks['source']} (bf16_tflops, burst)",
                             "flops_per_launch": lf, "bytes_per_launch": None, "mean_launch_ms": ms,
                             "timing": "the step's CUDA events, max over ranks"})

    # ── end to end through the C ABI with host buffers ──
    x_host = torch.from_numpy(x_bits.view(np.int16)).pin_memory()
    y_pinned = torch.empty((T, shape.hidden), dtype=torch.float32).pin_memory()
    bias_host = torch.from_numpy(bias_np).pin_memory() if wl["bias"] else None
    bias_ptr = bias_host.data_ptr() if wl["bias"] else None
    layer.forward_host_ptr(0, x_host.data_ptr(), T, y_pinned.data_ptr(), bias_ptr)
    e2e_total = 0.0
    barrier()
    for _ in range(args.steps):
        flush()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layer.forward_host_ptr(0, x_host.data_ptr(), T, y_pinned.data_ptr(), bias_ptr)
        e2e_total += time.perf_counter() - t0
    e2e_ms = max_over_ranks(1e3 * e2e_total / args.steps)
    e2e = {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": T * shape.hidden * 2, "d2h_bytes_per_step": T * shape.hidden * 4,
           "how": "lm_moe_forward_host from pinned host memory, wall clock per call (copies, status read-back "
                  "and one synchronisation inside)"}

    # ── parity of sampled tokens against the oracle (every rank its own tokens) ──
    parity = None
    if not args.no_parity:
        rows = np.linspace(0, T - 1, min(PARITY_SAMPLES, T)).astype(int)
        par = sampled_parity(y_host, x_bits, W, rows, bias=bias_np)
        if world > 1:
            t = torch.tensor([par["max_rel"], -par["min_cos"], float(not par["pass"])], dtype=torch.float64,
                             device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            par.update({"max_rel": float(t[0]), "min_cos": float(-t[1]), "pass": bool(t[2] == 0),
                        "tokens": par["tokens"] * world, "ranks": world,
                        "exempt_near_ties": "rank 0: " + str(par["exempt_near_ties"])})
        parity = par

    # ── one-GPU extras: the decode sweep, the prefill batch, the expert-parallel base ──
    sweep, prefill_obj, ep_base = [], None, None
    if extras and not args.no_sweep:
        for t in SWEEP:
            xs = bf16_tensor(syn.tokens(shape, t, seed=SEED_SWEEP))
            ys = torch.empty((t, shape.hidden), dtype=torch.float32, device="cuda")
            for _ in range(3):
                layer.forward(0, xs, y=ys)
            layer.sync()
            tt = int((layer.expert_counts() > 0).sum())
            m = time_steps(layer, xs, ys, flush, max(5, args.steps // 2), torch)
            b = layer_bytes(shape, tt, t)
            sweep.append({"tokens": t, "seed_tokens": SEED_SWEEP, "tokens_per_s": t / (m / 1e3), "ms": m,
                          "touched_experts": tt, "layer_gbs": b / (m / 1e3) / 1e9,
                          "frac_hbm": b / (m / 1e3) / 1e9 / peaks["hbm_gbs"],
                          "phase_trace_us": phase_trace(layer, xs, ys, flush, torch)})
    if extras and not args.no_prefill:
        prefill_obj = measure_prefill(layer, W, flush, args, torch, peaks)
    if extras and not args.no_ep_base:
        layer.upload_layer(1, syn.layer_weights(shape, seed=SEED_EP))
        ep_base = measure_ep_base(layer, flush, args, torch)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        xf = syn.bf16_to_f32(x_bits).reshape(T, -1)
        # A bounded sample (at most 256 tokens) of the same batch, per-token rate.
        cpu = cpu_reference_rate(W, xf[:256], args.cpu_seconds, bias=bias_np)

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": wl["config"],
        "roofline": roofline, "layer_roofline": layer_roofline, "cpu_baseline": cpu, "e2e": e2e,
        "clocks": clock_info, "gpu_launches": kernels_per_forward(T, world, sms=device_sms(torch)) * args.steps,
        "parity": parity, "wall_s_timed_region": wall,
    }
    if extras:
        line.update({"sweep": sweep, "prefill": prefill_obj, "ep_base": ep_base})
    if rank == 0:
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
