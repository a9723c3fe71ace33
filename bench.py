#!/usr/bin/env python3
"""Benchmark of the B200 MoE layer (driver contract: one JSON line on rank 0).

Workload at N=1: the batched-decode sweep of one MoE layer,
B in {1, 2, 4, 8, 16, 32, 64} tokens, seeded synthetic bf16 inputs and Q4_0 experts of the
target's shapes (2816 / 704 / 128 experts / top-8). One step = one layer call at every B
(127 tokens). The L2 (126 MB) is flushed before every timed layer call by writing a 256 MB
buffer outside the timed events, so expert weights always stream from HBM.

- value: tokens/s over the sweep, device time (CUDA events on the launching stream);
- decode: per-B us/layer and achieved HBM GB/s (algorithmic bytes: distinct experts x
  3,345,408 B + router + activations), the headline us/token at B=1;
- roofline: the expert GEMV phase (rvc_moe_experts) timed alone against the measured HBM peak;
- e2e: the same sweep through the C ABI from pinned host buffers (H2D of x, the layer, D2H
  of the output, all inside the timed region);
- cpu_baseline: the oracle's port of the reference CPU-experts Q8_0 path (AVX2, persistent
  pool, all host cores), on a bounded sample of the same sweep.

`--impl reference` times only that CPU path (the reference arm). With N>1 GPUs (torchrun) every
rank runs the sweep as an independent replica (decode at B <= 64 is not sharded), timing is the
max over ranks and value is the whole-job tokens/s.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer µs/token @B=1 (HBM GB/s) and prefill tokens/s @1/2/4/8 B200"
SWEEP = [1, 2, 4, 8, 16, 32, 64]
EXPERT_BYTES = 3_345_408
ROUTER_BYTES = 128 * 2816 * 2


def algorithmic_bytes(n_tok: int, distinct: int) -> int:
    return distinct * EXPERT_BYTES + ROUTER_BYTES + n_tok * 2816 * 2 + n_tok * 2816 * 4


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ------------------------------------------------------------------- clocks
def gpu_smi_id(local_rank: int) -> str:
    """nvidia-smi --id for the CUDA device local_rank: its UUID (independent of
    CUDA_VISIBLE_DEVICES renumbering), else its index."""
    import torch
    u = getattr(torch.cuda.get_device_properties(local_rank), "uuid", None)
    if u is not None:
        u = str(u)
        return u if u.startswith("GPU-") else "GPU-" + u
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return vis.split(",")[local_rank] if vis else str(local_rank)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.idx = gpu_id  # "GPU-<uuid>" of the device under test (or an nvidia-smi index)
        self.proc = None
        self.path = os.path.join("/tmp", f"rvc_clocks_{os.getpid()}.csv")

    def start(self):
        """Start sampling every 20 ms and wait (up to 5 s) until the first sample is written,
        so that the timed region that follows is covered from its start."""
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.01)
        self.t_start = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline
def cpu_sweep(weights, inputs, budget_s: float, threads: int | None = None) -> dict:
    """The oracle port of the reference CPU-experts Q8_0 path, timed per B on host cores."""
    from oracle import oracle as O
    O.build()
    pool = O.Pool(threads)
    per_b = {}
    try:
        for b in SWEEP:  # warm-up: page the weights in once
            O.moe_layer(pool, inputs[b], inputs[b], weights["w_router"], weights["gate_up"], weights["down"])
        per_b_budget = budget_s / len(SWEEP)
        for b in SWEEP:
            xs = inputs[b]
            ts = []
            t_end = time.perf_counter() + per_b_budget
            while time.perf_counter() < t_end or len(ts) < 3:
                t0 = time.perf_counter()
                O.moe_layer(pool, xs, xs, weights["w_router"], weights["gate_up"], weights["down"])
                ts.append(time.perf_counter() - t0)
            per_b[b] = statistics.median(ts)
        n = pool.threads
    finally:
        pool.close()
    step = sum(per_b.values())
    return {"value": sum(SWEEP) / step, "unit": "tokens/s", "cores": n, "kind": "port",
            "sample": f"median over >=3 calls per B of the B in {SWEEP} sweep, ~{budget_s:.0f} s of CPU work; "
                      f"oracle/rv_oracle.c AVX2 int8 routine, persistent pool",
            "b1_us_per_token": per_b[1] * 1e6, "per_b_ms": {str(b): per_b[b] * 1e3 for b in SWEEP}}


# ------------------------------------------------------------------- inputs
def make_inputs(seed: int = 0):
    from rosevine_b200 import synth
    gu, dn = synth.experts(seed + 2)
    weights = {"gate_up": gu, "down": dn, "w_router": synth.router(seed + 1)}
    inputs = {b: synth.tokens(b, seed + 1000 + b) for b in SWEEP}
    return weights, inputs


def distinct_experts(ids: np.ndarray) -> int:
    return int(np.unique(ids).size)


# ---------------------------------------------------------------- GPU arm
def run_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist
    from rosevine_b200 import rvcuda as rc
    from rosevine_b200.moe import MoeLayer, to_device_x

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    weights, inputs = make_inputs(args.seed + rank)
    layer = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=max(SWEEP), device=local_rank)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    xs = {b: to_device_x(inputs[b], dev) for b in SWEEP}
    outs = {b: torch.empty((b, 2816), dtype=torch.float32, device=dev) for b in SWEEP}
    ids = {b: torch.empty((b, 8), dtype=torch.int32, device=dev) for b in SWEEP}
    wts = {b: torch.empty((b, 8), dtype=torch.float32, device=dev) for b in SWEEP}
    # pinned host buffers for the e2e path
    hx = {b: torch.from_numpy(inputs[b].view(np.int16)).pin_memory() for b in SWEEP}
    ho = {b: torch.empty((b, 2816), dtype=torch.float32).pin_memory() for b in SWEEP}
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in SWEEP]

    # One CUDA graph per B holding the layer call (the C ABI call captured as-is: K0 on the
    # library's side lane, K1, gate/up, down+combine). Warm-up outside capture first.
    graphs, graphs_exp = {}, {}
    for b in SWEEP:
        layer.forward(xs[b], out=outs[b], ids=ids[b], wts=wts[b], stream=sh)
        layer.experts(xs[b], ids[b], wts[b], out=outs[b], stream=sh)
    torch.cuda.synchronize()
    for b in SWEEP:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.forward(xs[b], out=outs[b], ids=ids[b], wts=wts[b])
        graphs[b] = g
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2):
            layer.experts(xs[b], ids[b], wts[b], out=outs[b])
        graphs_exp[b] = g2
    torch.cuda.synchronize()

    def step_graph(timed: bool, which=graphs):
        for i, b in enumerate(SWEEP):
            flush.zero_()
            if timed:
                ev[i][0].record(stream)
            which[b].replay()
            if timed:
                ev[i][1].record(stream)

    def step_stream(timed: bool):
        for i, b in enumerate(SWEEP):
            flush.zero_()
            if timed:
                ev[i][0].record(stream)
            layer.forward(xs[b], out=outs[b], ids=ids[b], wts=wts[b], stream=sh)
            if timed:
                ev[i][1].record(stream)

    def step_e2e(timed: bool):
        for i, b in enumerate(SWEEP):
            flush.zero_()
            if timed:
                ev[i][0].record(stream)
            rc.check(rc.lib().rvc_upload_async(xs[b].data_ptr(), hx[b].data_ptr(), hx[b].numel() * 2, sh))
            layer.forward(xs[b], out=outs[b], ids=ids[b], wts=wts[b], stream=sh)
            rc.check(rc.lib().rvc_download_async(ho[b].data_ptr(), outs[b].data_ptr(), ho[b].numel() * 4, sh))
            if timed:
                ev[i][1].record(stream)

    def timed_loop(fn, steps, warmup):
        for _ in range(warmup):
            fn(False)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        per_b = {b: 0.0 for b in SWEEP}
        for _ in range(steps):
            fn(True)
            torch.cuda.synchronize()
            for i, b in enumerate(SWEEP):
                per_b[b] += ev[i][0].elapsed_time(ev[i][1])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return {b: per_b[b] / steps for b in SWEEP}  # ms per call

    clocks = ClockSampler(gpu_smi_id(local_rank))
    clocks.start()
    per_b = timed_loop(step_graph, args.steps, args.warmup)
    clk = clocks.stop()
    layer.status(stream=sh)
    per_b_stream = timed_loop(step_stream, args.steps, args.warmup)
    per_b_e2e = timed_loop(step_e2e, max(1, args.steps), max(1, args.warmup))
    phase = timed_loop(lambda t: step_graph(t, graphs_exp), args.steps, args.warmup)
    layer.status(stream=sh)

    distinct = {b: distinct_experts(ids[b].cpu().numpy()) for b in SWEEP}
    step_ms = sum(per_b.values())
    e2e_ms = sum(per_b_e2e.values())
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms = float(t[0]), float(t[1])
    if rank != 0:
        return None
    peaks = measured_peaks()
    tokens = sum(SWEEP)
    decode = []
    for b in SWEEP:
        byt = algorithmic_bytes(b, distinct[b])
        decode.append({"B": b, "us_per_layer": per_b[b] * 1e3, "distinct_experts": distinct[b],
                       "algorithmic_bytes": byt, "hbm_gbs": byt / (per_b[b] * 1e-3) / 1e9,
                       "frac_of_hbm": byt / (per_b[b] * 1e-3) / 1e9 / peaks["hbm_gbs"],
                       "us_per_layer_no_graph": per_b_stream[b] * 1e3,
                       "expert_phase_us": phase[b] * 1e3, "e2e_us": per_b_e2e[b] * 1e3})
    # roofline of the whole decode layer over the sweep (algorithmic bytes and device time
    # summed over B), and of the expert GEMV phase alone
    lay_bytes = sum(algorithmic_bytes(b, distinct[b]) for b in SWEEP)
    achieved = lay_bytes / (step_ms * 1e-3) / 1e9
    ph_bytes = sum(distinct[b] * EXPERT_BYTES for b in SWEEP)
    ph_gbs = ph_bytes / (sum(phase.values()) * 1e-3) / 1e9
    h2d = sum(b * 2816 * 2 for b in SWEEP)
    d2h = sum(b * 2816 * 4 for b in SWEEP)
    res = {
        "metric": METRIC, "value": world * tokens / (step_ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4 (Q8_0 x Q4_0, f32 accumulate)",
        "data": "synthetic (seeded; BASELINE distributions)",
        "config": {"workload": "configs[1]: batched decode sweep B in {1,2,4,8,16,32,64}, one MoE layer "
                               "(2816/704, 128 experts, top-8, Q4_0 experts, bf16 x)",
                   "tokens_per_step": tokens, "l2": "flushed (256 MB write) before every timed layer call",
                   "parallelism": "replicas" if world > 1 else "single GPU"},
        "decode": {"b1_us_per_token": per_b[1] * 1e3, "b1_hbm_gbs": decode[0]["hbm_gbs"], "per_b": decode},
        "roofline": {"bound": "hbm", "kernel": "decode layer (rvc_moe_forward: k_fd_route, k_fd_gate, k_fd_down), "
                                                "algorithmic bytes and device time summed over the sweep",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                     "expert_phase_gbs": ph_gbs, "expert_phase_frac": ph_gbs / peaks["hbm_gbs"],
                     "traffic": None},
        "e2e": {"value": world * tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": 3 * len(SWEEP) * args.steps,  # k_fd_route, k_fd_gate, k_fd_down per layer call
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu:
        res["cpu_baseline"] = cpu_sweep(weights, inputs, args.cpu_budget)
    return res


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    weights, inputs = make_inputs(args.seed)
    from oracle import oracle as O
    O.build()
    pool = O.Pool(None)
    for b in SWEEP:
        O.moe_layer(pool, inputs[b], inputs[b], weights["w_router"], weights["gate_up"], weights["down"])
    for _ in range(args.warmup):
        for b in SWEEP[:3]:
            O.moe_layer(pool, inputs[b], inputs[b], weights["w_router"], weights["gate_up"], weights["down"])
    step_times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for b in SWEEP:
            O.moe_layer(pool, inputs[b], inputs[b], weights["w_router"], weights["gate_up"], weights["down"])
        step_times.append(time.perf_counter() - t0)
    threads = pool.threads
    pool.close()
    step = statistics.median(step_times)
    v = sum(SWEEP) / step
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8xq4 (Q8_0 x Q4_0, f32 accumulate)",
            "data": "synthetic (seeded; BASELINE distributions)", "impl": "reference",
            "config": {"workload": "configs[1]: batched decode sweep B in {1,2,4,8,16,32,64} on the reference's "
                                   "CPU-experts Q8_0 path (oracle port: Rust toolchain absent)",
                       "tokens_per_step": sum(SWEEP), "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} full sweeps, median step"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank)
    else:
        if world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        res = run_gpu(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
