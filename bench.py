#!/usr/bin/env python3
"""Benchmark of the B200 MoE layer (driver contract: one JSON line on rank 0).

Metric (BASELINE): MoE layer us/token at B=1 (HBM GB/s) and prefill tokens/s at 1/2/4/8 GPUs.

- value: prefill tokens/s of one MoE layer over PREFILL_TOK = 16384 tokens (configs[3]: bf16
  N(0,1) RMS-normalised rows, the random router's natural, near-uniform routing, Q4_0 experts of
  the target's shapes 2816 / 704 / 128 experts / top-8). At N = 1 the tokens go through the
  single-device layer (rvc_moe_forward); at N > 1 (torchrun) each rank holds 128/N experts and
  16384/N tokens and the layer runs expert-parallel (rosevine_b200.ep: NCCL all-to-allv
  dispatch/combine). Total work is fixed (strong scaling); device time by CUDA events on the
  launching stream, max over ranks. The inputs (92 MB of x, 428 MB of experts, 1.5 GB of
  intermediates) exceed the 126 MB L2, so no flush is needed between steps.
- prefill: per-step ms, int8 TOPS against the int8 dense peak (2 x the measured bf16 peak), and
  at N > 1 the exposed all-to-all time (dispatch and combine, CUDA events).
- decode (N = 1): the batched-decode sweep of configs[1], B in {1, 2, 4, 8, 16, 32, 64}, L2
  flushed (256 MB write) before every timed call: per-B us/layer, achieved HBM GB/s
  (algorithmic bytes: distinct experts x 3,345,408 B + router + activations), the headline
  us/token at B = 1, and its roofline against the measured HBM peak.
- roofline: at N = 1 the dominant kernels, the two grouped expert GEMMs, re-run alone on the
  layer's plan and records (rvc_prefill_gemms) and timed with CUDA events, against the int8
  peak, with the whole layer's figure beside them; at N > 1 the expert-parallel layer. The
  decode sub-object carries the decode layer's HBM roofline.
- e2e: the prefill through the public API from pinned host buffers (H2D of x, the layer, D2H of
  the output inside the timed region).
- cpu_baseline (N = 1): the oracle port of the reference CPU-experts Q8_0 path (AVX2, all host
  cores) on a bounded sample of the prefill workload.

`--impl reference` times that CPU path alone on the prefill workload (rank 0 only).
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
PREFILL_TOK = 16384
# --workload: the configuration the prefill step runs (configs[3] unless asked otherwise):
#   config2  2,048 tokens, router logits plus a Zipf(1.1) per-expert bias (uneven expert groups)
#   config4  8,192 tokens, 90% of them forced onto experts 0-7 (all held by rank 0 under
#            expert parallelism: the adversarial hot-expert load)
WORKLOADS = {"config3": 16384, "config2": 2048, "config4": 8192}
WORKLOAD = "config3"
EXPERT_BYTES = 3_345_408
ROUTER_BYTES = 128 * 2816 * 2
OPS_PER_TOKEN = 2 * 8 * (1408 * 2816 + 2816 * 704)  # int8 MACs x 2 of the 8 experts' gate/up and down
DTYPE = "int8xq4 (Q8_0 x Q4_0, f32 accumulate)"
DATA = "synthetic (seeded; BASELINE distributions)"


def algorithmic_bytes(n_tok: int, distinct: int) -> int:
    return distinct * EXPERT_BYTES + ROUTER_BYTES + n_tok * 2816 * 2 + n_tok * 2816 * 4


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "int8_tops": 2 * d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "int8_tops": 2 * 1590.0, "source": "fallback"}


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
    """SM clock, power and clock-event (throttle) reasons of one GPU during the timed region,
    read-only. Sampled through NVML from a background thread of this process, every 20 ms (the
    thread never touches the CUDA context; an nvidia-smi subprocess polling at 100 ms stretched the
    expert-parallel step's host synchronisations); falls back to `nvidia-smi -lms 200`."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_id: str):
        self.idx = gpu_id  # "GPU-<uuid>" of the device under test (or an nvidia-smi index)
        self.proc = None
        self.thread = None
        self.samples = []
        self.path = os.path.join("/tmp", f"rvc_clocks_{os.getpid()}.csv")

    def _nvml_loop(self, nv, h):
        while not self.stop_flag.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:  # noqa: BLE001 - a failed read is a missing sample
                pass
            self.stop_flag.wait(0.02)

    def start(self):
        """Start sampling and wait (up to 5 s) for the first sample, so that the timed region that
        follows is covered from its start."""
        import threading
        self.stop_flag = threading.Event()
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = (nv.nvmlDeviceGetHandleByUUID(self.idx) if self.idx.startswith("GPU-")
                 else nv.nvmlDeviceGetHandleByIndex(int(self.idx)))
            self.nv = nv
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
            t_end = time.time() + 5.0
            while not self.samples and time.time() < t_end:
                time.sleep(0.01)
            return
        except Exception:  # noqa: BLE001 - no NVML: the nvidia-smi fallback
            self.thread = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            sm = [float(x[0]) for x in self.samples]
            mx = [float(x[1]) for x in self.samples]
            reasons = sorted({n for _, _, r in self.samples for n, bit in self.REASONS if r & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                    "reasons": reasons, "samples": len(sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
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
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ------------------------------------------------------------- CPU baseline
def cpu_prefill(budget_s: float, seed: int, threads: int | None = None) -> dict:
    """The oracle port of the reference CPU-experts Q8_0 path on host cores, over consecutive
    256-token slices of the prefill workload for about budget_s seconds."""
    from oracle import oracle as O
    O.build()
    weights, x, _ = prefill_inputs(seed, 0, 1)  # the headline workload only
    pool = O.Pool(threads)
    try:
        O.moe_layer(pool, x[:64], x[:64], weights["w_router"], weights["gate_up"], weights["down"])  # page in
        done, t_cpu, i = 0, 0.0, 0
        while t_cpu < budget_s or done == 0:
            s = x[(i * 256) % PREFILL_TOK:(i * 256) % PREFILL_TOK + 256]
            t0 = time.perf_counter()
            O.moe_layer(pool, s, s, weights["w_router"], weights["gate_up"], weights["down"])
            t_cpu += time.perf_counter() - t0
            done += s.shape[0]
            i += 1
        n = pool.threads
    finally:
        pool.close()
    return {"value": done / t_cpu, "unit": "tokens/s", "cores": n, "kind": "port",
            "sample": f"{done} of the {PREFILL_TOK} prefill tokens in 256-token calls, ~{t_cpu:.0f} s of CPU work; "
                      f"oracle/rv_oracle.c AVX2 int8 routine, persistent pool of {n} threads"}


# ------------------------------------------------------------------- inputs
def prefill_inputs(seed: int, rank: int, world: int):
    """Weights (all experts), this rank's shard of the prefill tokens, and its router bias (None,
    a per-expert [128] Zipf bias, or per-token [n, 128] hot-expert rows) for the workload."""
    from rosevine_b200 import synth
    gu, dn = synth.experts(seed + 2)
    weights = {"gate_up": gu, "down": dn, "w_router": synth.router(seed + 1)}
    x = synth.tokens(PREFILL_TOK, seed + 77)
    n = PREFILL_TOK // world
    bias = None
    if WORKLOAD == "config2":
        bias = synth.zipf_bias(seed + 5)
    elif WORKLOAD == "config4":
        bias = synth.hot_expert_bias(seed + 3, PREFILL_TOK, np.arange(8, dtype=np.int64))[rank * n:(rank + 1) * n]
    return weights, x[rank * n:(rank + 1) * n], bias


def bias_rows(bias, a: int, b: int):
    """The oracle's bias arguments for tokens a .. b - 1 of the workload: (bias, bias_stride)."""
    if bias is None:
        return None, 0
    return (bias, 0) if bias.ndim == 1 else (np.ascontiguousarray(bias[a:b]), bias.shape[1])


def make_inputs(seed: int = 0):
    from rosevine_b200 import synth
    gu, dn = synth.experts(seed + 2)
    weights = {"gate_up": gu, "down": dn, "w_router": synth.router(seed + 1)}
    inputs = {b: synth.tokens(b, seed + 1000 + b) for b in SWEEP}
    return weights, inputs


def distinct_experts(ids: np.ndarray) -> int:
    return int(np.unique(ids).size)


# ---------------------------------------------------------------- decode sweep (N = 1)
def run_decode(args, local_rank: int, peaks: dict) -> dict:
    import torch
    from rosevine_b200.moe import MoeLayer, to_device_x

    dev = torch.device("cuda", local_rank)
    weights, inputs = make_inputs(args.seed)
    layer = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=max(SWEEP), device=local_rank)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    xs = {b: to_device_x(inputs[b], dev) for b in SWEEP}
    outs = {b: torch.empty((b, 2816), dtype=torch.float32, device=dev) for b in SWEEP}
    ids = {b: torch.empty((b, 8), dtype=torch.int32, device=dev) for b in SWEEP}
    wts = {b: torch.empty((b, 8), dtype=torch.float32, device=dev) for b in SWEEP}
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in SWEEP]
    # one CUDA graph per B holding the layer call (warm-up outside capture first)
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

    def step(which, timed: bool):
        for i, b in enumerate(SWEEP):
            flush.zero_()
            if timed:
                ev[i][0].record(stream)
            which[b].replay()
            if timed:
                ev[i][1].record(stream)

    def timed_loop(which, steps, warmup):
        for _ in range(warmup):
            step(which, False)
        torch.cuda.synchronize()
        per_b = {b: 0.0 for b in SWEEP}
        for _ in range(steps):
            step(which, True)
            torch.cuda.synchronize()
            for i, b in enumerate(SWEEP):
                per_b[b] += ev[i][0].elapsed_time(ev[i][1])
        return {b: per_b[b] / steps for b in SWEEP}  # ms per call

    steps = max(10, args.decode_steps)
    per_b = timed_loop(graphs, steps, args.warmup)
    phase = timed_loop(graphs_exp, steps, args.warmup)
    layer.status(stream=sh)
    distinct = {b: distinct_experts(ids[b].cpu().numpy()) for b in SWEEP}
    rows = []
    for b in SWEEP:
        byt = algorithmic_bytes(b, distinct[b])
        rows.append({"B": b, "us_per_layer": per_b[b] * 1e3, "distinct_experts": distinct[b], "algorithmic_bytes": byt,
                     "hbm_gbs": byt / (per_b[b] * 1e-3) / 1e9, "frac_of_hbm": byt / (per_b[b] * 1e-3) / 1e9 /
                     peaks["hbm_gbs"], "expert_phase_us": phase[b] * 1e3})
    lay_bytes = sum(algorithmic_bytes(b, distinct[b]) for b in SWEEP)
    sweep_ms = sum(per_b.values())
    achieved = lay_bytes / (sweep_ms * 1e-3) / 1e9
    ph_gbs = sum(distinct[b] * EXPERT_BYTES for b in SWEEP) / (sum(phase.values()) * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "decode layer (rvc_moe_forward: k_fd_route, k_fd_gate, k_fd_down up to "
                                           "64 tokens, the prefill kernels above), algorithmic bytes and device time "
                                           "summed over the B sweep",
                "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "peak_source": peaks["source"], "b1_frac": rows[0]["frac_of_hbm"],
                "expert_phase_gbs": ph_gbs, "expert_phase_frac": ph_gbs / peaks["hbm_gbs"], "traffic": None}
    return {"workload": "configs[1]: batched decode sweep B in {1,2,4,8,16,32,64}, L2 flushed before every call",
            "steps": steps, "b1_us_per_token": per_b[1] * 1e3, "b1_hbm_gbs": rows[0]["hbm_gbs"],
            "sweep_tokens_per_s": sum(SWEEP) / (sweep_ms * 1e-3), "per_b": rows, "roofline": roofline,
            "gpu_launches_per_call": {str(b): (3 if b <= 64 else 7) for b in SWEEP}}  # decode / prefill kernels


# ---------------------------------------------------------------- prefill (all N)
def run_prefill(args, rank: int, world: int, local_rank: int, peaks: dict) -> dict:
    import torch
    import torch.distributed as dist
    from rosevine_b200.moe import MoeLayer, to_device_x

    dev = torch.device("cuda", local_rank)
    weights, xs, bias_np = prefill_inputs(args.seed, rank, world)
    n = xs.shape[0]
    x = to_device_x(xs, dev)
    bias = None if bias_np is None else torch.from_numpy(np.ascontiguousarray(bias_np)).to(dev)
    hx = torch.from_numpy(xs.view(np.int16)).pin_memory()
    ho = torch.empty((n, 2816), dtype=torch.float32).pin_memory()
    if world == 1:
        layer = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=n, device=local_rank)
        out = torch.empty((n, 2816), dtype=torch.float32, device=dev)

        def fwd():
            return layer.forward(x, out=out, bias=bias)
        launches = 7  # k_router_chains4, k_select, k_plan, k_pf_quant, 2 x k_pf_gemm_tc, k_pf_combine
        check = layer.status
    else:
        from rosevine_b200.ep import EpMoeLayer, GpuBackend, local_experts
        gl, dl = local_experts(weights["gate_up"], weights["down"], rank, world)
        be = GpuBackend(weights["w_router"], gl, dl, 128 // world, max_tok=n, max_rows=PREFILL_TOK, world=world,
                        device=local_rank)
        layer = EpMoeLayer(be, rank, world)

        def fwd():
            return layer.forward(x, bias=bias)
        # k_router_chains4, k_select, k_quant_rows, k_ep_count, k_ep_pack, k_ep_meta, k_plan, k_ep_scatter,
        # 2 x k_pf_gemm_tc, k_pf_combine, k_ep_reduce (NCCL's and torch's own kernels not counted)
        launches = 12
        check = be.status
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def loop(steps, e2e: bool):
        """K steps back to back between two events: no host synchronisation of the bench's own
        (the expert-parallel layer reads its row counts once per step)."""
        ev0.record(stream)
        for _ in range(steps):
            if e2e:
                x.copy_(hx.view(torch.bfloat16), non_blocking=True)
            o = fwd()
            if e2e:
                ho.copy_(o, non_blocking=True)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / steps

    for _ in range(args.warmup):
        fwd()
    torch.cuda.synchronize()
    # one sampler per node (local rank 0, its own GPU)
    clocks = ClockSampler(gpu_smi_id(local_rank)) if local_rank == 0 else None
    if clocks:
        clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    step_ms = loop(args.steps, False)
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    e2e_ms = loop(max(3, args.steps // 2), True)
    check()
    disp_ms = comb_ms = 0.0
    phases = {}
    if world > 1:
        # the phase split, in a separate pass: events between the phases, read after each step
        layer.timing = True
        k = max(3, args.steps // 2)
        for _ in range(k):
            fwd()
            torch.cuda.synchronize()
            st = layer.phase_times()
            disp_ms += st.dispatch_ms / k
            comb_ms += st.combine_ms / k
            for name, v in st.phases_ms.items():
                phases[name] = phases.get(name, 0.0) + v / k
        layer.timing = False
    gemm_ms = None
    if world == 1:
        # the dominant kernels alone: the two grouped GEMMs (k_pf_gemm_tc gate/up and down)
        # re-run on the last call's plan, records and scale planes (rvc_prefill_gemms), timed
        # with events on the stream they run on; weights and records exceed the L2
        from rosevine_b200 import rvcuda as rc
        fwd()
        for _ in range(2):
            rc.prefill_gemms(layer.w, layer.ws, stream.cuda_stream)
        torch.cuda.synchronize()
        k = max(3, args.steps // 2)
        ev0.record(stream)
        for _ in range(k):
            rc.prefill_gemms(layer.w, layer.ws, stream.cuda_stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        gemm_ms = ev0.elapsed_time(ev1) / k
        check()
    if world == 1:
        ids_t = torch.empty((n, 8), dtype=torch.int32, device=dev)
        o = layer.forward(x, ids=ids_t, bias=bias)
    else:
        o = layer.forward(x, bias=bias)
        ids_t = layer.last_ids
    par = prefill_parity(args, o, ids_t, xs, weights, rank, world, dev, bias_np)
    t = torch.tensor([step_ms, e2e_ms, disp_ms, comb_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms, disp_ms, comb_ms = (float(v) for v in t)
    par = reduce_parity(par, world, dev)
    tops = OPS_PER_TOKEN * PREFILL_TOK / world / (step_ms * 1e-3) / 1e12
    gemm_tops = OPS_PER_TOKEN * PREFILL_TOK / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    return {"gemm_ms": gemm_ms, "gemm_int8_tops": gemm_tops, "step_ms": step_ms, "e2e_ms": e2e_ms, "tokens_per_s": PREFILL_TOK / (step_ms * 1e-3),
            "e2e_tokens_per_s": PREFILL_TOK / (e2e_ms * 1e-3), "int8_tops_per_gpu": tops,
            "int8_frac_per_gpu": tops / peaks["int8_tops"], "exposed_all_to_all_ms": disp_ms + comb_ms,
            "dispatch_ms": disp_ms, "combine_ms": comb_ms, "launches": launches, "clocks": clk,
            "rank0_phases_ms": phases or None, "parity": par,
            "h2d_bytes_per_step": PREFILL_TOK * 2816 * 2, "d2h_bytes_per_step": PREFILL_TOK * 2816 * 4}


PARITY_ROWS = 32   # oracle-checked output rows per rank
PARITY_TOL = 1e-3  # max |gpu - cpu| / max |cpu| per row (the north star's tolerance)


def prefill_parity(args, out, ids_t, xs, weights, rank: int, world: int, dev, bias=None) -> dict:
    """A seeded sample of this rank's output rows against the oracle (the reference's scalar
    Q8_0 CPU path): expert ids exact, per-row relative error. Rows whose router has an exact
    tie among the top 9 probabilities would be left out and counted."""
    import torch
    from oracle import oracle as O
    O.build()
    n = xs.shape[0]
    rows = np.sort(np.random.default_rng(args.seed + 1000 + rank).choice(n, size=min(PARITY_ROWS, n), replace=False))
    got = out[torch.as_tensor(rows, device=dev)].cpu().numpy()
    ids = ids_t[torch.as_tensor(rows, device=dev)].cpu().numpy()
    threads = max(1, (os.cpu_count() or 1) // world)
    pool = O.Pool(threads, kernel=O.KERNEL_SCALAR)
    try:
        b = None if bias is None else (bias if bias.ndim == 1 else np.ascontiguousarray(bias[rows]))
        want, want_ids, _, lg = O.moe_layer(pool, xs[rows], xs[rows], weights["w_router"], weights["gate_up"],
                                            weights["down"], bias=b,
                                            bias_stride=0 if b is None or b.ndim == 1 else b.shape[1])
    finally:
        pool.close()
    _, _, probs = O.select_experts(lg, 8)
    srt = -np.sort(-probs, axis=1)
    tie = np.any(srt[:, :8] == srt[:, 1:9], axis=1)
    keep = ~tie
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    return {"rows": int(keep.sum()), "ties_excluded": int(tie.sum()),
            "ids_mismatch": int((ids[keep] != want_ids[keep]).any(axis=1).sum()),
            "max_row_rel_err": float(err[keep].max()) if keep.any() else 0.0}


def reduce_parity(p: dict, world: int, dev) -> dict:
    import torch
    import torch.distributed as dist
    t = torch.tensor([p["rows"], p["ties_excluded"], p["ids_mismatch"]], dtype=torch.float64, device=dev)
    e = torch.tensor([p["max_row_rel_err"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t)
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
    rows, ties, bad = (int(v) for v in t.tolist())
    err = float(e.item())
    return {"checked_rows": rows, "ranks": world, "ties_excluded": ties, "ids_mismatch_rows": bad,
            "max_row_rel_err": err, "tol": PARITY_TOL, "oracle": "oracle/rv_oracle.c scalar Q8_0 (reference order)",
            "pass": bad == 0 and err <= PARITY_TOL}


def roofline(pf: dict, peaks: dict) -> dict:
    """The dominant kernels (the two grouped GEMMs, timed alone at N=1) against the int8 peak
    (derived: 2 x the measured bf16 dense peak; no int8 GEMM is measured on this pool), with the
    fraction of the f16 tensor pipe they run on (kind::f16 MMAs) beside it; at N>1 the
    expert-parallel layer as a whole."""
    r = {"bound": "tensor", "peak": peaks["int8_tops"], "unit": "TOP/s",
         "peak_source": "derived: 2 x " + peaks["source"] + " bf16 dense", "traffic": None,
         "layer_achieved": pf["int8_tops_per_gpu"], "layer_frac": pf["int8_frac_per_gpu"]}
    if pf.get("gemm_int8_tops"):
        r.update(kernel="k_pf_gemm_tc<gate/up> + k_pf_gemm_tc<down> (the grouped expert GEMMs on tcgen05 kind::f16 "
                        "with f16-held integer operands, re-run alone by rvc_prefill_gemms on the layer's plan and "
                        "records), int8 MACs of the experts x 2 per average launch pair", achieved=pf["gemm_int8_tops"],
                 frac=pf["gemm_int8_tops"] / peaks["int8_tops"], gemm_ms=pf["gemm_ms"],
                 f16_pipe_frac=pf["gemm_int8_tops"] / (peaks["int8_tops"] / 2))
    else:
        r.update(kernel="expert-parallel prefill layer (router, pack, all-to-allv, grouped GEMMs k_pf_gemm_tc, "
                        "combine, reduce), int8 MACs of the experts x 2", achieved=pf["int8_tops_per_gpu"],
                 frac=pf["int8_frac_per_gpu"])
    return r


WORKLOAD_NAME = {"config3": "configs[3]", "config2": "configs[2] (Zipf(1.1) expert bias)",
                 "config4": "configs[4] (90% of tokens on experts 0-7)"}


def run_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    torch.cuda.set_device(local_rank)
    peaks = measured_peaks()
    pf = run_prefill(args, rank, world, local_rank, peaks)
    dec = run_decode(args, local_rank, peaks) if world == 1 and not args.no_decode else None
    if rank != 0:
        return None
    res = {
        "metric": METRIC, "value": pf["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": pf["step_ms"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": DTYPE, "data": DATA,
        "config": {"workload": f"{WORKLOAD_NAME[WORKLOAD]} at N={world}: prefill of {PREFILL_TOK} tokens through one "
                               f"MoE layer (2816/704, 128 experts, top-8, Q4_0 experts, bf16 x), "
                               + ("single device" if world == 1 else f"expert-parallel, {128 // world} experts "
                                  f"and {PREFILL_TOK // world} tokens per GPU, NCCL all-to-allv"),
                   "tokens_per_step": PREFILL_TOK, "l2": "inputs and intermediates larger than the 126 MB L2",
                   "parallelism": "single GPU" if world == 1 else f"ep{world}"},
        "prefill": {k: v for k, v in pf.items() if k != "clocks"},
        "roofline": roofline(pf, peaks),
        "e2e": {"value": pf["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": pf["h2d_bytes_per_step"],
                "d2h_bytes_per_step": pf["d2h_bytes_per_step"]},
        "gpu_launches": pf["launches"] * args.steps * world,
        "clocks": pf["clocks"],
    }
    if dec is not None:
        res["decode"] = dec
    if world == 1 and not args.no_cpu:
        res["cpu_baseline"] = cpu_prefill(args.cpu_budget, args.seed)
    return res


def run_reference(args, rank: int) -> dict | None:
    """The reference arm: the oracle port of the reference CPU-experts Q8_0 path on the host's
    cores, each step a 256-token slice of the same prefill workload (rank 0 only)."""
    if rank != 0:
        return None
    from oracle import oracle as O
    O.build()
    weights, x, bias = prefill_inputs(args.seed, 0, 1)
    pool = O.Pool(None)
    sl = 256
    O.moe_layer(pool, x[:64], x[:64], weights["w_router"], weights["gate_up"], weights["down"])
    for i in range(args.warmup):
        s = x[i * sl:(i + 1) * sl]
        b, bs = bias_rows(bias, i * sl, (i + 1) * sl)
        O.moe_layer(pool, s, s, weights["w_router"], weights["gate_up"], weights["down"], bias=b, bias_stride=bs)
    steps = max(1, min(args.steps, 8))  # bounded: a few minutes of host work at most
    ts = []
    for i in range(steps):
        a0 = (i * sl) % PREFILL_TOK
        s = x[a0:a0 + sl]
        b, bs = bias_rows(bias, a0, a0 + sl)
        t0 = time.perf_counter()
        O.moe_layer(pool, s, s, weights["w_router"], weights["gate_up"], weights["down"], bias=b, bias_stride=bs)
        ts.append(time.perf_counter() - t0)
    threads = pool.threads
    pool.close()
    step = statistics.median(ts)
    v = sl / step
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": args.warmup, "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE, "data": DATA, "impl": "reference",
            "config": {"workload": f"{WORKLOAD_NAME[WORKLOAD]} prefill workload ({PREFILL_TOK} tokens) on the reference's CPU-experts "
                                   f"Q8_0 path (oracle port: the Rust toolchain is absent), {sl}-token slices",
                       "tokens_per_step": sl, "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{steps} slices of {sl} tokens of the prefill workload, median"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--decode-steps", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config3",
                    help="prefill configuration (configs[3] is the headline; the others skip the decode "
                         "sweep and the CPU baseline)")
    args = ap.parse_args()
    global PREFILL_TOK, WORKLOAD
    WORKLOAD, PREFILL_TOK = args.workload, WORKLOADS[args.workload]
    if WORKLOAD != "config3":
        args.no_decode = args.no_cpu = True
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
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
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
