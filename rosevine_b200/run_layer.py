"""Run one MoE layer on synthetic inputs a few times (for profilers and quick timing).

    python -m rosevine_b200.run_layer --tokens 2048 --zipf --calls 3 [--time]

Builds the layer with the benchmark's seeded synthetic weights (synth.experts(2),
synth.router(1)), bf16 tokens synth.tokens(n, 3000 + n) and, with --zipf, the Zipf(1.1)
per-expert router bias of configs[2]; calls forward `--calls` times and checks the status word.
With --time it also prints the median CUDA-event time of further calls, each after an L2 flush.
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from . import synth
from .moe import MoeLayer, to_device_x


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--zipf", action="store_true")
    ap.add_argument("--time", action="store_true")
    a = ap.parse_args()
    n = a.tokens
    gu, dn = synth.experts(2)
    layer = MoeLayer(synth.router(1), gu, dn, max_tok=n)
    bias = torch.from_numpy(synth.zipf_bias(5)).cuda() if a.zipf else None
    x = to_device_x(synth.tokens(n, 3000 + n), "cuda")
    out = torch.empty((n, synth.N_EMBD), dtype=torch.float32, device="cuda")
    for _ in range(a.calls):
        layer.forward(x, out=out, bias=bias)
    torch.cuda.synchronize()
    layer.status()
    if a.time:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ts = []
        for _ in range(10):
            flush.zero_()
            ev[0].record()
            layer.forward(x, out=out, bias=bias)
            ev[1].record()
            torch.cuda.synchronize()
            ts.append(ev[0].elapsed_time(ev[1]))
        t = float(np.median(ts))
        print(f"{n} tokens: {t * 1e3:.1f} us per layer call, {n / t * 1e3:.0f} tokens/s")
        layer.status()
    print("ok")


if __name__ == "__main__":
    main()
