"""Where a decode layer call's time goes, from the phase marks of a profiling build.

Builds librvcuda with -DRVC_PROFILE (rosevine_b200/librvcuda_prof.so, once), runs one
rvc_moe_forward call per batch size on the synthetic target layer after three warm-up calls and
an L2 flush, and prints:
  - for every CTA of the three decode kernels, the global-timer marks (us from the router
    kernel's start): router start / end, gate start, plan done (routing read, exact fallback for
    uncertified tokens, stable plan), first weight stages in, gate end, down start / end;
  - CTA 0's trace of the gate/up units (weight stages ready, dots start, h phase start, unit
    done) and of the down stages (start, tiles in, records in, done).
The profiling build's marks cost a little time themselves; compare phases, not totals.

Run on a B200 from the repository root:
    python rosevine_b200/micro/decode_timeline.py 8 32
"""
import ctypes
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from rosevine_b200 import build, rvcuda  # noqa: E402

PROF_LIB = os.path.join(ROOT, "rosevine_b200", "librvcuda_prof.so")
MARKS = [(0, "router start"), (1, "router end"), (2, "gate start"), (3, "plan done"), (4, "first stages in"),
         (5, "gate end"), (6, "down start"), (7, "down end")]
G_PROF = (8, 1024, 8)  # g_prof[kernel slot][CTA or trace index][point] (common.cuh)


def main(batches):
    if not os.path.exists(PROF_LIB):
        build.build(profile_out=PROF_LIB)
    rvcuda.LIB_PATH = PROF_LIB
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer, to_device_x
    lib = rvcuda.lib()
    gu, dn = synth.experts(2)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    prof = np.zeros(G_PROF, np.uint64)
    clk = np.zeros(G_PROF, np.int64)

    def dump():
        rc = lib.rvc_profile_dump(prof.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(prof.nbytes),
                                  clk.ctypes.data_as(ctypes.c_void_p))
        assert rc == 0, rc

    G = torch.cuda.get_device_properties(0).multi_processor_count
    for B in batches:
        layer = MoeLayer(synth.router(1), gu, dn, max_tok=B)
        x = to_device_x(synth.tokens(B, 3000 + B), "cuda")
        out = torch.empty((B, synth.N_EMBD), dtype=torch.float32, device="cuda")
        for _ in range(3):
            layer.forward(x, out=out)
        torch.cuda.synchronize()
        layer.status()
        flush.zero_()
        torch.cuda.synchronize()
        dump()  # clears the marks of the warm-up calls
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        layer.forward(x, out=out)
        ev[1].record()
        torch.cuda.synchronize()
        dump()
        layer.status()
        m = prof[4, :G].astype(np.float64)
        t0 = m[:, 0][m[:, 0] > 0].min()
        print(f"B={B}: {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us (profiling build)")
        for p, name in MARKS:
            v = m[:, p]
            v = (v[v > 0] - t0) / 1e3
            if len(v):
                print(f"  {name:16s} min {v.min():7.1f}  median {np.median(v):7.1f}  max {v.max():7.1f} us")
        for slot, what, cols in [(5, "gate/up units", "stages ready / dots start / h start / done"),
                                 (6, "down stages", "start / tiles in / records in / done")]:
            tr = prof[slot].astype(np.float64)
            rows = [(i, tr[i]) for i in range(G_PROF[1]) if tr[i, 0] > 0]
            if rows:
                base = rows[0][1][0]
                print(f"  CTA 0 {what} ({len(rows)}), us from the first: {cols}")
                for i, r in rows[:12]:
                    print("    %3d " % i + " ".join("%7.2f" % v for v in (r[:4] - base) / 1e3))
        prof[:] = 0


if __name__ == "__main__":
    main([int(b) for b in sys.argv[1:]] or [1, 8, 32])
