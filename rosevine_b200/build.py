"""Build librvcuda.so in-tree with nvcc for sm_100a (no GPU needed to compile)."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "librvcuda.so")
SOURCES = ["csrc/rvcuda.cu"]
HEADERS = ["csrc/common.cuh", "csrc/norm.cuh", "csrc/router.cuh", "csrc/router_fast.cuh", "csrc/decode_fused.cuh", "csrc/pack.cuh",
           "csrc/prefill.cuh", "csrc/prefill_tc.cuh", "csrc/gguf.h", "csrc/dense.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC", "-shared", "-cudart", "static"]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = SOURCES + HEADERS + [os.path.join("..", "include", "rvcuda.h")]
    return any(os.path.getmtime(os.path.join(HERE, d)) > t for d in deps)


def build(force: bool = False, verbose: bool = False, profile_out: str | None = None) -> str:
    """Build librvcuda.so; with profile_out, build a profiling variant (phase timestamps,
    -DRVC_PROFILE) at that path instead."""
    out = profile_out or LIB
    if not force and not profile_out and not stale():
        return LIB
    cmd = [NVCC, *FLAGS, *([] if not verbose else ["-Xptxas", "-v"]), *(["-DRVC_PROFILE"] if profile_out else []),
           "-o", out, *[os.path.join(HERE, s) for s in SOURCES]]
    subprocess.run(cmd, check=True, cwd=HERE)
    return out


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(LIB)
