"""ctypes binding of the CPU oracle (oracle/rv_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
legs import this module; the product package never does.

The C code restates Rosevine's Q8_0 CPU-experts path (runtime/src/ops.rs,
expert_kernel.rs, expert_pool.rs, exec.rs); see rv_oracle.h for citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "librvoracle.so")

F32, BF16 = 0, 1
KERNEL_SCALAR, KERNEL_AVX2, KERNEL_BEST = 0, 1, 2

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc only; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, F, U16 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint16
        L.rvo_f16_to_f32.argtypes, L.rvo_f16_to_f32.restype = [U16], F
        L.rvo_f32_to_f16.argtypes, L.rvo_f32_to_f16.restype = [F], U16
        L.rvo_bf16_to_f32.argtypes, L.rvo_bf16_to_f32.restype = [U16], F
        L.rvo_quantize_q8_0.argtypes, L.rvo_quantize_q8_0.restype = [P, I, P], None
        L.rvo_gelu.argtypes, L.rvo_gelu.restype = [F], F
        L.rvo_softmax.argtypes, L.rvo_softmax.restype = [P, I], None
        L.rvo_rms_norm.argtypes, L.rvo_rms_norm.restype = [P, P, P, I, I, F, F], None
        L.rvo_matmul_q4_0.argtypes, L.rvo_matmul_q4_0.restype = [P, I, P, I, P, I], None
        L.rvo_shared_mlp.argtypes, L.rvo_shared_mlp.restype = [P, P, P, P, P, P, I, I, I, F, P], None
        L.rvo_top_k.argtypes, L.rvo_top_k.restype = [P, I, I, P], None
        L.rvo_router_logits.argtypes = [P, I, P, I, P, I, I, I, I, P]
        L.rvo_router_logits.restype = None
        L.rvo_select_experts.argtypes, L.rvo_select_experts.restype = [P, I, I, I, P, P], None
        L.rvo_dot_q8_scalar.argtypes, L.rvo_dot_q8_scalar.restype = [P, P, I], F
        L.rvo_dot_q8_avx2.argtypes, L.rvo_dot_q8_avx2.restype = [P, P, I], F
        L.rvo_have_avx2.argtypes, L.rvo_have_avx2.restype = [], I
        L.rvo_block_sumi.argtypes, L.rvo_block_sumi.restype = [P, P], ctypes.c_int32
        L.rvo_moe_plan.argtypes, L.rvo_moe_plan.restype = [P, I, I, P, P, P], None
        L.rvo_pool_new.argtypes, L.rvo_pool_new.restype = [I, I], P
        L.rvo_pool_free.argtypes, L.rvo_pool_free.restype = [P], None
        L.rvo_pool_threads.argtypes, L.rvo_pool_threads.restype = [P], I
        L.rvo_experts_q8.argtypes = [P, P, I, P, P, P, P, P, I, I, I, I, I, P, P, P]
        L.rvo_experts_q8.restype = I
        L.rvo_moe_layer.argtypes = [P, P, P, I, P, I, P, I, P, P, P, I, I, I, I, I, P, P, P, P]
        L.rvo_moe_layer.restype = I
        _lib = L
    return _lib


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:  # bf16 bit patterns
        return BF16
    raise TypeError(f"activations must be float32 or bf16 bits (uint16), got {a.dtype}")


def f16_to_f32(h: int) -> float:
    return lib().rvo_f16_to_f32(h)


def f32_to_f16(f: float) -> int:
    return lib().rvo_f32_to_f16(f)


def gelu(x: float) -> float:
    return lib().rvo_gelu(x)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros((rows, k // 32 * 34), np.uint8)
    for r in range(rows):
        lib().rvo_quantize_q8_0(_p(x.reshape(rows, k)[r:r + 1]), k, _p(out[r:r + 1]))
    return out


def rms_norm(x: np.ndarray, weight: np.ndarray | None = None, eps: float = 1e-6, post: float = 1.0) -> np.ndarray:
    """rvo_rms_norm over the rows of x [rows, width] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, width = x.shape
    out = np.empty_like(x)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
    lib().rvo_rms_norm(_p(x), _p(out), _p(w), rows, width, eps, post)
    return out


def matmul_q4_0(w: np.ndarray, x: np.ndarray, n_out: int) -> np.ndarray:
    """rvo_matmul_q4_0: y [n_in, n_out] = dequant(W) . x for Q4_0 rows w (bytes) and x [n_in, k] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w).view(np.uint8)
    n_in, k = x.shape
    assert w.size == n_out * (k // 32) * 18
    y = np.empty((n_in, n_out), np.float32)
    lib().rvo_matmul_q4_0(_p(w), k, _p(x), n_in, _p(y), n_out)
    return y


def shared_mlp(gate, up, down, ffn_norm, post_norm, x, ff: int, eps: float = 1e-6) -> np.ndarray:
    """rvo_shared_mlp: the dense MLP with its norms on x [n_tok, n_embd] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_tok, n_embd = x.shape
    gate, up, down = (np.ascontiguousarray(a).view(np.uint8) for a in (gate, up, down))
    fn, pn = (np.ascontiguousarray(a, dtype=np.float32) for a in (ffn_norm, post_norm))
    out = np.empty_like(x)
    lib().rvo_shared_mlp(_p(gate), _p(up), _p(down), _p(fn), _p(pn), _p(x), n_tok, n_embd, ff, eps, _p(out))
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().rvo_softmax(_p(y), y.size)
    return y


def top_k(x: np.ndarray, k: int) -> list[int]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    idx = np.zeros(k, np.int32)
    lib().rvo_top_k(_p(x), x.size, k, _p(idx))
    return idx.tolist()


def router_logits(x, w, bias=None, bias_stride=0):
    x, w = np.ascontiguousarray(x), np.ascontiguousarray(w)
    n_tok, n_embd = x.shape
    ne = w.shape[0]
    out = np.zeros((n_tok, ne), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().rvo_router_logits(_p(x), _dtype_code(x), _p(w), _dtype_code(w), _p(b), bias_stride, n_tok, n_embd, ne,
                            _p(out))
    return out


def select_experts(logits: np.ndarray, used: int = 8):
    lg = np.array(logits, dtype=np.float32, copy=True)
    n_tok, ne = lg.shape
    ids = np.zeros((n_tok, used), np.int32)
    w = np.zeros((n_tok, used), np.float32)
    lib().rvo_select_experts(_p(lg), n_tok, ne, used, _p(ids), _p(w))
    return ids, w, lg


def dot_q8(row_q4: np.ndarray, xq8: np.ndarray, k: int, kernel: int = KERNEL_SCALAR) -> float:
    row_q4, xq8 = np.ascontiguousarray(row_q4), np.ascontiguousarray(xq8)
    fn = lib().rvo_dot_q8_avx2 if kernel == KERNEL_AVX2 else lib().rvo_dot_q8_scalar
    return fn(_p(row_q4), _p(xq8), k)


def block_sumi(blk_q4: np.ndarray, blk_q8: np.ndarray) -> int:
    return lib().rvo_block_sumi(_p(np.ascontiguousarray(blk_q4)), _p(np.ascontiguousarray(blk_q8)))


def moe_plan(ids: np.ndarray, n_experts: int = 128):
    ids = np.ascontiguousarray(ids.reshape(-1), dtype=np.int32)
    n = ids.size
    order, pos_of, counts = np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n_experts, np.int32)
    lib().rvo_moe_plan(_p(ids), n, n_experts, _p(order), _p(pos_of), _p(counts))
    return order, pos_of, counts


class Pool:
    """Persistent worker pool (expert_pool.rs WorkerPool) used by the expert path."""

    def __init__(self, threads: int | None = None, kernel: int = KERNEL_BEST):
        self.threads = threads or os.cpu_count() or 1
        self.h = lib().rvo_pool_new(self.threads, kernel)
        if not self.h:
            raise RuntimeError("oracle pool creation failed")

    def close(self):
        if self.h:
            lib().rvo_pool_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def experts_q8(pool: Pool, x_expert, gate_up, down, down_scale, ids, weights, n_embd=2816, ff=704, n_experts=128,
               debug=False):
    x = np.ascontiguousarray(x_expert)
    n_tok = x.shape[0]
    used = ids.shape[1]
    out = np.zeros((n_tok, n_embd), np.float32)
    h = np.zeros((n_tok * used, ff), np.float32) if debug else None
    y = np.zeros((n_tok * used, n_embd), np.float32) if debug else None
    ds = None if down_scale is None else np.ascontiguousarray(down_scale, dtype=np.float32)
    rc = lib().rvo_experts_q8(pool.h, _p(x), _dtype_code(x), _p(np.ascontiguousarray(gate_up)),
                              _p(np.ascontiguousarray(down)), _p(ds), _p(np.ascontiguousarray(ids, dtype=np.int32)),
                              _p(np.ascontiguousarray(weights, dtype=np.float32)), n_tok, n_embd, ff, n_experts, used,
                              _p(out), _p(h), _p(y))
    if rc != 0:
        raise ValueError("oracle experts_q8 rejected its arguments")
    return (out, h, y) if debug else out


def moe_layer(pool: Pool, x_router, x_expert, w_router, gate_up, down, down_scale=None, bias=None, bias_stride=0,
              used=8, ff=704):
    """Router + selection + routed experts (exec.rs:456-475). Returns (out, ids, weights, logits)."""
    xr, xe = np.ascontiguousarray(x_router), np.ascontiguousarray(x_expert)
    if _dtype_code(xr) != _dtype_code(xe):
        raise TypeError("router and expert inputs must share a dtype")
    n_tok, n_embd = xr.shape
    ne = w_router.shape[0]
    out = np.zeros((n_tok, n_embd), np.float32)
    ids = np.zeros((n_tok, used), np.int32)
    w = np.zeros((n_tok, used), np.float32)
    lg = np.zeros((n_tok, ne), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    ds = None if down_scale is None else np.ascontiguousarray(down_scale, dtype=np.float32)
    wr = np.ascontiguousarray(w_router)
    rc = lib().rvo_moe_layer(pool.h, _p(xr), _p(xe), _dtype_code(xr), _p(wr), _dtype_code(wr), _p(b), bias_stride,
                             _p(np.ascontiguousarray(gate_up)), _p(np.ascontiguousarray(down)), _p(ds), n_tok, n_embd,
                             ff, ne, used, _p(lg), _p(ids), _p(w), _p(out))
    if rc != 0:
        raise ValueError("oracle moe_layer rejected its arguments")
    return out, ids, w, lg
