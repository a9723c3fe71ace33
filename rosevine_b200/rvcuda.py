"""Safe Python wrapper over the C ABI in include/rvcuda.h (librvcuda.so).

Mirrors the reference's Rust wrapper runtime/src/hip.rs: device memory is owned by
:class:`DevBuf` (rvc_alloc / rvc_free), every range a kernel reads or writes is checked
against its owning allocation before the call (hip.rs:258-263), and a non-zero return code
becomes :class:`DeviceError` carrying the code and rvc_error_string (hip.rs:120-122,
runtime/src/error.rs:26-27).

There is no fallback: if librvcuda.so is missing or fails to load, importing the entry points
raises. Device pointers may also come from torch tensors (``tensor.data_ptr()``); torch is only
used for plumbing (allocation, streams, distributed), never for the MoE arithmetic.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librvcuda.so")

F32, BF16 = 0, 1
ERR_DEVICE_TIMEOUT, ERR_DEVICE_INDEX, ERR_UNSUPPORTED, ERR_WORKSPACE = 10001, 10002, 10003, 10004

# Every symbol include/rvcuda.h declares (checked by tests/test_abi.py).
EXPORTS = [
    "rvc_init", "rvc_mem_info", "rvc_alloc", "rvc_free", "rvc_upload", "rvc_download", "rvc_copy", "rvc_sync",
    "rvc_error_string", "rvc_event_create", "rvc_event_destroy", "rvc_event_record", "rvc_event_sync",
    "rvc_event_elapsed", "rvc_upload_async", "rvc_download_async", "rvc_event_record_on", "rvc_stream_sync",
    "rvc_packed_bytes", "rvc_pack_experts", "rvc_moe_workspace_bytes", "rvc_moe_router", "rvc_moe_experts",
    "rvc_moe_forward", "rvc_workspace_reset", "rvc_status", "rvc_debug_block_sums", "rvc_moe_forward_noalloc",
    "rvc_debug_gemm_block_dots", "rvc_q8_record_bytes", "rvc_ep_row_bytes", "rvc_quant_q8_rows", "rvc_ep_pack",
    "rvc_ep_workspace_bytes", "rvc_ep_experts", "rvc_ep_reduce", "rvc_prefill_gemms", "rvc_rms_norm",
    "rvc_gguf_open", "rvc_gguf_parse", "rvc_gguf_close", "rvc_gguf_tensor", "rvc_gguf_moe_layer",
    "rvc_q4_mm", "rvc_geglu", "rvc_shared_mlp_workspace_bytes", "rvc_shared_mlp",
]
ERR_GGUF = 10100  # + a reason (rvc_error_string gives the reference parser's wording)


class DeviceError(RuntimeError):
    def __init__(self, code: int):
        self.code = code
        super().__init__(f"rvcuda error {code}: {error_string(code)}")


class MoeWeights(ctypes.Structure):
    """rvc_moe_weights (include/rvcuda.h)."""
    _fields_ = [
        ("n_embd", ctypes.c_int),
        ("ff", ctypes.c_int),
        ("n_experts", ctypes.c_int),
        ("used", ctypes.c_int),
        ("router_dtype", ctypes.c_int),
        ("router", ctypes.c_void_p),
        ("packed", ctypes.c_void_p),
        ("down_scale", ctypes.c_void_p),
    ]


class GgufMoe(ctypes.Structure):
    """rvc_gguf_moe (include/rvcuda.h): host views of one layer's MoE tensors."""
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("gate_up", "down", "router", "down_scale", "gate_inp_scale", "pre_norm", "post_norm")]


_lib = None


def lib() -> ctypes.CDLL:
    """Load librvcuda.so (built in-tree by rosevine_b200/build.py). Raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m rosevine_b200.build` (no CPU fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        P, I, Z, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float
        W = ctypes.POINTER(MoeWeights)
        sig = {
            "rvc_init": ([I], I),
            "rvc_mem_info": ([ctypes.POINTER(Z), ctypes.POINTER(Z)], I),
            "rvc_alloc": ([Z, ctypes.POINTER(P)], I),
            "rvc_free": ([P], I),
            "rvc_upload": ([P, P, Z], I),
            "rvc_download": ([P, P, Z], I),
            "rvc_copy": ([P, P, Z], I),
            "rvc_sync": ([], I),
            "rvc_error_string": ([I], ctypes.c_char_p),
            "rvc_event_create": ([ctypes.POINTER(P)], I),
            "rvc_event_destroy": ([P], I),
            "rvc_event_record": ([P], I),
            "rvc_event_sync": ([P], I),
            "rvc_event_elapsed": ([P, P, ctypes.POINTER(F)], I),
            "rvc_upload_async": ([P, P, Z, P], I),
            "rvc_download_async": ([P, P, Z, P], I),
            "rvc_event_record_on": ([P, P], I),
            "rvc_stream_sync": ([P], I),
            "rvc_packed_bytes": ([I, I, I], Z),
            "rvc_pack_experts": ([P, P, I, I, I, P, P], I),
            "rvc_moe_workspace_bytes": ([I, I, I, I, I], Z),
            "rvc_moe_router": ([W, P, I, P, I, I, P, P, P, P, P, P, Z, P], I),
            "rvc_moe_experts": ([W, P, I, P, P, I, P, P, Z, P], I),
            "rvc_moe_forward": ([W, P, P, I, P, I, I, P, P, P, P, Z, P], I),
            "rvc_workspace_reset": ([P, P], I),
            "rvc_status": ([P, P], I),
            "rvc_rms_norm": ([P, P, P, I, I, F, F, P], I),
            "rvc_debug_block_sums": ([W, I, I, P, I, P, I, P, P], I),
            "rvc_moe_forward_noalloc": ([W, P, P, I, P, I, I, P, P, P, P], I),
            "rvc_debug_gemm_block_dots": ([W, I, I, I, P, I, P, P, Z, P], I),
            "rvc_q8_record_bytes": ([I], Z),
            "rvc_ep_row_bytes": ([I, I], Z),
            "rvc_quant_q8_rows": ([P, I, I, I, P, P], I),
            "rvc_ep_pack": ([P, P, P, I, I, I, I, I, P, P, P, P, P], I),
            "rvc_ep_workspace_bytes": ([I, I, I, I, I], Z),
            "rvc_ep_experts": ([W, P, I, I, P, P, Z, P], I),
            "rvc_ep_reduce": ([P, P, I, I, I, P, P], I),
            "rvc_prefill_gemms": ([W, P, Z, P], I),
            "rvc_gguf_open": ([ctypes.c_char_p, ctypes.POINTER(P)], I),
            "rvc_gguf_parse": ([P, Z, ctypes.POINTER(P)], I),
            "rvc_gguf_close": ([P], None),
            "rvc_gguf_tensor": ([P, ctypes.c_char_p, ctypes.POINTER(I), ctypes.POINTER(I),
                                 ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(P), ctypes.POINTER(ctypes.c_uint64)], I),
            "rvc_gguf_moe_layer": ([P, I, I, I, I, ctypes.POINTER(GgufMoe)], I),
            "rvc_q4_mm": ([P, P, P, I, I, I, P], I),
            "rvc_geglu": ([P, P, P, I, P], I),
            "rvc_shared_mlp_workspace_bytes": ([I, I, I], Z),
            "rvc_shared_mlp": ([P, P, P, P, P, P, P, I, I, I, F, P, Z, P], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, res
        _lib = L
    return _lib


def error_string(code: int) -> str:
    try:
        s = lib().rvc_error_string(code)
        return s.decode() if s else f"code {code}"
    except ImportError:
        return f"code {code}"


def check(code: int) -> None:
    if code != 0:
        raise DeviceError(code)


def init(device: int = 0) -> None:
    check(lib().rvc_init(device))


def sync() -> None:
    check(lib().rvc_sync())


# ------------------------------------------------------------------- buffers
@dataclass
class View:
    """A checked (pointer, length-in-bytes) view of device memory."""
    ptr: int
    nbytes: int

    def need(self, nbytes: int) -> int:
        if nbytes < 0 or nbytes > self.nbytes:
            raise ValueError(f"device range of {nbytes} B outside its allocation of {self.nbytes} B")
        return self.ptr


class DevBuf:
    """Owned device allocation (hip.rs DevBuf), freed on close / garbage collection."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib().rvc_alloc(nbytes, ctypes.byref(p)))
        self.ptr = p.value
        self.nbytes = nbytes

    def view(self, off: int = 0, nbytes: int | None = None) -> View:
        n = self.nbytes - off if nbytes is None else nbytes
        if off < 0 or n < 0 or off + n > self.nbytes:
            raise ValueError("device range outside its allocation")
        return View(self.ptr + off, n)

    def upload(self, host: np.ndarray, off: int = 0) -> None:
        host = np.ascontiguousarray(host)
        v = self.view(off, host.nbytes)
        check(lib().rvc_upload(v.ptr, host.ctypes.data, host.nbytes))

    def download(self, out: np.ndarray, off: int = 0) -> np.ndarray:
        assert out.flags.c_contiguous
        v = self.view(off, out.nbytes)
        check(lib().rvc_download(out.ctypes.data, v.ptr, out.nbytes))
        return out

    def close(self) -> None:
        if getattr(self, "ptr", None):
            lib().rvc_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def of(host: np.ndarray) -> "DevBuf":
        b = DevBuf(max(1, np.ascontiguousarray(host).nbytes))
        b.upload(host)
        return b


def view_of(obj, nbytes: int | None = None) -> View:
    """A View of a DevBuf, a View, a torch CUDA tensor, or None."""
    if obj is None:
        return View(0, 0)
    if isinstance(obj, View):
        return obj
    if isinstance(obj, DevBuf):
        return obj.view()
    if hasattr(obj, "data_ptr"):  # torch tensor
        if not obj.is_cuda or not obj.is_contiguous():
            raise ValueError("device tensors must be contiguous CUDA tensors")
        return View(obj.data_ptr(), obj.numel() * obj.element_size())
    raise TypeError(f"not a device buffer: {type(obj)}")


def _ptr(obj, nbytes: int) -> int | None:
    if obj is None:
        return None
    return view_of(obj).need(nbytes)


# -------------------------------------------------------------- MoE entries
def packed_bytes(n_experts: int, n_embd: int, ff: int) -> int:
    return lib().rvc_packed_bytes(n_experts, n_embd, ff)


def workspace_bytes(max_tok: int, n_embd: int, ff: int, n_experts: int, used: int) -> int:
    return lib().rvc_moe_workspace_bytes(max_tok, n_embd, ff, n_experts, used)


def pack_experts(gate_up, down, n_experts: int, n_embd: int, ff: int, packed, stream: int | None = None) -> None:
    gu_bytes = n_experts * 2 * ff * (n_embd // 32) * 18
    dn_bytes = n_experts * n_embd * (ff // 32) * 18
    check(lib().rvc_pack_experts(_ptr(gate_up, gu_bytes), _ptr(down, dn_bytes), n_experts, n_embd, ff,
                                 _ptr(packed, packed_bytes(n_experts, n_embd, ff)), stream))


def weights_struct(n_embd, ff, n_experts, used, router_dtype, router, packed, down_scale) -> MoeWeights:
    rb = 2 if router_dtype == BF16 else 4
    return MoeWeights(n_embd, ff, n_experts, used, router_dtype, _ptr(router, n_experts * n_embd * rb),
                      _ptr(packed, packed_bytes(n_experts, n_embd, ff)),
                      _ptr(down_scale, n_experts * 4) if down_scale is not None else None)


def _xbytes(x_dtype: int) -> int:
    return 2 if x_dtype == BF16 else 4


def moe_router(w: MoeWeights, x, x_dtype: int, n_tok: int, workspace, bias=None, bias_stride: int = 0, ids=None,
               wts=None, hist=None, perm=None, logits=None, stream: int | None = None) -> None:
    ws = view_of(workspace)
    bias_rows = (n_tok - 1) * bias_stride + w.n_experts if bias is not None else 0
    check(lib().rvc_moe_router(ctypes.byref(w), _ptr(x, n_tok * w.n_embd * _xbytes(x_dtype)), x_dtype,
                               _ptr(bias, bias_rows * 4), bias_stride, n_tok, _ptr(ids, n_tok * w.used * 4),
                               _ptr(wts, n_tok * w.used * 4), _ptr(hist, w.n_experts * 4),
                               _ptr(perm, n_tok * w.used * 4), _ptr(logits, n_tok * w.n_experts * 4), ws.ptr,
                               ws.nbytes, stream))


def moe_experts(w: MoeWeights, x, x_dtype: int, ids, wts, n_tok: int, out, workspace,
                stream: int | None = None) -> None:
    ws = view_of(workspace)
    check(lib().rvc_moe_experts(ctypes.byref(w), _ptr(x, n_tok * w.n_embd * _xbytes(x_dtype)), x_dtype,
                                _ptr(ids, n_tok * w.used * 4), _ptr(wts, n_tok * w.used * 4), n_tok,
                                _ptr(out, n_tok * w.n_embd * 4), ws.ptr, ws.nbytes, stream))


def moe_forward(w: MoeWeights, x_router, x_expert, x_dtype: int, n_tok: int, out, workspace, bias=None,
                bias_stride: int = 0, ids=None, wts=None, stream: int | None = None) -> None:
    ws = view_of(workspace)
    xb = n_tok * w.n_embd * _xbytes(x_dtype)
    bias_rows = (n_tok - 1) * bias_stride + w.n_experts if bias is not None else 0
    check(lib().rvc_moe_forward(ctypes.byref(w), _ptr(x_router, xb), _ptr(x_expert, xb), x_dtype,
                                _ptr(bias, bias_rows * 4), bias_stride, n_tok, _ptr(out, n_tok * w.n_embd * 4),
                                _ptr(ids, n_tok * w.used * 4), _ptr(wts, n_tok * w.used * 4), ws.ptr, ws.nbytes,
                                stream))


NOALLOC_SCRATCH_BYTES = 8 << 20


def moe_forward_noalloc(w: MoeWeights, x_router, x_expert, x_dtype: int, n_tok: int, out, bias=None,
                        bias_stride: int = 0, ids=None, wts=None, stream: int | None = None) -> None:
    """rvc_moe_forward on the library's fixed device scratch: for callers that cannot provide
    (allocate) a workspace. Up to 64 tokens at the target's shapes; calls must not overlap."""
    xb = n_tok * w.n_embd * _xbytes(x_dtype)
    bias_rows = (n_tok - 1) * bias_stride + w.n_experts if bias is not None else 0
    check(lib().rvc_moe_forward_noalloc(ctypes.byref(w), _ptr(x_router, xb), _ptr(x_expert, xb), x_dtype,
                                        _ptr(bias, bias_rows * 4), bias_stride, n_tok,
                                        _ptr(out, n_tok * w.n_embd * 4), _ptr(ids, n_tok * w.used * 4),
                                        _ptr(wts, n_tok * w.used * 4), stream))


def prefill_gemms(w: MoeWeights, workspace, stream: int | None = None) -> None:
    """Re-enqueue the grouped GEMMs of the last prefill call made with this workspace and
    these weights (rvc_prefill_gemms): for timing the layer's dominant kernels alone."""
    ws = view_of(workspace)
    check(lib().rvc_prefill_gemms(ctypes.byref(w), ws.ptr, ws.nbytes, stream))


def workspace_reset(workspace, stream: int | None = None) -> None:
    check(lib().rvc_workspace_reset(view_of(workspace).need(256), stream))


def status(workspace, stream: int | None = None) -> None:
    check(lib().rvc_status(view_of(workspace).need(256), stream))


def debug_block_sums(w: MoeWeights, which: int, expert: int, rows, n_rows: int, xq8, n_in: int, out,
                     stream: int | None = None) -> None:
    nblk = w.n_embd // 32 if which == 0 else w.ff // 32
    check(lib().rvc_debug_block_sums(ctypes.byref(w), which, expert, _ptr(rows, n_rows * 4), n_rows,
                                     _ptr(xq8, n_in * nblk * 34), n_in, _ptr(out, n_in * n_rows * nblk * 4), stream))


def debug_gemm_block_dots(w: MoeWeights, which: int, expert: int, row_tile: int, records, n: int, out, scratch,
                          stream: int | None = None) -> None:
    """int32 block dots of one prefill-GEMM tile from the production tensor-core kernel:
    out [nblk][128 positions][128 rows] int32 (rvc_debug_gemm_block_dots)."""
    k = w.n_embd if which == 0 else w.ff
    nblk = k // 32
    sv = view_of(scratch)
    check(lib().rvc_debug_gemm_block_dots(ctypes.byref(w), which, expert, row_tile, _ptr(records, n * (k // 32) * 64),
                                          n, _ptr(out, nblk * 128 * 128 * 4), sv.need(256 + nblk * 4 * ((n + 3) // 4 * 4)),
                                          sv.nbytes, stream))


def q8_record_bytes(n_embd: int) -> int:
    return lib().rvc_q8_record_bytes(n_embd)


def ep_row_bytes(n_embd: int, used: int) -> int:
    return lib().rvc_ep_row_bytes(n_embd, used)


def ep_workspace_bytes(max_rows: int, used: int, n_embd: int, ff: int, n_experts: int) -> int:
    return lib().rvc_ep_workspace_bytes(max_rows, used, n_embd, ff, n_experts)


def rms_norm(x, out, weight, rows: int, width: int, eps: float, post: float = 1.0,
             stream: int | None = None) -> None:
    """rvc_rms_norm: out [rows, width] f32 = RMS-normalised x (out may be x)."""
    nb = rows * width * 4
    check(lib().rvc_rms_norm(_ptr(x, nb), _ptr(out, nb), _ptr(weight, width * 4), rows, width, eps, post, stream))


def quant_q8_rows(x, x_dtype: int, n_rows: int, n_embd: int, records, stream: int | None = None) -> None:
    check(lib().rvc_quant_q8_rows(_ptr(x, n_rows * n_embd * _xbytes(x_dtype)), x_dtype, n_rows, n_embd,
                                  _ptr(records, n_rows * q8_record_bytes(n_embd)), stream))


def ep_pack(ids, wts, records, n_tok: int, used: int, n_embd: int, n_local: int, world: int, counts, send,
            owner_map, status, stream: int | None = None) -> None:
    rb = ep_row_bytes(n_embd, used)
    check(lib().rvc_ep_pack(_ptr(ids, n_tok * used * 4), _ptr(wts, n_tok * used * 4),
                            _ptr(records, n_tok * q8_record_bytes(n_embd)), n_tok, used, n_embd, n_local, world,
                            _ptr(counts, 2 * world * 4), _ptr(send, n_tok * world * rb),
                            _ptr(owner_map, n_tok * world * 4), _ptr(status, 4), stream))


def ep_experts(w: MoeWeights, rows, n_rows: int, used: int, partial, workspace, stream: int | None = None) -> None:
    ws = view_of(workspace)
    check(lib().rvc_ep_experts(ctypes.byref(w), _ptr(rows, n_rows * ep_row_bytes(w.n_embd, used)), n_rows, used,
                               _ptr(partial, n_rows * w.n_embd * 4), ws.ptr, ws.nbytes, stream))


def ep_reduce(back, n_back: int, owner_map, n_tok: int, world: int, n_embd: int, out,
              stream: int | None = None) -> None:
    check(lib().rvc_ep_reduce(_ptr(back, n_back * n_embd * 4), _ptr(owner_map, n_tok * world * 4), n_tok, world,
                              n_embd, _ptr(out, n_tok * n_embd * 4), stream))


def q4_mm(w, x, y, n_out: int, k: int, n_in: int, stream: int | None = None) -> None:
    """rvc_q4_mm: y [n_in][n_out] = W . x, W Q4_0 rows (GGUF layout), x [n_in][k] f32."""
    check(lib().rvc_q4_mm(_ptr(w, n_out * (k // 32) * 18), _ptr(x, n_in * k * 4), _ptr(y, n_in * n_out * 4),
                          n_out, k, n_in, stream))


def geglu(g, u, out, n: int, stream: int | None = None) -> None:
    check(lib().rvc_geglu(_ptr(g, 4 * n), _ptr(u, 4 * n), _ptr(out, 4 * n), n, stream))


def shared_mlp_workspace_bytes(max_tok: int, n_embd: int, ff: int) -> int:
    return lib().rvc_shared_mlp_workspace_bytes(max_tok, n_embd, ff)


def shared_mlp(w_gate, w_up, w_down, ffn_norm, post_norm, x, out, n_tok: int, n_embd: int, ff: int, eps: float,
               workspace, stream: int | None = None) -> None:
    """rvc_shared_mlp: the layer's dense MLP with its two norms (exec.rs:438-453)."""
    wb_gu, wb_dn = ff * (n_embd // 32) * 18, n_embd * (ff // 32) * 18
    ws = view_of(workspace)
    check(lib().rvc_shared_mlp(_ptr(w_gate, wb_gu), _ptr(w_up, wb_gu), _ptr(w_down, wb_dn), _ptr(ffn_norm, 4 * n_embd),
                               _ptr(post_norm, 4 * n_embd), _ptr(x, 4 * n_tok * n_embd), _ptr(out, 4 * n_tok * n_embd),
                               n_tok, n_embd, ff, eps, ws.ptr, ws.nbytes, stream))


class GgufFile:
    """A GGUF v3 file mapped and validated by the library (rvc_gguf_open / rvc_gguf_parse): the
    checks of the reference's parser (runtime/src/gguf.rs, Gguf::parse). Tensors are numpy views
    into the mapping, valid until close()."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        h = ctypes.c_void_p()
        if path is not None:
            check(lib().rvc_gguf_open(os.fsencode(path), ctypes.byref(h)))
            self._buf = None
        else:
            self._buf = ctypes.create_string_buffer(bytes(data), len(data)) if data else None
            check(lib().rvc_gguf_parse(self._buf, len(data) if data else 0, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib().rvc_gguf_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def tensor(self, name: str):
        """(ggml type, shape in ggml order, uint8 view of the tensor's bytes)."""
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_uint64 * 4)()
        data, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        check(lib().rvc_gguf_tensor(self._h, name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape,
                                    ctypes.byref(data), ctypes.byref(nbytes)))
        return dt.value, tuple(shape[:nd.value]), _host_view(data.value, nbytes.value)

    def moe_layer(self, layer: int, n_embd: int, ff: int, n_experts: int) -> dict:
        """Views of one layer's MoE tensors, shapes and types checked (rvc_gguf_moe_layer)."""
        m = GgufMoe()
        check(lib().rvc_gguf_moe_layer(self._h, layer, n_embd, ff, n_experts, ctypes.byref(m)))
        nb, nh = n_embd // 32, ff // 32
        f32 = lambda p, n: _host_view(p, 4 * n).view(np.float32)  # noqa: E731
        return {
            "gate_up": _host_view(m.gate_up, n_experts * 2 * ff * nb * 18).reshape(n_experts, 2 * ff, nb * 18),
            "down": _host_view(m.down, n_experts * n_embd * nh * 18).reshape(n_experts, n_embd, nh * 18),
            "router": f32(m.router, n_experts * n_embd).reshape(n_experts, n_embd),
            "down_scale": f32(m.down_scale, n_experts),
            "gate_inp_scale": f32(m.gate_inp_scale, n_embd),
            "pre_norm": f32(m.pre_norm, n_embd),
            "post_norm": f32(m.post_norm, n_embd),
        }


def _host_view(ptr: int, nbytes: int) -> np.ndarray:
    if nbytes == 0:
        return np.zeros(0, np.uint8)
    return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(ptr))
