"""MoE layer session object: the B200 counterpart of the HIP executor's MoE branch.

``HipSession::new_with_experts`` uploads one layer's router and expert tensors
(runtime/src/hip_exec.rs:429-433) and ``HipSession::layer`` runs router -> selection ->
experts -> combine (:780-846). :class:`MoeLayer` does the same through librvcuda.so:
weights are uploaded once and repacked on the device (rvc_pack_experts), a workspace is
reserved up front for ``max_tok`` tokens (nothing allocates per call, as the reference's
Session::new preallocates its scratch, runtime/src/exec.rs:14-15), and each call enqueues the
fused kernels on one stream with no host synchronisation.

torch provides device memory and streams only; every arithmetic step runs in librvcuda.so.
"""
from __future__ import annotations

import numpy as np
import torch

from . import rvcuda as rc
from . import synth


def _stream_handle(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


class MoeLayer:
    def __init__(self, w_router: np.ndarray, gate_up: np.ndarray, down: np.ndarray, down_scale=None,
                 max_tok: int = 64, device: int = 0, n_embd: int = synth.N_EMBD, ff: int = synth.FF,
                 used: int = synth.USED):
        rc.lib()  # fail loudly before touching the GPU if the extension is missing
        self.device = torch.device("cuda", device)
        torch.cuda.set_device(self.device)
        self.n_embd, self.ff, self.used = n_embd, ff, used
        self.n_experts = w_router.shape[0]
        self.max_tok = max_tok
        if w_router.dtype == np.uint16:
            self.router_dtype = rc.BF16
        elif w_router.dtype == np.float32:
            self.router_dtype = rc.F32
        else:
            raise TypeError("router weights must be bf16 bits (uint16) or float32")
        dev = self.device
        self.router_w = torch.from_numpy(np.ascontiguousarray(w_router).view(np.uint8)).to(dev)
        self.down_scale = None if down_scale is None else torch.from_numpy(
            np.ascontiguousarray(down_scale, dtype=np.float32)).to(dev)
        self.packed = torch.empty(rc.packed_bytes(self.n_experts, n_embd, ff), dtype=torch.uint8, device=dev)
        gu = torch.from_numpy(np.ascontiguousarray(gate_up).reshape(-1)).to(dev)
        dn = torch.from_numpy(np.ascontiguousarray(down).reshape(-1)).to(dev)
        rc.pack_experts(gu, dn, self.n_experts, n_embd, ff, self.packed, _stream_handle(None))
        torch.cuda.current_stream().synchronize()
        del gu, dn
        self.ws = torch.empty(rc.workspace_bytes(max_tok, n_embd, ff, self.n_experts, used), dtype=torch.uint8,
                              device=dev)
        rc.workspace_reset(self.ws, _stream_handle(None))
        self.w = rc.weights_struct(n_embd, ff, self.n_experts, used, self.router_dtype, self.router_w, self.packed,
                                   self.down_scale)

    @classmethod
    def from_gguf(cls, path: str, layer: int, max_tok: int = 64, device: int = 0, n_embd: int = synth.N_EMBD,
                  ff: int = synth.FF, n_experts: int = synth.N_EXPERTS, used: int = synth.USED) -> "MoeLayer":
        """The MoE layer of block `layer` of a GGUF model file (runtime/src/model.rs:61-107 binds the
        same tensors): F32 router, Q4_0 experts packed on the device, the experts' down scales. The
        branch's norm weights are kept as `norms` (gate_inp_scale, pre_norm, post_norm: host f32)."""
        with rc.GgufFile(path) as g:
            t = g.moe_layer(layer, n_embd, ff, n_experts)
            lyr = cls(t["router"], t["gate_up"], t["down"], down_scale=t["down_scale"], max_tok=max_tok,
                      device=device, n_embd=n_embd, ff=ff, used=used)
            lyr.norms = {k: np.array(t[k]) for k in ("gate_inp_scale", "pre_norm", "post_norm")}
        return lyr

    @staticmethod
    def x_dtype(x: torch.Tensor) -> int:
        if x.dtype == torch.bfloat16:
            return rc.BF16
        if x.dtype == torch.float32:
            return rc.F32
        raise TypeError("activations must be bf16 or f32")

    def _check_tok(self, n_tok: int):
        if not 0 < n_tok <= self.max_tok:
            raise ValueError(f"{n_tok} tokens outside this layer's workspace (max {self.max_tok})")

    def forward(self, x: torch.Tensor, x_expert: torch.Tensor | None = None, out: torch.Tensor | None = None,
                ids: torch.Tensor | None = None, wts: torch.Tensor | None = None, bias: torch.Tensor | None = None,
                bias_stride: int = 0, stream=None) -> torch.Tensor:
        """Router on x, experts on x_expert (default x); returns out [n_tok, n_embd] f32."""
        n = x.shape[0]
        self._check_tok(n)
        xe = x if x_expert is None else x_expert
        if out is None:
            out = torch.empty((n, self.n_embd), dtype=torch.float32, device=self.device)
        rc.moe_forward(self.w, x, xe, self.x_dtype(x), n, out, self.ws, bias=bias, bias_stride=bias_stride, ids=ids,
                       wts=wts, stream=_stream_handle(stream))
        return out

    def router(self, x: torch.Tensor, bias: torch.Tensor | None = None, bias_stride: int = 0, stream=None):
        """(ids, wts, hist, perm, logits) device tensors."""
        n = x.shape[0]
        self._check_tok(n)
        dev = self.device
        ids = torch.empty((n, self.used), dtype=torch.int32, device=dev)
        wts = torch.empty((n, self.used), dtype=torch.float32, device=dev)
        hist = torch.empty(self.n_experts, dtype=torch.int32, device=dev)
        perm = torch.empty(n * self.used, dtype=torch.int32, device=dev)
        logits = torch.empty((n, self.n_experts), dtype=torch.float32, device=dev)
        rc.moe_router(self.w, x, self.x_dtype(x), n, self.ws, bias=bias, bias_stride=bias_stride, ids=ids, wts=wts,
                      hist=hist, perm=perm, logits=logits, stream=_stream_handle(stream))
        return ids, wts, hist, perm, logits

    def experts(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, out: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        n = x.shape[0]
        self._check_tok(n)
        if out is None:
            out = torch.empty((n, self.n_embd), dtype=torch.float32, device=self.device)
        rc.moe_experts(self.w, x, self.x_dtype(x), ids, wts, n, out, self.ws, stream=_stream_handle(stream))
        return out

    def status(self, stream=None) -> None:
        """Synchronise and raise if a device-side check fired (bounded wait, index check)."""
        rc.status(self.ws, _stream_handle(stream))


def to_device_x(x_bits: np.ndarray, device) -> torch.Tensor:
    """bf16 bit patterns (uint16) -> a bf16 CUDA tensor."""
    return torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).to(device).view(torch.bfloat16)
