"""Expert-parallel MoE layer: experts sharded 128/N per GPU, tokens exchanged by all-to-allv.

The reference runs every expert on one device (runtime/src/hip_exec.rs:820-843); this module is
the multi-GPU form of the same layer. Rank r of N holds experts [r E/N, (r + 1) E/N) and starts
with its own shard of the tokens. One forward:

  1. route     the rank's tokens with the full router (reference order: rvc_moe_router),
  2. pack      the Q8_0 records, quantised once (rvc_quant_q8_rows), into one row per (token,
               destination rank holding one of its experts), each row carrying the token's
               slots there in slot order (rvc_ep_pack),
  3. dispatch  row counts (all-to-all), then the rows (one all-to-allv over NCCL),
  4. experts   the resident experts over the received rows (rvc_ep_experts): one partial sum
               per row, over its slots in slot order,
  5. combine   partials back to their owners (all-to-allv), summed per token in rank order
               (rvc_ep_reduce).

Each (token, expert) output is bit-identical to the single-device path; the owner adds the
per-rank partials, so the f32 summation order differs from the reference's slot order and the
layer output matches within the 1e-3 tolerance, not bitwise.

The collectives are torch.distributed calls (NCCL on GPUs); the compute steps go through a
backend object. `GpuBackend` (the product) calls the CUDA library; the tests substitute a
CPU backend built on the oracle to check the exchange logic over gloo.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import rvcuda as rc
from . import synth
from .moe import _stream_handle


@dataclass
class EpStats:
    """Device time of the last forward's exchanges, in ms (CUDA events; 0 on CPU)."""
    dispatch_ms: float = 0.0
    combine_ms: float = 0.0
    rows_sent: int = 0
    rows_received: int = 0
    phases_ms: dict | None = None  # device time of each phase of the last forward


class GpuBackend:
    """The CUDA library on this rank's device: full router, resident experts."""

    def __init__(self, w_router: np.ndarray, gate_up_local: np.ndarray, down_local: np.ndarray, n_local: int,
                 max_tok: int, max_rows: int, world: int, down_scale_local=None, device: int | None = None,
                 n_embd: int = synth.N_EMBD, ff: int = synth.FF, used: int = synth.USED):
        rc.lib()  # fail loudly before touching the GPU if the extension is missing
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.device, self.n_embd, self.ff, self.used, self.world = dev, n_embd, ff, used, world
        self.n_experts = w_router.shape[0]
        self.router_dtype = rc.BF16 if w_router.dtype == np.uint16 else rc.F32
        self.router_w = torch.from_numpy(np.ascontiguousarray(w_router).view(np.uint8)).to(dev)
        self.down_scale = None if down_scale_local is None else torch.from_numpy(
            np.ascontiguousarray(down_scale_local, dtype=np.float32)).to(dev)
        self.packed = torch.empty(rc.packed_bytes(n_local, n_embd, ff), dtype=torch.uint8, device=dev)
        gu = torch.from_numpy(np.ascontiguousarray(gate_up_local).reshape(-1)).to(dev)
        dn = torch.from_numpy(np.ascontiguousarray(down_local).reshape(-1)).to(dev)
        rc.pack_experts(gu, dn, n_local, n_embd, ff, self.packed, _stream_handle(None))
        torch.cuda.current_stream().synchronize()
        del gu, dn
        # routing uses the full router (n_experts); rvc_moe_router reads only the router rows, so
        # its weights struct points at the resident experts' planes without covering all experts
        self.w_route = rc.MoeWeights(n_embd, ff, self.n_experts, used, self.router_dtype,
                                     rc.view_of(self.router_w).need(self.n_experts * n_embd * (2 if self.router_dtype
                                                                                                == rc.BF16 else 4)),
                                     self.packed.data_ptr(), None)
        self.w_local = rc.weights_struct(n_embd, ff, n_local, min(used, n_local), self.router_dtype, self.router_w,
                                         self.packed, self.down_scale)
        self.n_local, self.max_tok, self.max_rows = n_local, max_tok, max_rows
        self.ws_route = torch.empty(rc.workspace_bytes(max_tok, n_embd, ff, self.n_experts, used), dtype=torch.uint8,
                                    device=dev)
        rc.workspace_reset(self.ws_route, _stream_handle(None))
        self.ws_ep = torch.empty(rc.ep_workspace_bytes(max_rows, used, n_embd, ff, n_local), dtype=torch.uint8,
                                 device=dev)
        rc.workspace_reset(self.ws_ep, _stream_handle(None))
        self.row_bytes = rc.ep_row_bytes(n_embd, used)
        # per-forward buffers, allocated once
        self.rec = torch.empty((max_tok, rc.q8_record_bytes(n_embd)), dtype=torch.uint8, device=dev)
        self.send = torch.empty((max_tok * world, self.row_bytes), dtype=torch.uint8, device=dev)
        self.counts = torch.empty(2 * world, dtype=torch.int32, device=dev)
        self.owner = torch.empty((max_tok, world), dtype=torch.int32, device=dev)
        self.status_ws = self.ws_ep  # the pack kernel reports bad ids in the EP workspace's status word

    def route(self, x: torch.Tensor, bias: torch.Tensor | None = None):
        """ids, wts [n, used]; bias: per-expert logit offsets [n_experts] or [n, n_experts]."""
        n = x.shape[0]
        ids = torch.empty((n, self.used), dtype=torch.int32, device=self.device)
        wts = torch.empty((n, self.used), dtype=torch.float32, device=self.device)
        stride = self.n_experts if bias is not None and bias.dim() == 2 else 0
        rc.moe_router(self.w_route, x, _xdtype(x), n, self.ws_route, bias=bias, bias_stride=stride, ids=ids, wts=wts,
                      stream=_stream_handle(None))
        return ids, wts

    def pack(self, x: torch.Tensor, ids, wts):
        """Rows to send grouped by destination rank, their counts (host list) and the owner map."""
        n = x.shape[0]
        if n > self.max_tok:
            raise ValueError(f"{n} tokens exceed the layer's {self.max_tok}")
        sh = _stream_handle(None)
        rc.quant_q8_rows(x, _xdtype(x), n, self.n_embd, self.rec, sh)
        rc.ep_pack(ids, wts, self.rec, n, self.used, self.n_embd, self.n_local, self.world, self.counts, self.send,
                   self.owner, self.status_ws, sh)
        # the row counts stay on the device: the layer reads them from the host once, together
        # with the counts it receives
        return self.send, self.counts[:self.world], self.owner[:n]

    def experts(self, rows) -> torch.Tensor:
        n_rows = rows.shape[0]
        if n_rows > self.max_rows:
            raise ValueError(f"{n_rows} rows exceed the workspace's {self.max_rows}")
        partial = torch.empty((n_rows, self.n_embd), dtype=torch.float32, device=self.device)
        rc.ep_experts(self.w_local, rows, n_rows, self.used, partial, self.ws_ep, _stream_handle(None))
        return partial

    def reduce(self, back, owner_map, n_tok: int) -> torch.Tensor:
        out = torch.empty((n_tok, self.n_embd), dtype=torch.float32, device=self.device)
        rc.ep_reduce(back if back.shape[0] else None, back.shape[0], owner_map, n_tok, self.world, self.n_embd, out,
                     _stream_handle(None))
        return out

    def status(self) -> None:
        rc.status(self.ws_route, _stream_handle(None))
        rc.status(self.ws_ep, _stream_handle(None))


def _xdtype(x: torch.Tensor) -> int:
    if x.dtype == torch.bfloat16:
        return rc.BF16
    if x.dtype == torch.float32:
        return rc.F32
    raise TypeError("activations must be bf16 or f32")


@dataclass
class _Plan:
    send_tok: torch.Tensor    # [S] int64: owner-local token of each sent row, grouped by destination rank
    send_counts: list         # rows per destination rank
    meta_e: torch.Tensor      # [S, used] int32: the row's experts at the destination (local ids), -1 if none
    meta_w: torch.Tensor      # [S, used] f32: their routing weights


def plan_dispatch(ids: torch.Tensor, wts: torch.Tensor, world: int, n_local: int) -> _Plan:
    """Rows to send: token t goes once to every rank holding one of its experts; its slots there
    keep the token's slot order (absent slots -1)."""
    n, used = ids.shape
    dest = (ids // n_local).to(torch.int64)                                  # [n, used]
    hit = torch.zeros((n, world), dtype=torch.bool, device=ids.device)
    hit.scatter_(1, dest, True)
    # rows grouped by destination rank, tokens ascending within a rank
    r_idx, t_idx = torch.nonzero(hit.t(), as_tuple=True)
    counts = torch.bincount(r_idx, minlength=world)
    sel = dest[t_idx] == r_idx[:, None]                                      # [S, used]
    meta_e = torch.where(sel, (ids[t_idx] - (r_idx[:, None] * n_local).to(ids.dtype)), torch.full_like(ids[t_idx], -1))
    meta_w = torch.where(sel, wts[t_idx], torch.zeros_like(wts[t_idx]))
    return _Plan(t_idx, counts.tolist(), meta_e.to(torch.int32).contiguous(), meta_w.contiguous())


def pack_host(rec: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, world: int, n_local: int):
    """rvc_ep_pack's rows with torch operations (any device): per sent row the record bytes, then
    the slot metadata (int32 local expert ids, -1 when elsewhere; f32 weights). Returns the rows
    grouped by destination rank, the counts per rank and the owner map [n, world] (row or -1);
    used by backends without the CUDA library (the CPU tests)."""
    p = plan_dispatch(ids, wts, world, n_local)
    meta = torch.cat([p.meta_e.view(torch.uint8).reshape(p.meta_e.shape[0], -1),
                      p.meta_w.view(torch.uint8).reshape(p.meta_w.shape[0], -1)], dim=1)
    rows = torch.cat([rec.index_select(0, p.send_tok), meta], dim=1)
    owner = torch.full((ids.shape[0], world), -1, dtype=torch.int32, device=ids.device)
    r_idx = torch.repeat_interleave(torch.arange(world, device=ids.device), torch.tensor(p.send_counts, device=ids.device))
    owner[p.send_tok, r_idx] = torch.arange(p.send_tok.shape[0], dtype=torch.int32, device=ids.device)
    return rows, p.send_counts, owner


class EpMoeLayer:
    """One rank of the expert-parallel layer. `backend` does the compute on this rank's device;
    `group` is the process group of the N ranks (rank r holds experts [r E/N, (r + 1) E/N)).
    With timing=True each forward records CUDA events between its phases (no synchronisation);
    phase_times() reads them once the caller has synchronised. With `health` (an
    ep_health.EpHealth) every forward first checks, on the host, that all peers reached the same
    step, and raises ep_health.PeerLost instead of entering an exchange a lost peer would stall."""

    def __init__(self, backend, rank: int, world: int, n_experts: int = synth.N_EXPERTS, group=None,
                 timing: bool = False, health=None):
        if n_experts % world:
            raise ValueError("experts must divide evenly over the ranks")
        self.be, self.rank, self.world, self.group = backend, rank, world, group
        self.n_local = n_experts // world
        self.timing = timing
        self.health, self.step = health, 0
        self.marks = []
        self.stats = EpStats()

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's tokens x [n, n_embd] (bf16 or f32) -> their layer output [n, n_embd] f32.
        bias: router logit offsets, [n_experts] or [n, n_experts] (the skewed-load configs).
        One host synchronisation: the row counts (sent and received) are read together."""
        be = self.be
        dev = x.device
        marks = []
        if self.health is not None:
            self.health.begin_step(self.step)  # raises PeerLost before any collective of this step
        self.step += 1

        def mark(name):  # device timestamps between the phases (CUDA, timing=True only)
            if self.timing and dev.type == "cuda":
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append((name, e))

        mark("start")
        ids, wts = be.route(x, bias)
        self.last_ids = ids
        mark("route")
        send, counts, owner_map = be.pack(x, ids, wts)
        mark("pack")
        # dispatch: row counts, then the rows (records with their slot metadata)
        sc = torch.as_tensor(counts, device=dev).to(torch.int64)
        rcnt = torch.empty_like(sc)
        self._a2a(rcnt, sc, None, None)
        both = torch.cat([sc, rcnt]).tolist()  # the step's one host read
        send_counts, recv_counts = both[:self.world], both[self.world:]
        send = send[:sum(send_counts)]
        recv = torch.empty((int(sum(recv_counts)), send.shape[1]), dtype=send.dtype, device=dev)
        self._a2a(recv, send, recv_counts, send_counts)
        mark("dispatch")
        partial = be.experts(recv)
        back = torch.empty((send.shape[0], partial.shape[1]), dtype=partial.dtype, device=dev)
        mark("experts")
        self._a2a(back, partial, send_counts, recv_counts)  # partials back to their owners
        mark("combine")
        out = be.reduce(back, owner_map, x.shape[0])
        mark("reduce")
        self.marks = marks
        self.stats = EpStats(rows_sent=int(send.shape[0]), rows_received=int(recv.shape[0]))
        return out

    def phase_times(self) -> EpStats:
        """Device time of each phase of the last forward (timing=True; the caller has synchronised)."""
        st = self.stats
        if self.marks:
            st.phases_ms = {n1: e0.elapsed_time(e1) for (_, e0), (n1, e1) in zip(self.marks, self.marks[1:])}
            st.dispatch_ms, st.combine_ms = st.phases_ms["dispatch"], st.phases_ms["combine"]
        return st


def local_experts(gate_up: np.ndarray, down: np.ndarray, rank: int, world: int):
    """This rank's slices of the expert tensors (reference layout, one expert per leading index)."""
    n = gate_up.shape[0] // world
    return gate_up[rank * n:(rank + 1) * n], down[rank * n:(rank + 1) * n]
