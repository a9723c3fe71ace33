"""Expert-parallel exchange logic on CPU ranks (gloo), with the oracle as the compute.

Each rank holds n_experts / world experts and a shard of the tokens; EpMoeLayer routes, plans
the dispatch (each token sent once per rank holding one of its experts, its slots there in slot
order), exchanges rows, runs the resident experts and returns per-rank partial sums that the
owner adds in rank order. The oracle backend stands in for the CUDA library, so this checks the
plan, the splits, the metadata and the reduction order; the GPU tests run the same layer on the
CUDA library over NCCL. Outputs match the single-device oracle within the EP tolerance (the
partials are summed in rank order, not slot order).
"""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rosevine_b200 import synth
from rosevine_b200.ep import EpMoeLayer, pack_host, plan_dispatch

N_TOK = 24
EP_RTOL = 1e-3


class OracleBackend:
    """Compute on the host through the oracle: a sent row is the token's raw bf16 bits followed by
    its slot metadata (pack_host, the same row layout rvc_ep_pack writes after a Q8_0 record)."""

    def __init__(self, oracle, pool, w_router, gate_up, down, rank, world, n_local):
        self.O, self.pool, self.wr, self.gu, self.dn = oracle, pool, w_router, gate_up, down
        self.base, self.world, self.n_local = rank * n_local, world, n_local
        self.xb = synth.N_EMBD * 2

    def route(self, x, bias=None):
        b = None if bias is None else bias.numpy()
        lg = self.O.router_logits(x.numpy().view(np.uint16), self.wr, bias=b,
                                  bias_stride=(self.wr.shape[0] if b is not None and b.ndim == 2 else 0))
        ids, w, _ = self.O.select_experts(lg, synth.USED)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def pack(self, x, ids, wts):
        rec = x.contiguous().view(torch.uint8).reshape(x.shape[0], -1)
        return pack_host(rec, ids, wts, self.world, self.n_local)

    def experts(self, rows):
        used = synth.USED
        r = rows.numpy()
        x = np.ascontiguousarray(r[:, :self.xb]).view(np.uint16)
        e = np.ascontiguousarray(r[:, self.xb:self.xb + 4 * used]).view(np.int32)
        w = np.ascontiguousarray(r[:, self.xb + 4 * used:self.xb + 8 * used]).view(np.float32)
        out = np.zeros((x.shape[0], synth.N_EMBD), np.float32)
        for i in range(x.shape[0]):
            k = e[i] >= 0
            if k.any():
                out[i] = self.O.experts_q8(self.pool, x[i:i + 1], self.gu, self.dn, None,
                                           (e[i][k] + self.base)[None, :], w[i][k][None, :])[0]
        return torch.from_numpy(out)

    def reduce(self, back, owner_map, n_tok):
        out = torch.zeros((n_tok, back.shape[1] if back.dim() == 2 else synth.N_EMBD), dtype=torch.float32)
        om = owner_map.numpy()
        for t in range(n_tok):
            acc = None
            for r in range(om.shape[1]):
                if om[t, r] >= 0:
                    v = back[om[t, r]]
                    acc = v.clone() if acc is None else acc + v
            if acc is not None:
                out[t] = acc
        return out


def _rank(rank, world, port, tmp, hot):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        O.build()
        pool = O.Pool(threads=2, kernel=O.KERNEL_SCALAR)
        gu, dn = synth.experts(2)
        wr = synth.router(1)
        x = synth.tokens(N_TOK, 5)
        n = N_TOK // world
        mine = torch.from_numpy(x[rank * n:(rank + 1) * n].view(np.int16))
        be = OracleBackend(O, pool, wr, gu, dn, rank, world, synth.N_EXPERTS // world)
        layer = EpMoeLayer(be, rank, world)
        bias = None
        if hot:  # 90% of the tokens pick experts 0..7, all on rank 0
            b = np.zeros((N_TOK, synth.N_EXPERTS), np.float32)
            b[: int(0.9 * N_TOK), :8] = 50.0
            bias = torch.from_numpy(b[rank * n:(rank + 1) * n].copy())
        out = layer.forward(mine, bias)
        np.save(os.path.join(tmp, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(tmp, f"ids{rank}.npy"), layer.last_ids.numpy())
        pool.close()
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,hot", [(2, False), (4, False), (2, True)])
def test_ep_matches_single_device(oracle, pool, world, hot):
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_rank, args=(world, _free_port(), tmp, hot), nprocs=world, join=True)
        got = np.concatenate([np.load(os.path.join(tmp, f"out{r}.npy")) for r in range(world)])
        ids = np.concatenate([np.load(os.path.join(tmp, f"ids{r}.npy")) for r in range(world)])
    gu, dn = synth.experts(2)
    wr = synth.router(1)
    x = synth.tokens(N_TOK, 5)
    bias = None
    if hot:
        bias = np.zeros((N_TOK, synth.N_EXPERTS), np.float32)
        bias[: int(0.9 * N_TOK), :8] = 50.0
    want, want_ids, _, _ = oracle.moe_layer(pool, x, x, wr, gu, dn, bias=bias,
                                            bias_stride=synth.N_EXPERTS if hot else 0)
    assert np.array_equal(ids, want_ids)
    # per row: max |got - want| over the row / max |want| over the row
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() <= EP_RTOL, err.max()
    if hot:
        assert (ids[: int(0.9 * N_TOK)] < 8).all()


def test_plan_dispatch_dedups_and_keeps_slot_order():
    ids = torch.tensor([[0, 5, 1, 9], [12, 13, 2, 3]], dtype=torch.int32)  # 4 experts per rank, 4 ranks
    wts = torch.tensor([[0.4, 0.3, 0.2, 0.1], [0.25, 0.25, 0.25, 0.25]])
    p = plan_dispatch(ids, wts, world=4, n_local=4)
    # token 0 -> ranks 0 (slots 0, 2), 1 (slot 1), 2 (slot 3); token 1 -> ranks 0 (slots 2, 3), 3 (slots 0, 1)
    assert p.send_counts == [2, 1, 1, 1]
    assert p.send_tok.tolist() == [0, 1, 0, 0, 1]
    assert p.meta_e[0].tolist() == [0, -1, 1, -1]
    assert p.meta_e[1].tolist() == [-1, -1, 2, 3]
    assert p.meta_e[4].tolist() == [0, 1, -1, -1]
    assert p.meta_w[0].tolist() == pytest.approx([0.4, 0.0, 0.2, 0.0])


def test_pack_host_rows_and_owner_map():
    ids = torch.tensor([[0, 5, 1, 9], [12, 13, 2, 3]], dtype=torch.int32)
    wts = torch.tensor([[0.4, 0.3, 0.2, 0.1], [0.25, 0.25, 0.25, 0.25]])
    rec = torch.arange(2 * 16, dtype=torch.uint8).reshape(2, 16)
    rows, counts, owner = pack_host(rec, ids, wts, world=4, n_local=4)
    assert counts == [2, 1, 1, 1]
    assert rows.shape == (5, 16 + 4 * 8)
    assert owner.tolist() == [[0, 2, 3, -1], [1, -1, -1, 4]]
    assert torch.equal(rows[1, :16], rec[1])
    assert rows[1, 16:32].view(torch.int32).tolist() == [-1, -1, 2, 3]
