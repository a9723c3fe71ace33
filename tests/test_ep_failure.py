"""Failure handling of the expert-parallel layer on CPU ranks (gloo), no GPU involved.

Ranks run EpMoeLayer steps with an EpHealth liveness check (rosevine_b200.ep_health) and a
cheap stand-in backend (the exchange logic is the product's; the compute is a row sum). Cases:

- a rank leaves between steps: the others raise PeerLost("left") at the next step, before any
  collective, within a fraction of the timeout;
- a rank stalls past the timeout: the others raise PeerLost("timeout") after the timeout, and
  the stalled rank, when it comes back, raises PeerLost ("left", or "unreachable" once the rank
  hosting the store has exited) instead of waiting on them;
- every process exits on its own within a bound (no hang), and the healthy path still runs
  steps back to back.

The failure is made on the host (a rank that returns early or sleeps), as the reference's pool
tests make a worker fail (runtime/src/expert_pool.rs, worker_panic_is_reported_and_pool_remains_
usable): nothing here can fault or hang a device.
"""
import json
import os
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rosevine_b200.ep import EpMoeLayer, pack_host
from rosevine_b200.ep_health import EpHealth, PeerLost, abort_ep_group, init_ep_group

N_EXP, USED, WIDTH, N_TOK = 12, 2, 16, 6
HEALTH_S = 2.0


class SumBackend:
    """Routes token t to experts (t + k) % N_EXP; an expert's output is its row times (1 + id)."""

    def __init__(self, rank, world):
        self.world, self.n_local, self.base = world, N_EXP // world, rank * (N_EXP // world)

    def route(self, x, bias=None):
        t = torch.arange(x.shape[0], dtype=torch.int32)[:, None]
        ids = (t + torch.arange(USED, dtype=torch.int32)[None, :]) % N_EXP
        return ids, torch.full((x.shape[0], USED), 1.0 / USED)

    def pack(self, x, ids, wts):
        return pack_host(x.contiguous().view(torch.uint8).reshape(x.shape[0], -1), ids, wts, self.world, self.n_local)

    def experts(self, rows):
        xb = WIDTH * 4
        x = rows[:, :xb].contiguous().view(torch.float32)
        e = rows[:, xb:xb + 4 * USED].contiguous().view(torch.int32)
        w = rows[:, xb + 4 * USED:xb + 8 * USED].contiguous().view(torch.float32)
        out = torch.zeros_like(x)
        for k in range(USED):
            on = e[:, k] >= 0
            out[on] += x[on] * (w[on, k] * (1.0 + (e[on, k] + self.base).float()))[:, None]
        return out

    def reduce(self, back, owner_map, n_tok):
        out = torch.zeros((n_tok, WIDTH))
        for t in range(n_tok):
            for r in range(owner_map.shape[1]):
                if owner_map[t, r] >= 0:
                    out[t] += back[owner_map[t, r]]
        return out


def _rank(rank, world, port, tmp, scenario):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    rec = {"rank": rank, "steps": 0, "error": None, "why": None, "ranks": None, "t_detect": None}
    init_ep_group("gloo", rank, world, timeout_s=20.0)
    try:
        store = dist.distributed_c10d._get_default_store()
        health = EpHealth(store, rank, world, timeout_s=HEALTH_S)
        layer = EpMoeLayer(SumBackend(rank, world), rank, world, n_experts=N_EXP, health=health)
        x = torch.arange(N_TOK * WIDTH, dtype=torch.float32).reshape(N_TOK, WIDTH) + 100 * rank
        for step in range(4):
            if scenario == "leave" and rank == world - 1 and step == 2:
                health.leave()  # between steps: nothing in flight
                break
            if scenario == "stall" and rank == 1 and step == 2:
                time.sleep(3 * HEALTH_S)
            t0 = time.monotonic()
            try:
                out = layer.forward(x)
            except PeerLost as e:
                rec.update(error="PeerLost", why=e.why, ranks=e.ranks, step=e.step, t_detect=time.monotonic() - t0)
                break
            assert torch.isfinite(out).all()
            rec["steps"] += 1
    finally:
        with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
            json.dump(rec, f)
        abort_ep_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, scenario):
    with tempfile.TemporaryDirectory() as tmp:
        t0 = time.monotonic()
        mp.spawn(_rank, args=(world, _free_port(), tmp, scenario), nprocs=world, join=True)
        wall = time.monotonic() - t0
        recs = [json.load(open(os.path.join(tmp, f"r{r}.json"))) for r in range(world)]
    return recs, wall


@pytest.mark.timeout(120)
def test_healthy_steps_run():
    recs, _ = _run(3, "none")
    assert all(r["steps"] == 4 and r["error"] is None for r in recs), recs


@pytest.mark.timeout(120)
def test_rank_leaving_between_steps_is_reported():
    recs, wall = _run(3, "leave")
    assert recs[2]["steps"] == 2 and recs[2]["error"] is None
    for r in recs[:2]:
        assert r["steps"] == 2 and r["error"] == "PeerLost" and r["why"] == "left", r
        assert 2 in r["ranks"], r
        assert r["t_detect"] < HEALTH_S, r  # the leave notice, not the timeout
    assert wall < 60


@pytest.mark.timeout(120)
def test_stalled_rank_is_reported_after_the_timeout():
    recs, wall = _run(3, "stall")
    for r in (recs[0], recs[2]):
        assert r["steps"] == 2 and r["error"] == "PeerLost" and r["why"] == "timeout", r
        assert r["ranks"] == [1], r
        # the first rank to run out of time tells the other, whose own wait started within
        # the previous step's exchange of it
        assert HEALTH_S - 0.5 <= r["t_detect"] < HEALTH_S + 5, r
    # the stalled rank comes back to peers that gave up: told (their leave notice, or the store
    # gone with rank 0), not left waiting in an all-to-all
    assert recs[1]["error"] == "PeerLost" and recs[1]["why"] in ("left", "unreachable"), recs[1]
    assert wall < 60
