"""Expert-parallel layer on GPUs: the CUDA library's EP entry points over NCCL.

With one rank every token goes to rank 0 with all its slots, so the partial is the slot-order
sum and the layer output is bit-identical to the single-device reference path. With two or more
ranks (skipped on a one-GPU box) the owner adds per-rank partials in rank order: ids bit-exact,
output within the EP tolerance. The hot-expert case routes 90% of the tokens to experts 0..7,
all on rank 0.
"""
import os
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu

EP_RTOL = 1e-3


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bias(n_tok, hot):
    from rosevine_b200 import synth
    if not hot:
        return None
    b = np.zeros((n_tok, synth.N_EXPERTS), np.float32)
    b[: int(0.9 * n_tok), :8] = 50.0
    return b


def _rank(rank, world, port, tmp, n_tok, hot):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from rosevine_b200 import synth
        from rosevine_b200.ep import EpMoeLayer, GpuBackend, local_experts
        from rosevine_b200.moe import to_device_x
        gu, dn = synth.experts(2)
        wr = synth.router(1)
        x = synth.tokens(n_tok, 9)
        n = n_tok // world
        gl, dl = local_experts(gu, dn, rank, world)
        be = GpuBackend(wr, gl, dl, synth.N_EXPERTS // world, max_tok=n, max_rows=n_tok, world=world)
        layer = EpMoeLayer(be, rank, world)
        b = _bias(n_tok, hot)
        bias = None if b is None else torch.from_numpy(b[rank * n:(rank + 1) * n].copy()).cuda()
        out = layer.forward(to_device_x(x[rank * n:(rank + 1) * n], "cuda"), bias)
        be.status()
        np.save(os.path.join(tmp, f"out{rank}.npy"), out.cpu().numpy())
        np.save(os.path.join(tmp, f"ids{rank}.npy"), layer.last_ids.cpu().numpy())
    finally:
        dist.destroy_process_group()


def _run(world, n_tok, hot):
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_rank, args=(world, _free_port(), tmp, n_tok, hot), nprocs=world, join=True)
        got = np.concatenate([np.load(os.path.join(tmp, f"out{r}.npy")) for r in range(world)])
        ids = np.concatenate([np.load(os.path.join(tmp, f"ids{r}.npy")) for r in range(world)])
    return got, ids


def _want(oracle, pool, n_tok, hot):
    from rosevine_b200 import synth
    gu, dn = synth.experts(2)
    x = synth.tokens(n_tok, 9)
    b = _bias(n_tok, hot)
    want, want_ids, _, _ = oracle.moe_layer(pool, x, x, synth.router(1), gu, dn, bias=b,
                                            bias_stride=synth.N_EXPERTS if hot else 0)
    return want, want_ids


def test_ep_single_rank_bit_exact(oracle, pool):
    got, ids = _run(1, 96, False)
    want, want_ids = _want(oracle, pool, 96, False)
    assert np.array_equal(ids, want_ids)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"max abs {np.abs(got - want).max():.3e}"


@pytest.mark.parametrize("hot", [False, True])
def test_ep_multi_rank(oracle, pool, hot):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    while synth_experts() % world:
        world -= 1
    n_tok = 64 * world
    got, ids = _run(world, n_tok, hot)
    want, want_ids = _want(oracle, pool, n_tok, hot)
    assert np.array_equal(ids, want_ids)
    # per row, as the north star's bar: max |gpu - cpu| over the row / max |cpu| over the row
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() <= EP_RTOL, f"max row rel err {err.max():.3e} (row {int(err.argmax())})"


def synth_experts():
    from rosevine_b200 import synth
    return synth.N_EXPERTS
