"""GPU parity of the prefill path (batches above 16 tokens: the grouped expert GEMMs).

The first test checks one tensor-core tile (the tcgen05.mma kind::i8 debug kernel, through the
shared-memory layouts and tensor-memory reads) against numpy's int32 product. The layer tests
compare rvc_moe_forward with the oracle's scalar kernel: the router runs in the reference's
order, the int32 block dots come from the tensor cores (mma.sync) exactly, and the epilogue
accumulates them in the scalar reference's order with separately rounded operations, so ids,
weights and the output are bit-identical.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [16, 48, 128])
def test_tensor_core_tile_exact(n):
    from rosevine_b200 import rvcuda as rc
    rng = np.random.default_rng(n)
    a = rng.integers(-128, 128, size=(128, 32), dtype=np.int8)
    b = rng.integers(-128, 128, size=(n, 32), dtype=np.int8)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    d = torch.zeros((128, n), dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc.debug_mma_i8(da, db, n, d, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = a.astype(np.int32) @ b.astype(np.int32).T
    assert np.array_equal(d.cpu().numpy(), want)


@pytest.fixture(scope="module")
def weights():
    from rosevine_b200 import synth
    gu, dn = synth.experts(2)
    return {"gate_up": gu, "down": dn, "w_router": synth.router(1)}


@pytest.fixture(scope="module")
def layer(weights):
    from rosevine_b200.moe import MoeLayer
    return MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=2048)


@pytest.mark.parametrize("n_tok", [65, 200])
def test_prefill_layer_bit_exact(layer, weights, oracle, pool, n_tok):
    from rosevine_b200 import synth
    from rosevine_b200.moe import to_device_x
    x = synth.tokens(n_tok, 700 + n_tok)
    ids = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
    wts = torch.empty((n_tok, 8), dtype=torch.float32, device="cuda")
    out = layer.forward(to_device_x(x, "cuda"), ids=ids, wts=wts)
    layer.status()
    want, want_ids, want_w, _ = oracle.moe_layer(pool, x, x, weights["w_router"], weights["gate_up"], weights["down"])
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"max abs diff {np.abs(got - want).max():.3e}"


def test_prefill_f32_inputs_bit_exact(layer, weights, oracle, pool):
    """f32 activations (the reference model's own format) through the f32 loads of the router
    chains and of the quantisation kernel."""
    from rosevine_b200 import synth
    n_tok = 100
    x = synth.rms_normalise(np.random.default_rng(901).standard_normal((n_tok, 2816)).astype(np.float32))
    ids = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
    out = layer.forward(torch.from_numpy(x).cuda(), ids=ids)
    layer.status()
    want, want_ids, _, _ = oracle.moe_layer(pool, x, x, weights["w_router"], weights["gate_up"], weights["down"])
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"max abs diff {np.abs(got - want).max():.3e}"


def test_prefill_zipf_groups(weights, oracle, pool):
    """2048 tokens, router logits biased per expert by Zipf(1.1) weights, so the
    expert groups run from empty to several hundred tokens (tiles that end mid-group, experts
    with no tokens, groups larger than one 128-token tile)."""
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer, to_device_x
    n_tok = 2048
    lyr = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], down_scale=synth.down_scales(3),
                   max_tok=n_tok)
    x = synth.tokens(n_tok, 2024)
    bias = synth.zipf_bias(5)
    out = lyr.forward(to_device_x(x, "cuda"), bias=torch.from_numpy(bias).cuda())
    lyr.status()
    want, want_ids, _, _ = oracle.moe_layer(pool, x, x, weights["w_router"], weights["gate_up"], weights["down"],
                                            bias=bias, down_scale=synth.down_scales(3))
    counts = np.bincount(want_ids.ravel(), minlength=128)
    assert counts.max() > 128  # some group spans more than one 128-token tile
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"max abs diff {np.abs(got - want).max():.3e}"


def test_prefill_gemms_rerun_leaves_workspace_unchanged(weights):
    """rvc_prefill_gemms re-runs the last prefill call's grouped GEMMs on its plan and records
    (bench.py times them this way): they rewrite the same h records, scales and y, so the whole
    workspace is byte-identical afterwards; a workspace without such a call, or reset since, is
    refused."""
    from rosevine_b200 import rvcuda as rc
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer, to_device_x
    lyr = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=300)
    with pytest.raises(rc.DeviceError):
        rc.prefill_gemms(lyr.w, lyr.ws)
    lyr.forward(to_device_x(synth.tokens(300, 1300), "cuda"))
    torch.cuda.synchronize()
    before = lyr.ws.clone()
    rc.prefill_gemms(lyr.w, lyr.ws)
    rc.prefill_gemms(lyr.w, lyr.ws)
    torch.cuda.synchronize()
    assert torch.equal(lyr.ws, before)
    lyr.status()
    rc.workspace_reset(lyr.ws)  # any other use of the workspace ends what may be re-run on it
    with pytest.raises(rc.DeviceError):
        rc.prefill_gemms(lyr.w, lyr.ws)
