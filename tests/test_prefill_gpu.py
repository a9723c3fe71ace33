"""GPU parity of the prefill path (batches above 64 tokens: the grouped expert GEMMs).

The grouped GEMM (k_pf_gemm_tc) forms each 32-column block's integer dot on the tensor cores
(tcgen05.mma into tensor memory, the integer operands held exactly as f16, f32 accumulation exact
for these integers) and scales and accumulates the dots on the CUDA cores in the scalar
reference's order, each operation rounded where the reference rounds it
(expert_kernel.rs:147-161). The first tests read the block dots of one tile straight from the
production kernel (its debug mode writes them instead of scaling them) and compare them with the
exact integer dots; the layer tests compare rvc_moe_forward with the oracle's scalar kernel:
ids, weights and the output are bit-identical.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _records(xq: np.ndarray) -> np.ndarray:
    """Reference Q8_0 rows (34-byte blocks: f16 d, 32 int8) -> the prefill GEMM's activation
    operand rows: each block's 32 quants as f16 integers (exact), 64 bytes per block."""
    n, nb = xq.shape[0], xq.shape[1] // 34
    q = xq.reshape(n, nb, 34)[:, :, 2:].copy().view(np.int8)
    return np.ascontiguousarray(q.astype(np.float16).reshape(n, nb * 32)).view(np.uint8)


def _block_dots_want(mat: np.ndarray, xq: np.ndarray) -> np.ndarray:
    """Exact int32 block dots [nblk][n][rows] of Q4_0 rows mat [rows][nblk*18] with Q8_0 rows."""
    rows, n = mat.shape[0], xq.shape[0]
    nb = mat.shape[1] // 18
    nib = mat.reshape(rows, nb, 18)[:, :, 2:]
    w = np.concatenate([(nib & 15).astype(np.int64) - 8, (nib >> 4).astype(np.int64) - 8], axis=2)  # [r][b][32]
    x = xq.reshape(n, nb, 34)[:, :, 2:].view(np.int8).astype(np.int64)                               # [n][b][32]
    return np.einsum("rbk,nbk->bnr", w, x).astype(np.int32)


@pytest.mark.parametrize("which,expert,row_tile,n,extreme", [(0, 3, 0, 128, False), (0, 77, 10, 37, True),
                                                             (1, 5, 21, 128, False), (1, 127, 7, 64, True)])
def test_gemm_block_dots_bit_exact(layer, weights, oracle, which, expert, row_tile, n, extreme):
    """The production GEMM's int32 block dots for one tile (row_tile: 128 packed rows; gate_up
    rows interleave gate and up per 32) against the exact integer dots, pinned to the oracle's
    block_sumi on a sample. Extreme: every quant +-127, the largest |dot| the formats allow."""
    from rosevine_b200 import rvcuda as rc
    rng = np.random.default_rng(100 * which + expert)
    k = layer.n_embd if which == 0 else layer.ff
    nb = k // 32
    if extreme:
        xq = np.zeros((n, nb * 34), np.uint8)
        for t in range(n):
            for b in range(nb):
                xq[t, 34 * b:34 * b + 2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
                xq[t, 34 * b + 2:34 * b + 34] = 0x81 if (t + b) % 2 else 0x7F
    else:
        xq = oracle.quantize_q8_0(rng.standard_normal((n, k)).astype(np.float32))
    src = weights["gate_up"] if which == 0 else weights["down"]
    rows_total = 2 * layer.ff if which == 0 else layer.n_embd
    mat = src[expert].reshape(rows_total, nb * 18)
    packed = np.arange(row_tile * 128, row_tile * 128 + 128)
    if which == 0:  # packed row R = q 64 + s 32 + i holds original row s ff + q 32 + i
        orig = (packed % 64 // 32) * layer.ff + (packed // 64) * 32 + packed % 32
    else:
        orig = packed
    want = _block_dots_want(mat[orig], xq)
    for b, t, r in [(0, 0, 0), (nb - 1, n - 1, 127), (nb // 2, n // 2, 64)]:
        assert want[b, t, r] == oracle.block_sumi(mat[orig[r], 18 * b:18 * b + 18], xq[t, 34 * b:34 * b + 34])
    rec = torch.from_numpy(_records(xq)).cuda()
    out = torch.full((nb, 128, 128), -1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(256 + nb * 4 * 128, dtype=torch.uint8, device="cuda")
    rc.debug_gemm_block_dots(layer.w, which, expert, row_tile, rec, n, out, scratch)
    torch.cuda.synchronize()
    assert int(scratch[12:16].view(torch.int32).item()) == 0, "device status set"
    got = out.cpu().numpy()
    assert np.array_equal(got[:, :n, :], want)
    end = (n + 31) // 32 * 32  # the rest of the last loaded 32-position chunk: zero-filled operands
    assert not got[:, n:end, :].any()


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


def test_prefill_gemms_refused_after_free(weights):
    """A workspace freed through rvc_free ends what rvc_prefill_gemms may re-run on it, even
    when the next allocation gets the same address."""
    from rosevine_b200 import rvcuda as rc
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer, to_device_x
    lyr = MoeLayer(weights["w_router"], weights["gate_up"], weights["down"], max_tok=100)
    nbytes = rc.workspace_bytes(100, 2816, 704, 128, 8)
    ws = rc.DevBuf(nbytes)
    rc.workspace_reset(ws.view())
    x = to_device_x(synth.tokens(100, 1400), "cuda")
    out = torch.empty((100, 2816), dtype=torch.float32, device="cuda")
    rc.moe_forward(lyr.w, x, x, rc.BF16, 100, out, ws.view())
    rc.prefill_gemms(lyr.w, ws.view())
    rc.status(ws.view())
    ws.close()
    ws2 = rc.DevBuf(nbytes)
    try:
        with pytest.raises(rc.DeviceError):
            rc.prefill_gemms(lyr.w, ws2.view())
    finally:
        ws2.close()
