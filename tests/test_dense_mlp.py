"""The layer's shared dense MLP (rvc_q4_mm, rvc_geglu, rvc_shared_mlp; rosevine_b200/csrc/dense.cuh).

Reference: runtime/src/exec.rs:438-453 (CPU) and runtime/src/hip_exec.rs:770-778 (device): the
Q4_0 x F32 matmul of ops.rs:249-266 (each dot a sequential f32 sum of rounded products), GELU-tanh
times up, and the two RMS norms. The reference accepts its own device matmul at an L2 relative
error below 1e-5 with each token's row bitwise equal to its single-token result
(runtime/tests/hip_ops.rs:56-80, shapes (2112, 2816) and (2816, 2112) among them); the kernels
here keep the sequential order, so the bar is bit-exactness against the oracle's restatement.

CPU: the oracle pinned against a numpy restatement of the sequential sum, the reference's Q4_0
decode fixtures and its gated-FFN fixture (research/fixtures/scalar-operators-v1.json via
tests/golden). GPU (marked): bit-exact matmul at the reference's shapes and token counts, batch
invariance, the GELU product, and the whole MLP with its norms.
"""
import numpy as np
import pytest


def q4_rows(rng, n_rows, k):
    from rosevine_b200 import synth
    return synth.q4_rows(rng, (n_rows, k // 32))


def np_matmul_q4_0(w, x, n_out):
    """ops.rs:83-92 and :249-266 in numpy: dequantised rows, products rounded to f32, summed
    in sequence from -0."""
    n_in, k = x.shape
    nb = k // 32
    rows = np.ascontiguousarray(w).view(np.uint8).reshape(n_out, nb, 18)
    d = rows[:, :, :2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    q = rows[:, :, 2:]
    lo = (q & 15).astype(np.int32) - 8
    hi = (q >> 4).astype(np.int32) - 8
    deq = (np.concatenate([lo, hi], axis=2).astype(np.float32) * d[:, :, None]).reshape(n_out, k)
    y = np.empty((n_in, n_out), np.float32)
    for t in range(n_in):
        for r in range(n_out):
            p = (deq[r] * x[t]).astype(np.float32)
            s = np.float32(-0.0)
            for v in p:
                s = np.float32(s + v)
            y[t, r] = s
    return y


def test_oracle_matmul_is_the_sequential_sum(oracle):
    rng = np.random.default_rng(1)
    w = q4_rows(rng, 3, 96)
    x = rng.standard_normal((2, 96)).astype(np.float32)
    got = oracle.matmul_q4_0(w, x, 3)
    assert np.array_equal(got.view(np.uint32), np_matmul_q4_0(w, x, 3).view(np.uint32))


def _q4_from_values(rows):
    """Q4_0 rows (d = 1) holding small integer matrices, zero-padded to 32 columns."""
    out = np.zeros((len(rows), 18), np.uint8)
    for r, vals in enumerate(rows):
        out[r, :2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
        q = [8] * 32
        for i, v in enumerate(vals):
            q[i] = int(v) + 8
        for j in range(16):
            out[r, 2 + j] = q[j] | (q[j + 16] << 4)
    return out


def test_oracle_gated_ffn_matches_the_reference_fixture(oracle, golden):
    g = golden["gated_ffn"]
    fx, want = g["fixture"], g["result"]
    x = np.zeros((1, 32), np.float32)
    x[0, :2] = fx["input"]
    gate = oracle.matmul_q4_0(_q4_from_values(fx["gate_matrix_rows"]), x, 2)[0]
    up = oracle.matmul_q4_0(_q4_from_values(fx["up_matrix_rows"]), x, 2)[0]
    assert list(gate) == want["gate"] and list(up) == want["up"]
    gated = np.array([oracle.gelu(float(a)) * np.float32(b) for a, b in zip(gate, up)], np.float32)
    np.testing.assert_allclose(gated, want["gated"], rtol=1e-6)
    h = np.zeros((1, 32), np.float32)
    h[0, :2] = gated
    out = oracle.matmul_q4_0(_q4_from_values(fx["down_matrix_rows"]), h, 1)[0]
    np.testing.assert_allclose(out, want["output"], rtol=1e-6)


def test_oracle_dequant_matches_the_reference_fixture(oracle, golden):
    # a Q4_0 row times unit vectors reads back each dequantised value (q4_0_decode fixture)
    for case in golden["q4_0_decode"]:
        blk = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
        y = oracle.matmul_q4_0(blk, np.eye(32, dtype=np.float32), 1)[:, 0]
        assert np.array_equal(np.abs(y), np.abs(np.array(case["values"], np.float32)))


@pytest.mark.gpu
@pytest.mark.parametrize("n_out,k", [(2112, 2816), (2816, 2112), (100, 96)])
def test_q4_mm_bit_exact_and_batch_invariant(oracle, n_out, k):
    torch = pytest.importorskip("torch")
    import rosevine_b200.rvcuda as rc
    rng = np.random.default_rng(n_out + k)
    w = q4_rows(rng, n_out, k)
    wd = torch.from_numpy(np.ascontiguousarray(w).reshape(-1)).cuda()
    for n_in in (1, 7, 64):
        x = rng.standard_normal((n_in, k)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        y = torch.empty((n_in, n_out), dtype=torch.float32, device="cuda")
        rc.q4_mm(wd, xd, y, n_out, k, n_in)
        want = oracle.matmul_q4_0(w, x, n_out)
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"n_in={n_in}"
        if n_in > 1:  # batch invariance: the last token alone gives the same bits
            y1 = torch.empty((1, n_out), dtype=torch.float32, device="cuda")
            rc.q4_mm(wd, xd[-1:].contiguous(), y1, n_out, k, 1)
            assert torch.equal(y1[0], y[-1])


@pytest.mark.gpu
def test_geglu_bit_exact(oracle):
    torch = pytest.importorskip("torch")
    import rosevine_b200.rvcuda as rc
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(5000) * 4).astype(np.float32)
    u = rng.standard_normal(5000).astype(np.float32)
    out = torch.empty(5000, dtype=torch.float32, device="cuda")
    rc.geglu(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda(), out, 5000)
    want = np.array([np.float32(oracle.gelu(float(a))) * b for a, b in zip(g, u)], np.float32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("n_tok", [1, 5, 40])
def test_shared_mlp_bit_exact(oracle, n_tok):
    torch = pytest.importorskip("torch")
    import rosevine_b200.rvcuda as rc
    n_embd, ff, eps = 2816, 2112, 1e-6
    rng = np.random.default_rng(10 + n_tok)
    wg, wu, wdn = q4_rows(rng, ff, n_embd), q4_rows(rng, ff, n_embd), q4_rows(rng, n_embd, ff)
    fn = rng.uniform(0.5, 1.5, n_embd).astype(np.float32)
    pn = rng.uniform(0.5, 1.5, n_embd).astype(np.float32)
    x = (rng.standard_normal((n_tok, n_embd)) * 2).astype(np.float32)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v).reshape(-1)).cuda()
           for k, v in {"wg": wg, "wu": wu, "wd": wdn, "fn": fn, "pn": pn, "x": x}.items()}
    out = torch.empty((n_tok, n_embd), dtype=torch.float32, device="cuda")
    ws = torch.empty(rc.shared_mlp_workspace_bytes(n_tok, n_embd, ff), dtype=torch.uint8, device="cuda")
    rc.shared_mlp(dev["wg"], dev["wu"], dev["wd"], dev["fn"], dev["pn"], dev["x"], out, n_tok, n_embd, ff, eps, ws)
    want = oracle.shared_mlp(wg, wu, wdn, fn, pn, x, ff, eps)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
