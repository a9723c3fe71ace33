"""Pins the CPU oracle (oracle/rv_oracle.c) to the reference's own known answers.

Two sources: (1) the reference's Rust unit tests, restated here with their exact vectors and
bounds (runtime/src/ops.rs:354-448, runtime/src/expert_kernel.rs:257-401,
runtime/src/expert_pool.rs:502-539); (2) tests/golden/golden_v1.json, produced by the
reference's binary64 scalar oracle scripts/correctness_oracle.py through
tests/golden/make_golden.py.
"""
import ctypes
import math
import struct

import numpy as np
import pytest

libm = ctypes.CDLL("libm.so.6")
libm.sinf.argtypes, libm.sinf.restype = [ctypes.c_float], ctypes.c_float
libm.cosf.argtypes, libm.cosf.restype = [ctypes.c_float], ctypes.c_float


def f32(v):
    return struct.unpack("<f", struct.pack("<f", v))[0]


class XorShift:
    """The reference tests' xorshift64 generator (expert_kernel.rs:304-310)."""

    def __init__(self, seed):
        self.s = seed

    def next(self):
        s = self.s
        s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 7
        s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
        self.s = s
        return s


# ----------------------------------------------------------------- ops.rs tests
def test_f16_round_trip_and_rounding(oracle):
    # ops.rs:358-368
    for h in [0, 0x3C00, 0xBC00, 0x7BFF, 0x0001, 0x03FF, 0x0400, 0x7C00, 0x3555]:
        assert oracle.f32_to_f16(oracle.f16_to_f32(h)) == h, hex(h)
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f32_to_f16(65520.0) == 0x7C00
    assert oracle.f32_to_f16(1.0 + 1.0 / 2048.0) == 0x3C00
    assert oracle.f32_to_f16(1.0 + 3.0 / 2048.0) == 0x3C02
    assert oracle.f16_to_f32(oracle.f32_to_f16(5.9604645e-8)) == f32(5.9604645e-8)


def test_f16_conversion_matches_ieee_for_all_halves(oracle):
    # numpy's float16 is IEEE binary16 with RNE: every finite half converts identically.
    for h in range(0, 0x10000, 7):
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        got = oracle.f16_to_f32(h)
        if np.isnan(want):
            assert math.isnan(got)
        else:
            assert got == want, hex(h)
    rng = np.random.default_rng(3)
    for v in np.concatenate([rng.standard_normal(2000).astype(np.float32) * 100,
                             rng.standard_normal(2000).astype(np.float32) * 1e-5]):
        assert oracle.f32_to_f16(float(v)) == int(np.float32(v).astype(np.float16).view(np.uint16))


def test_norm_softmax_topk(oracle):
    # ops.rs:405-415
    p = oracle.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(float(p.sum()) - 1.0) < 1e-6 and p[2] > p[1]
    assert oracle.top_k(np.array([0.1, 0.5, 0.5, 0.2], np.float32), 3) == [1, 2, 3]


def test_top_k_total_order_and_ties(oracle):
    x = np.array([0.0, -0.0, 1.0, 1.0, -1.0, np.inf, 0.5], np.float32)
    assert oracle.top_k(x, 7) == [5, 2, 3, 6, 0, 1, 4]


# --------------------------------------------------------- expert_kernel.rs tests
def _q8_case(iteration, k, nxt, oracle):
    x = np.array([f32(libm.sinf(f32((i + iteration) * f32(0.37)))) * (1 + i % 5) for i in range(k)], np.float32)
    xq = oracle.quantize_q8_0(x)[0]
    row = bytearray(k // 32 * 18)
    scales = [0.0, 0.01, -0.1, 0.00000006, 3.0]
    for i in range(k // 32):
        h = oracle.f32_to_f16(scales[(iteration + i) % 5])
        row[18 * i:18 * i + 2] = struct.pack("<H", h)
        for j in range(16):
            row[18 * i + 2 + j] = nxt() & 0xFF
    if iteration % 7 == 0:
        for i in range(k // 32):
            row[18 * i + 2:18 * i + 18] = bytes(16)
        for i in range(k // 32):
            xq[34 * i + 2:34 * i + 34] = 0x81 if iteration % 2 == 0 else 0x7F
    return np.frombuffer(bytes(row), np.uint8).copy(), xq


def test_q8_kernels_match_exact_integer_reference(oracle):
    # expert_kernel.rs:302-356
    g = XorShift(5)
    for k in [32, 96, 704, 2816]:
        for iteration in range(256):
            row, xq = _q8_case(iteration, k, g.next, oracle)
            exact = magnitude = 0.0
            for b in range(k // 32):
                w, xb = row[18 * b:18 * b + 18], xq[34 * b:34 * b + 34]
                d = float(oracle.f16_to_f32(int(w[0]) | int(w[1]) << 8)) * float(
                    oracle.f16_to_f32(int(xb[0]) | int(xb[1]) << 8))
                lo = (w[2:18] & 15).astype(np.int64) - 8
                hi = (w[2:18] >> 4).astype(np.int64) - 8
                qx = xb[2:34].view(np.int8).astype(np.int64)
                prod = np.concatenate([lo * qx[:16], hi * qx[16:]])
                exact += float(prod.sum()) * d
                magnitude += float(np.abs(prod).sum()) * abs(d)
            scalar = oracle.dot_q8(row, xq, k, oracle.KERNEL_SCALAR)
            for kern in [oracle.KERNEL_SCALAR, oracle.KERNEL_AVX2]:
                v = oracle.dot_q8(row, xq, k, kern)
                assert abs(v - exact) <= 4e-6 * magnitude + 1e-30, (k, iteration, kern, v, exact)
            assert struct.pack("<f", oracle.dot_q8(row, xq, k)) == struct.pack("<f", scalar)


def test_q8_dot_tracks_f32_dot_within_activation_quantization_error(oracle):
    # expert_kernel.rs:358-382
    k = 2816
    x = np.array([f32(libm.cosf(f32(i * f32(0.011)))) * 0.5 for i in range(k)], np.float32)
    xq = oracle.quantize_q8_0(x)[0]
    row = bytearray(k // 32 * 18)
    for i in range(k // 32):
        row[18 * i:18 * i + 2] = struct.pack("<H", oracle.f32_to_f16(0.02))
        for j in range(16):
            row[18 * i + 2 + j] = (i * 31 + j * 7) & 0xFF
    row = np.frombuffer(bytes(row), np.uint8)
    deq = np.zeros(k, np.float32)
    for i in range(k // 32):
        d = oracle.f16_to_f32(oracle.f32_to_f16(0.02))
        nib = row[18 * i + 2:18 * i + 18]
        deq[32 * i:32 * i + 16] = ((nib & 15).astype(np.int32) - 8) * np.float32(d)
        deq[32 * i + 16:32 * i + 32] = ((nib >> 4).astype(np.int32) - 8) * np.float32(d)
    reference = float(np.dot(deq.astype(np.float64), x.astype(np.float64)))
    bound = sum(float(np.abs(deq[32 * i:32 * i + 32]).sum()) * float(np.abs(x[32 * i:32 * i + 32]).max()) / 127.0
                for i in range(k // 32))
    for kern in [oracle.KERNEL_SCALAR, oracle.KERNEL_AVX2]:
        assert abs(oracle.dot_q8(row, xq, k, kern) - reference) <= bound


def test_quantize_q8_0_rounding_rules(oracle):
    # ops.rs:95-105: d = amax/127 in f32, f16 RNE scale, q = round-half-away(v * (1/d))
    x = np.zeros(32, np.float32)
    x[0], x[1], x[2], x[3] = 127.0, 0.5, -0.5, -1.5
    q = oracle.quantize_q8_0(x)[0]
    assert struct.unpack("<H", q[:2].tobytes())[0] == oracle.f32_to_f16(1.0)
    assert list(q[2:6].view(np.int8)) == [127, 1, -1, -2]
    z = oracle.quantize_q8_0(np.zeros(32, np.float32))[0]
    assert not z.any()


# ----------------------------------------------------------- golden fixtures
def test_golden_q4_decode_through_block_sums(oracle, golden):
    # one-hot Q8 activation blocks extract each decoded nibble: (n - 8) * d
    for case in golden["q4_0_decode"]:
        blk = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
        d = oracle.f16_to_f32(int(blk[0]) | int(blk[1]) << 8)
        for j in range(32):
            xb = np.zeros(34, np.uint8)
            xb[2 + j] = 1
            v = oracle.block_sumi(blk, xb) * float(d)
            assert v == case["values"][j] or (v == 0 and case["values"][j] == 0), (case["block"], j)


def test_golden_gelu(oracle, golden):
    g = golden["gelu_tanh"]
    for x, want in zip(g["input"], g["output"]):
        got = oracle.gelu(x)
        assert abs(got - want) <= 1e-5 + 1e-4 * abs(want), (x, got, want)


def test_golden_softmax_extremes(oracle, golden):
    g = golden["softmax"]
    got = oracle.softmax(np.array(g["input"], np.float32))
    assert np.allclose(got, g["output"], rtol=1e-6, atol=1e-7)


def test_golden_router_selection(oracle, golden):
    for c in golden["router_selected_weights"]:
        lg = np.array([c["logits"]], np.float32)
        used = len(c["ids"])
        ids, w, probs = oracle.select_experts(lg, used)
        assert ids[0].tolist() == c["ids"]
        assert np.allclose(w[0], c["weights"], rtol=2e-6, atol=1e-9)
        assert np.allclose(probs[0], c["probabilities"], rtol=2e-6, atol=1e-12)


def test_golden_gated_ffn(oracle, golden):
    f = golden["gated_ffn"]["fixture"]
    x = np.array(f["input"], np.float64)
    up = np.array(f["up_matrix_rows"]) @ x
    gate = np.array(f["gate_matrix_rows"]) @ x
    h = np.array([oracle.gelu(float(gv)) * float(uv) for gv, uv in zip(gate, up)])
    out = np.array(f["down_matrix_rows"]) @ h
    want = golden["gated_ffn"]["result"]["output"]
    assert np.allclose(out, want, rtol=1e-4, atol=1e-5)


def test_golden_q4_q8_dots(oracle, golden):
    for c in golden["q4_q8_dots"]:
        row = np.frombuffer(bytes.fromhex(c["row"]), np.uint8)
        xq = np.frombuffer(bytes.fromhex(c["xq"]), np.uint8)
        for kern in [oracle.KERNEL_SCALAR, oracle.KERNEL_AVX2]:
            v = oracle.dot_q8(row, xq, c["k"], kern)
            assert abs(v - c["exact"]) <= 4e-6 * c["magnitude"] + 1e-30, (c["k"], kern, v, c["exact"])


# ------------------------------------------------------------- pool + plan
def test_moe_plan_is_the_stable_sort(oracle):
    rng = np.random.default_rng(7)
    ids = rng.integers(0, 16, size=200).astype(np.int32)
    order, pos_of, counts = oracle.moe_plan(ids, 16)
    want = sorted(range(200), key=lambda i: (ids[i], i))
    assert order.tolist() == want
    assert all(order[pos_of[p]] == p for p in range(200))
    assert counts.tolist() == np.bincount(ids, minlength=16).tolist()


@pytest.mark.parametrize("threads", [1, 3, 12])
def test_pool_matches_kernel_dot_on_every_segment(oracle, threads):
    # expert_pool.rs:502-539: pool outputs bitwise equal dot_q8 per element, any thread count
    from rosevine_b200 import synth
    n_embd, ff, ne, used, n_tok = 256, 64, 6, 2, 5
    gu, dn = synth.experts(11, ne, n_embd, ff)
    x = synth.tokens(n_tok, 12, n_embd)
    rng = np.random.default_rng(13)
    ids = np.array([rng.choice(ne, used, replace=False) for _ in range(n_tok)], np.int32)
    w = rng.random((n_tok, used)).astype(np.float32)
    pool = oracle.Pool(threads, oracle.KERNEL_SCALAR)
    try:
        out, h, y = oracle.experts_q8(pool, x, gu, dn, None, ids, w, n_embd, ff, ne, debug=True)
    finally:
        pool.close()
    order, pos_of, _ = oracle.moe_plan(ids, ne)
    dn_rows = dn.reshape(ne, n_embd, -1)
    qh = oracle.quantize_q8_0(h)
    for k in range(n_tok * used):
        e = ids.reshape(-1)[order[k]]
        for r in range(0, n_embd, 17):
            v = oracle.dot_q8(dn_rows[e, r], qh[k], ff, oracle.KERNEL_SCALAR)
            assert struct.pack("<f", v) == struct.pack("<f", float(y[k, r]))
    # combine in slot order (exec.rs:626-638), bitwise
    for t in range(n_tok):
        o = None
        for j in range(used):
            p = t * used + j
            v = y[pos_of[p]] * np.float32(1.0) * w[t, j]
            o = v if o is None else (o + v).astype(np.float32)
        assert np.array_equal(o, out[t])


def test_layer_is_batch_invariant(oracle, pool):
    # runtime/tests/exec.rs:181-199: batched and stepped evaluation are bitwise identical
    from rosevine_b200 import synth
    n_embd, ff, ne, n_tok = 256, 64, 16, 6
    gu, dn = synth.experts(21, ne, n_embd, ff)
    x = synth.tokens(n_tok, 22, n_embd)
    wr = synth.router(23, ne, n_embd)
    out, ids, w, lg = oracle.moe_layer(pool, x, x, wr, gu, dn, ff=ff)
    for t in range(n_tok):
        o1, i1, w1, l1 = oracle.moe_layer(pool, x[t:t + 1], x[t:t + 1], wr, gu, dn, ff=ff)
        assert np.array_equal(o1[0], out[t]) and np.array_equal(i1[0], ids[t]) and np.array_equal(l1[0], lg[t])
