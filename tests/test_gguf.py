"""GGUF weights: the library's reader (rvc_gguf_*, rosevine_b200/csrc/gguf.h) against the checks of
the reference's parser, and the MoE layer built from a GGUF file.

CPU: the reference's own synthetic GGUF cases (runtime/tests/synthetic.rs:9-178: a minimal v3
writer, a valid file with exact views, every truncation, header, metadata and tensor-descriptor
violations), restated with a writer of our own; each rejection must carry the reference's reason
(rvc_error_string of the returned code). Then the binding of one layer's MoE tensors by name and
contract shape (runtime/src/model.rs:61-107, contract.rs:66-70).

GPU (marked): MoeLayer.from_gguf on a file with the target's shapes produces the same outputs,
bit for bit, as a layer built from the same arrays directly, and matches the oracle.
"""
import os
import struct
import tempfile

import numpy as np
import pytest

import rosevine_b200.rvcuda as rc


def _s(v: bytes) -> bytes:
    return struct.pack("<Q", len(v)) + v


class Builder:
    """GGUF v3 bytes: header, metadata, tensor descriptors, padding to 32, data i % 251."""

    def __init__(self):
        self.kv, self.tensors, self.data_len, self.version = [], [], 0, 3

    def raw_kv(self, key, tv: bytes):
        self.kv.append((key, tv))
        return self

    def kv_str(self, key, v):
        return self.raw_kv(key, struct.pack("<I", 8) + _s(v.encode()))

    def kv_u32(self, key, v):
        return self.raw_kv(key, struct.pack("<II", 4, v))

    def tensor(self, name, shape, ty, off):
        self.tensors.append((name, list(shape), ty, off))
        return self

    def data(self, n):
        self.data_len = n
        return self

    def build(self, payload: bytes | None = None) -> bytes:
        out = b"GGUF" + struct.pack("<IQQ", self.version, len(self.tensors), len(self.kv))
        for k, v in self.kv:
            out += _s(k.encode()) + v
        for name, shape, ty, off in self.tensors:
            out += _s(name.encode()) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
            out += struct.pack("<IQ", ty, off)
        out += b"\0" * (-len(out) % 32)
        return out + (payload if payload is not None else bytes(i % 251 for i in range(self.data_len)))


def valid() -> Builder:
    """One F32 [8] tensor at 0 and one Q4_0 [32, 2] tensor at 32: 32 + 36 bytes of data."""
    return (Builder().kv_str("general.architecture", "test").kv_u32("general.alignment", 32)
            .tensor("a", [8], 0, 0).tensor("b", [32, 2], 2, 32).data(68))


def reason(b) -> str:
    data = b.build() if isinstance(b, Builder) else b
    with pytest.raises(rc.DeviceError) as e:
        rc.GgufFile(data=data)
    assert rc.ERR_GGUF <= e.value.code < rc.ERR_GGUF + 100
    return rc.error_string(e.value.code)


def test_valid_file_parses_with_exact_views():
    data = valid().build()
    g = rc.GgufFile(data=data)
    dt, shape, a = g.tensor("a")
    assert (dt, shape, a.nbytes) == (0, (8,), 32)
    dt, shape, b = g.tensor("b")
    assert (dt, shape, b.nbytes) == (2, (32, 2), 36)
    off = len(data) - 68
    assert bytes(a) == data[off:off + 32] and bytes(b) == data[off + 32:off + 68]
    with pytest.raises(rc.DeviceError) as e:
        g.tensor("c")
    assert rc.error_string(e.value.code) == "missing tensor"
    g.close()


def test_every_truncation_is_rejected():
    data = valid().build()
    for n in range(len(data)):
        with pytest.raises(rc.DeviceError):
            rc.GgufFile(data=data[:n])


def test_header_violations():
    bad = bytearray(valid().build())
    bad[0] = ord("X")
    assert reason(bytes(bad)) == "bad magic"
    v2 = valid()
    v2.version = 2
    assert reason(v2) == "expected GGUF version 3"
    assert reason(Builder().data(0)) == "descriptor count limit exceeded"
    many = bytearray(valid().build())
    many[16:24] = struct.pack("<Q", 1 << 40)
    assert reason(bytes(many)) == "descriptor count limit exceeded"


def test_metadata_violations():
    assert reason(valid().kv_str("general.architecture", "x")) == "duplicate metadata key"
    assert reason(valid().kv_str("", "x")) == "empty metadata key"
    for align in (0, 3, 48, 1 << 21):
        b = valid()
        b.kv[1] = ("general.alignment", struct.pack("<II", 4, align))
        assert reason(b) == "invalid alignment", align
    assert reason(valid().raw_kv("k", struct.pack("<I", 7) + b"\x02")) == "invalid bool"
    assert reason(valid().raw_kv("k", struct.pack("<IIQ", 9, 9, 1))) == "unsupported array element type"
    assert reason(valid().raw_kv("k", struct.pack("<IIQ", 9, 4, 1 << 40))) == "array length limit exceeded"
    assert reason(valid().raw_kv("k", struct.pack("<IIQ", 9, 8, 4_000_000))) == "truncated header"
    assert reason(valid().raw_kv("k", struct.pack("<IQ", 8, 1 << 40))) == "string length limit exceeded"
    assert reason(valid().raw_kv("k", struct.pack("<IQ", 8, 1) + b"\xff")) == "string is not UTF-8"
    assert reason(valid().raw_kv("k", struct.pack("<I", 13))) == "unsupported metadata type"


def test_tensor_descriptor_violations():
    def base():
        return Builder().data(4096)
    assert reason(base().tensor("x", [8], 0, 0).tensor("x", [8], 0, 32)) == "empty or duplicate tensor name"
    assert reason(base().tensor("", [8], 0, 0)) == "empty or duplicate tensor name"
    assert reason(base().tensor("x", [], 0, 0)) == "invalid tensor rank"
    assert reason(base().tensor("x", [1, 1, 1, 1, 1], 0, 0)) == "invalid tensor rank"
    assert reason(base().tensor("x", [8, 0], 0, 0)) == "invalid tensor shape"
    assert reason(base().tensor("x", [33], 2, 0)) == "invalid tensor shape"
    assert reason(base().tensor("x", [8], 1, 0)) == "unsupported tensor type"
    assert reason(base().tensor("x", [8], 0, 16)) == "misaligned tensor offset"
    assert reason(base().tensor("x", [1 << 40, 1 << 40], 0, 0)) == "tensor element count overflow"
    assert reason(base().tensor("x", [16], 0, 0).tensor("y", [8], 0, 32)) == \
        "overlapping or out-of-file tensor range"
    assert reason(base().tensor("x", [2048], 0, 0)) == "overlapping or out-of-file tensor range"
    assert reason(base().tensor("x", [8], 0, (1 << 64) - 32)) == "tensor range overflow"


def moe_file(layer, n_embd, ff, ne, seed, skip=None, bad_shape=None):
    """GGUF bytes holding one layer's MoE tensors (contract.rs:42-51, 66-70 names, ggml shapes) and
    the arrays written: synthetic Q4_0 experts, an F32 router, scales and norm weights."""
    from rosevine_b200 import synth
    gu, dn = synth.experts(seed, n_experts=ne, n_embd=n_embd, ff=ff)
    rng = np.random.default_rng(seed)
    arrays = {
        "ffn_gate_up_exps.weight": (2, [n_embd, 2 * ff, ne], np.ascontiguousarray(gu).view(np.uint8)),
        "ffn_down_exps.weight": (2, [ff, n_embd, ne], np.ascontiguousarray(dn).view(np.uint8)),
        "ffn_gate_inp.weight": (0, [n_embd, ne], (rng.standard_normal((ne, n_embd)) * 0.02).astype(np.float32)),
        "ffn_down_exps.scale": (0, [ne], rng.uniform(0.9, 1.2, ne).astype(np.float32)),
        "ffn_gate_inp.scale": (0, [n_embd], rng.uniform(0.5, 1.5, n_embd).astype(np.float32)),
        "pre_ffw_norm_2.weight": (0, [n_embd], rng.uniform(0.5, 1.5, n_embd).astype(np.float32)),
        "post_ffw_norm_2.weight": (0, [n_embd], rng.uniform(0.5, 1.5, n_embd).astype(np.float32)),
    }
    b = Builder().kv_str("general.architecture", "gemma4")
    payload, off = b"", 0
    for name, (ty, shape, arr) in arrays.items():
        if name == skip:
            continue
        shp = list(shape)
        if name == bad_shape:
            shp[-1] += 1  # one row (or element) more than the contract's
        raw = arr.tobytes()
        need = int(np.prod(shp)) // (32 if ty == 2 else 1) * (18 if ty == 2 else 4)
        raw = raw + b"\0" * (need - len(raw)) if need > len(raw) else raw[:need]
        b.tensor(f"blk.{layer}.{name}", shp, ty, off)
        payload += raw + b"\0" * (-len(raw) % 32)
        off = len(payload)
    return b.build(payload), {k: v[2] for k, v in arrays.items()}


def test_moe_layer_tensors_bound_by_name_and_contract():
    data, arrays = moe_file(3, 256, 64, 4, seed=5)
    g = rc.GgufFile(data=data)
    t = g.moe_layer(3, 256, 64, 4)
    assert np.array_equal(t["gate_up"].reshape(-1), arrays["ffn_gate_up_exps.weight"].reshape(-1))
    assert np.array_equal(t["down"].reshape(-1), arrays["ffn_down_exps.weight"].reshape(-1))
    assert np.array_equal(t["router"], arrays["ffn_gate_inp.weight"])
    for k, name in (("down_scale", "ffn_down_exps.scale"), ("gate_inp_scale", "ffn_gate_inp.scale"),
                    ("pre_norm", "pre_ffw_norm_2.weight"), ("post_norm", "post_ffw_norm_2.weight")):
        assert np.array_equal(t[k], arrays[name]), k
    with pytest.raises(rc.DeviceError) as e:
        g.moe_layer(2, 256, 64, 4)  # no such layer
    assert rc.error_string(e.value.code) == "missing tensor"
    with pytest.raises(rc.DeviceError) as e:
        g.moe_layer(3, 256, 64, 8)  # another expert count than the file's
    assert rc.error_string(e.value.code) == "tensor shape or type differs from the layer's contract"
    g.close()
    data, _ = moe_file(0, 256, 64, 4, seed=6, skip="ffn_down_exps.scale")
    with pytest.raises(rc.DeviceError) as e:
        rc.GgufFile(data=data).moe_layer(0, 256, 64, 4)
    assert rc.error_string(e.value.code) == "missing tensor"
    data, _ = moe_file(0, 256, 64, 4, seed=7, bad_shape="ffn_gate_inp.weight")
    with pytest.raises(rc.DeviceError) as e:
        rc.GgufFile(data=data).moe_layer(0, 256, 64, 4)
    assert rc.error_string(e.value.code) == "tensor shape or type differs from the layer's contract"


def test_open_maps_a_file_like_parse():
    data, arrays = moe_file(1, 256, 64, 4, seed=8)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.gguf")
        with open(p, "wb") as f:
            f.write(data)
        with rc.GgufFile(p) as g:
            t = g.moe_layer(1, 256, 64, 4)
            assert np.array_equal(t["router"], arrays["ffn_gate_inp.weight"])
        with pytest.raises(rc.DeviceError) as e:
            rc.GgufFile(os.path.join(d, "absent.gguf"))
        assert rc.error_string(e.value.code) == "cannot open or map the file"


@pytest.mark.gpu
def test_layer_from_gguf_matches_the_same_weights_and_the_oracle(oracle, pool):
    torch = pytest.importorskip("torch")
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer, to_device_x
    ne, n_tok = 16, 5
    data, arrays = moe_file(2, synth.N_EMBD, synth.FF, ne, seed=9)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.gguf")
        with open(p, "wb") as f:
            f.write(data)
        lg = MoeLayer.from_gguf(p, 2, max_tok=n_tok, n_experts=ne)
    assert np.array_equal(lg.norms["pre_norm"], arrays["pre_ffw_norm_2.weight"])
    gu = arrays["ffn_gate_up_exps.weight"].reshape(ne, 2 * synth.FF, -1)
    dn = arrays["ffn_down_exps.weight"].reshape(ne, synth.N_EMBD, -1)
    ld = MoeLayer(arrays["ffn_gate_inp.weight"], gu, dn, down_scale=arrays["ffn_down_exps.scale"], max_tok=n_tok)
    x = synth.tokens(n_tok, 11)
    xd = to_device_x(x, "cuda")
    ids_g = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
    got = lg.forward(xd, ids=ids_g).cpu().numpy()
    want_same = ld.forward(xd).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want_same.view(np.uint32))
    want, want_ids, _, _ = oracle.moe_layer(pool, x, x, arrays["ffn_gate_inp.weight"], gu, dn,
                                            down_scale=arrays["ffn_down_exps.scale"])
    assert np.array_equal(ids_g.cpu().numpy(), want_ids)
    err = (np.abs(got - want).max(axis=1) / np.abs(want).max(axis=1)).max()
    assert err <= 1e-4, err
