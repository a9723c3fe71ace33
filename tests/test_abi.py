"""The C ABI library loads without a GPU, exports every symbol include/rvcuda.h declares, and
rejects bad scalar arguments before any device work (the reference ABI's CHECK_DIMS
convention, runtime/hip/rvhip.hip:511-514). No compute call is made here."""
import ctypes
import os
import re
import subprocess

import pytest

from rosevine_b200 import rvcuda as rc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            syms |= set(re.findall(r"\b(rvc_\w+)\s*\(", text))
    return syms


@pytest.fixture(scope="module")
def lib():
    from rosevine_b200 import build
    build.build()
    return rc.lib()


def test_every_declared_symbol_is_exported(lib):
    declared = declared_symbols()
    assert declared, "no declarations found"
    out = subprocess.run(["nm", "-D", "--defined-only", rc.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (rvc_\w+)", out))
    assert declared <= exported, declared - exported
    assert set(rc.EXPORTS) == declared
    for s in declared:
        assert hasattr(lib, s)


def test_host_size_queries(lib):
    assert rc.packed_bytes(128, 2816, 704) == 523370496  # 428,212,224 GGUF bytes + f32 scale tiles
    assert rc.packed_bytes(128, 2816, 700) == 0
    assert rc.workspace_bytes(64, 2816, 704, 128, 8) > 0
    assert rc.workspace_bytes(0, 2816, 704, 128, 8) == 0
    assert rc.workspace_bytes(128, 2816, 704, 128, 8) > rc.workspace_bytes(64, 2816, 704, 128, 8)


def test_noalloc_scratch_holds_the_decode_layout_at_the_target_shapes(lib):
    # rvc_moe_forward_noalloc runs the decode kernels (up to 64 tokens) on a fixed
    # RVC_NOALLOC_SCRATCH_BYTES array. A workspace for 64 tokens, the largest call that
    # rvc_moe_forward also gives the decode kernels, has the decode layout alone and fits it.
    import rosevine_b200.rvcuda as rc
    dec32 = rc.workspace_bytes(32, 2816, 704, 128, 8)
    dec64 = rc.workspace_bytes(64, 2816, 704, 128, 8)
    assert 0 < dec32 < dec64 < rc.NOALLOC_SCRATCH_BYTES, (dec32, dec64)


def test_error_strings(lib):
    assert "timeout" in rc.error_string(rc.ERR_DEVICE_TIMEOUT) or "ran out" in rc.error_string(rc.ERR_DEVICE_TIMEOUT)
    assert "workspace" in rc.error_string(rc.ERR_WORKSPACE)
    assert rc.error_string(1)  # cudaErrorInvalidValue text


def test_invalid_scalars_rejected_without_device_work(lib):
    w = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, None, None, None)
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    assert lib.rvc_moe_forward(ctypes.byref(w), p, p, rc.BF16, None, 0, 1, p, None, None, p, 1 << 20, None) == 1
    w2 = rc.MoeWeights(2816, 700, 128, 8, rc.BF16, 16, 16, None)  # ff not a multiple of 32
    assert lib.rvc_moe_experts(ctypes.byref(w2), p, rc.BF16, p, p, 1, p, p, 1 << 20, None) == 1
    w3 = rc.MoeWeights(2816, 704, 128, 17, rc.BF16, 16, 16, None)  # used > 16
    assert lib.rvc_moe_router(ctypes.byref(w3), p, rc.BF16, None, 0, 1, p, p, None, None, None, p, 1 << 20,
                              None) == 1
    assert lib.rvc_pack_experts(None, p, 128, 2816, 704, p, None) == 1
    assert lib.rvc_alloc(16, None) == 1
    assert lib.rvc_workspace_reset(None, None) == 1
    # misaligned activations or packed weights are refused (16 B for vector loads, 256 B for TMA)
    w4 = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, 4096, 4096 + 16, None)
    q = ctypes.c_void_p(4096)
    assert lib.rvc_moe_forward(ctypes.byref(w4), q, q, rc.BF16, None, 0, 1, q, None, None, q, 1 << 20, None) == 1
    w5 = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, 4096, 4096, None)
    odd = ctypes.c_void_p(4096 + 8)
    assert lib.rvc_moe_forward(ctypes.byref(w5), odd, q, rc.BF16, None, 0, 1, q, None, None, q, 1 << 20, None) == 1


def test_prefill_gemms_needs_a_prior_prefill_call(lib):
    """rvc_prefill_gemms re-runs a prefill call's GEMMs on its workspace; a workspace that never
    held one (as here) is refused on the host, before any device work."""
    w = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, 4096, 4096, None)
    p = ctypes.c_void_p(4096)  # aligned, never dereferenced
    big = rc.workspace_bytes(64, 2816, 704, 128, 8)
    assert lib.rvc_prefill_gemms(ctypes.byref(w), p, big, None) == 1
    assert lib.rvc_prefill_gemms(None, p, big, None) == 1


def test_workspace_too_small_is_rejected(lib):
    w = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, 4096, 4096, None)
    p = ctypes.c_void_p(4096)  # aligned, never dereferenced: the size check fails first
    small = rc.workspace_bytes(4, 2816, 704, 128, 8)
    assert lib.rvc_moe_forward(ctypes.byref(w), p, p, rc.BF16, None, 0, 5, p, None, None, p, small,
                               None) == rc.ERR_WORKSPACE


def test_noalloc_scratch_refusals_on_the_host(lib):
    """rvc_moe_forward_noalloc refuses, before any device work, a call of at most 64 tokens whose
    decode layout exceeds its fixed array (n_embd 8192, ff 4096: the down partials alone take
    16 MB) and a call of more than 64 tokens at the target's shapes."""
    p = ctypes.c_void_p(4096)  # aligned, never dereferenced
    assert rc.workspace_bytes(64, 8192, 4096, 128, 8) > rc.NOALLOC_SCRATCH_BYTES
    wide = rc.MoeWeights(8192, 4096, 128, 8, rc.BF16, 4096, 4096, None)
    assert lib.rvc_moe_forward_noalloc(ctypes.byref(wide), p, p, rc.BF16, None, 0, 64, p, None, None,
                                       None) == rc.ERR_WORKSPACE
    target = rc.MoeWeights(2816, 704, 128, 8, rc.BF16, 4096, 4096, None)
    assert lib.rvc_moe_forward_noalloc(ctypes.byref(target), p, p, rc.BF16, None, 0, 65, p, None, None,
                                       None) == rc.ERR_WORKSPACE


def test_checked_views_refuse_out_of_range():
    v = rc.View(1 << 20, 100)
    assert v.need(100) == 1 << 20
    with pytest.raises(ValueError):
        v.need(101)


def test_integration_names_only_declared_symbols():
    """Every library entry INTEGRATION.md's bindings call (rvc_* names and the cuda:: wrappers,
    each a thin shim over rvc_<name>) is declared in include/rvcuda.h."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    declared = declared_symbols()
    header = open(os.path.join(ROOT, "include", "rvcuda.h")).read()
    types = {a or b for a, b in re.findall(r"typedef struct \w+ (rvc_\w+);|\}\s*(rvc_\w+);", header)}
    assert {"rvc_moe_weights", "rvc_gguf", "rvc_gguf_moe"} <= types, types
    named = set(re.findall(r"\b(rvc_\w+)\b", text)) - types
    wrapped = {"rvc_" + n for n in re.findall(r"\bcuda::(\w+)\s*\(", text)}
    assert named, "no rvc_ names found"
    assert named <= declared, named - declared
    assert wrapped <= declared, wrapped - declared
