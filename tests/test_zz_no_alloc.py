"""rvc_moe_forward_noalloc: the MoE layer for callers that cannot hand the library a workspace.

Hosts whose device memory is carved up once by their own allocator, or that must not risk a
failing or synchronising allocation in the middle of a decode step, cannot call cudaMalloc
(or rvc_alloc) for scratch. This entry point runs the same layer on a fixed array compiled
into librvcuda.so, always with the decode kernels (up to 64 tokens). The test calls it through
the C ABI and checks it against rvc_moe_forward (with its own workspace) on two calls in a row:
expert ids equal, and the output within the decode tolerance (bit for bit when both take the
decode kernels; above 64 tokens rvc_moe_forward takes the prefill kernels, whose routing weights
come from the exact router chains). It lives in its own file, collected last, and builds its own
layer so it also passes in a fresh process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-4  # row relative error, as the decode layer's tests


@pytest.fixture(scope="module")
def small_layer():
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer
    ne = 32
    gu, dn = synth.experts(31, n_experts=ne)
    return MoeLayer(synth.router(32, n_experts=ne), gu, dn, down_scale=synth.down_scales(33, ne), max_tok=64)


def test_noalloc_forward_matches_workspace_forward_twice(small_layer):
    from rosevine_b200 import rvcuda as rc
    from rosevine_b200 import synth
    from rosevine_b200.moe import to_device_x
    lyr = small_layer
    stream = torch.cuda.current_stream().cuda_stream
    for call, n_tok in enumerate([37, 5]):  # a larger call, then a smaller one over its leftovers
        x = to_device_x(synth.tokens(n_tok, 500 + call), "cuda")
        want_ids = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
        want = lyr.forward(x, ids=want_ids)
        got = torch.full_like(want, float("nan"))
        ids = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
        rc.moe_forward_noalloc(lyr.w, x, x, rc.BF16, n_tok, got, ids=ids, stream=stream)
        torch.cuda.synchronize()
        assert torch.equal(ids, want_ids), f"call {call}: expert ids differ from rvc_moe_forward"
        g, w = got.cpu().numpy(), want.cpu().numpy()
        err = (np.abs(g - w).max(axis=1) / np.maximum(np.abs(w).max(axis=1), 1e-30)).max()
        assert err <= DECODE_TOL, f"call {call}: row relative error {err:.2e} against rvc_moe_forward"
        if n_tok <= 64:  # the same kernels on both sides
            assert torch.equal(got, want), f"call {call}: differs from rvc_moe_forward"


def test_noalloc_rejects_requests_beyond_its_scratch(small_layer):
    from rosevine_b200 import rvcuda as rc
    lyr = small_layer
    n_tok = 400  # needs more than RVC_NOALLOC_SCRATCH_BYTES of scratch
    assert rc.workspace_bytes(n_tok, lyr.n_embd, lyr.ff, lyr.n_experts, lyr.used) > rc.NOALLOC_SCRATCH_BYTES
    x = torch.zeros((n_tok, lyr.n_embd), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((n_tok, lyr.n_embd), dtype=torch.float32, device="cuda")
    with pytest.raises(rc.DeviceError) as e:
        rc.moe_forward_noalloc(lyr.w, x, x, rc.BF16, n_tok, out)
    assert e.value.code == rc.ERR_WORKSPACE
