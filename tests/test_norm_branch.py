"""RMS norm (rvc_rms_norm, the rvh_rms_norm contract) and the MoE branch of a session.

CPU: the oracle's rms_norm against a numpy restatement of ops.rs:131-139 (f64 sum of squares,
f32 mean, scale and products) on seeded rows, edge widths included.

GPU (marked): rvc_rms_norm bit-exact against the oracle for the shapes the MoE branch uses and
for ragged widths (the scalar path); then the MoE branch as the HIP executor runs it
(runtime/src/hip_exec.rs:780-846): router input = rms_norm(o) * (1 / sqrt(n_embd)) *
gate_inp_scale, expert input = rms_norm(o) * pre_ffw_norm_2, the layer, and the post norm
rms_norm(moe) * post_ffw_norm_2, all on the device through the C ABI, against the same chain on
the oracle. Bars: expert ids exact; the branch output within max-rel 1e-3 per row.
"""
import numpy as np
import pytest

EPS = 1e-6


def np_rms_norm(x, w=None, eps=EPS, post=1.0):
    x = np.asarray(x, np.float32)
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        s = float(np.sum(x[r].astype(np.float64) ** 2))
        mean = np.float32(s / x.shape[1])
        scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(eps)), dtype=np.float32)
        v = (x[r] * scale).astype(np.float32)
        if post != 1.0:
            v = (v * np.float32(post)).astype(np.float32)
        if w is not None:
            v = (v * np.asarray(w, np.float32)).astype(np.float32)
        out[r] = v
    return out


@pytest.mark.parametrize("width", [1, 7, 2816])
def test_oracle_rms_norm_matches_ops_rs(oracle, width):
    rng = np.random.default_rng(width)
    x = (rng.standard_normal((5, width)) * 3).astype(np.float32)
    w = rng.uniform(0.5, 1.5, width).astype(np.float32)
    post = float(np.float32(1.0 / np.sqrt(np.float32(width))))
    for wt, p in [(None, 1.0), (w, 1.0), (w, post)]:
        assert np.array_equal(oracle.rms_norm(x, wt, EPS, p), np_rms_norm(x, wt, EPS, p))


def test_oracle_rms_norm_zero_row(oracle):
    x = np.zeros((2, 64), np.float32)
    assert np.array_equal(oracle.rms_norm(x), np.zeros_like(x))


# ------------------------------------------------------------------------ GPU
def _cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,width", [(1, 2816), (37, 2816), (16, 7), (3, 2818), (300, 64)])
def test_rms_norm_bit_exact(oracle, rows, width):
    import torch
    from rosevine_b200 import rvcuda as rc
    rng = np.random.default_rng(rows * 1000 + width)
    x = (rng.standard_normal((rows, width)) * 2).astype(np.float32)
    w = rng.uniform(0.5, 1.5, width).astype(np.float32)
    post = float(np.float32(1.0 / np.sqrt(np.float32(width))))
    xd, wd = _cuda(x), _cuda(w)
    for wt, p in [(None, 1.0), (w, 1.0), (w, post)]:
        out = torch.empty_like(xd)
        rc.rms_norm(xd, out, None if wt is None else wd, rows, width, EPS, p,
                    torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), oracle.rms_norm(x, wt, EPS, p)), (rows, width, wt is None, p)
    # in place (out = x), as the post norm is called
    inplace = xd.clone()
    rc.rms_norm(inplace, inplace, wd, rows, width, EPS, 1.0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(inplace.cpu().numpy(), oracle.rms_norm(x, w, EPS, 1.0))


@pytest.mark.gpu
def test_rms_norm_rejects_bad_arguments():
    import torch
    from rosevine_b200 import rvcuda as rc
    x = torch.zeros((4, 8), dtype=torch.float32, device="cuda")
    assert rc.lib().rvc_rms_norm(x.data_ptr(), x.data_ptr(), None, 0, 8, EPS, 1.0, None) == 1
    assert rc.lib().rvc_rms_norm(None, x.data_ptr(), None, 4, 8, EPS, 1.0, None) == 1
    assert rc.lib().rvc_rms_norm(x.data_ptr() + 2, x.data_ptr(), None, 4, 8, EPS, 1.0, None) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("n_tok", [1, 8, 96])
def test_moe_branch_session(oracle, pool, n_tok):
    """hip_exec.rs:786 (router input), :796 (expert input), the layer, :846 (post norm)."""
    import torch
    from rosevine_b200 import rvcuda as rc
    from rosevine_b200 import synth
    from rosevine_b200.moe import MoeLayer
    e = synth.N_EMBD
    rng = np.random.default_rng(500 + n_tok)
    o = (rng.standard_normal((n_tok, e)) * 4).astype(np.float32)  # the attention output (residual branch)
    g_scale = rng.uniform(0.5, 1.5, e).astype(np.float32)          # gate_inp_scale
    pre2 = rng.uniform(0.5, 1.5, e).astype(np.float32)             # pre_ffw_norm_2
    post2 = rng.uniform(0.5, 1.5, e).astype(np.float32)            # post_ffw_norm_2
    inv_sqrt = float(np.float32(1.0) / np.sqrt(np.float32(e)))
    gu, dn = synth.experts(2)
    w_router = synth.router(1)

    # CPU chain on the oracle
    rx = oracle.rms_norm(o, g_scale, EPS, inv_sqrt)
    mx = oracle.rms_norm(o, pre2, EPS, 1.0)
    want, want_ids, _, _ = oracle.moe_layer(pool, rx, mx, w_router, gu, dn)
    want = oracle.rms_norm(want, post2, EPS, 1.0)

    # the device chain through the C ABI
    layer = MoeLayer(w_router, gu, dn, max_tok=max(n_tok, 64))
    s = torch.cuda.current_stream().cuda_stream
    od, gd, pd, qd = _cuda(o), _cuda(g_scale), _cuda(pre2), _cuda(post2)
    router_x, moe_in = torch.empty_like(od), torch.empty_like(od)
    rc.rms_norm(od, router_x, gd, n_tok, e, EPS, inv_sqrt, s)
    rc.rms_norm(od, moe_in, pd, n_tok, e, EPS, 1.0, s)
    ids = torch.empty((n_tok, 8), dtype=torch.int32, device="cuda")
    moe = layer.forward(router_x, moe_in, ids=ids)
    rc.rms_norm(moe, moe, qd, n_tok, e, EPS, 1.0, s)
    layer.status()
    got = moe.cpu().numpy()
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    den = np.maximum(np.abs(want).max(axis=1), 1e-30)
    err = np.abs(got - want).max(axis=1) / den
    assert err.max() <= 1e-3, err.max()
