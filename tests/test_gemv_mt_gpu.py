"""The multi-token streaming kernel (hq4_gemv_mt.cu) behind the GEMV and
stage entry points for two or more fp32 tokens (passes of up to 8 tokens;
the one-token kernel's exact digit product, the tokens sharing each weight
fragment).

Bars:
  * against an fp64 evaluation of the exactly dequantised weights (the
    reference's float path, kernel/q4gemv.c:113-139 per token): relative L2
    <= 2e-6, the one-token kernel's own bar;
  * against the one-token kernel on the same inputs, token by token, for the
    fused epilogues (row add + residual, SiLU(gate) * up, q|k|v with RoPE and
    the cache writes): relative L2 <= 2e-6;
  * bit-identical repeated calls.
"""
import numpy as np
import pytest

from hetero_infer_b200 import synth

TOL = 2e-6


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def _linear(n_out, n_in, gs, seed, m):
    w, s, b = synth.q4_linear(seed, "w", n_out, n_in, gs)
    b = (np.random.default_rng(seed).standard_normal(b.shape) * 0.05).astype(np.float16)
    x = synth.activation(seed, "x", (m, n_in))
    return w, s, b, x


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("n_out,n_in,m", [(1024, 3584, 2), (3584, 18944, 5), (18944, 3584, 7),
                                          (4608, 3584, 13), (1000, 512, 3), (3584, 3584, 32)])
def test_tokens_match_fp64_and_one_token_kernel(oracle, cuda, n_out, n_in, m):
    import torch
    from hetero_infer_b200 import ops
    gs = 64
    w, s, b, x = _linear(n_out, n_in, gs, n_out + m, m)
    dw, ds, db, dx = _dev(w), _dev(s), _dev(b), _dev(x)
    ra = torch.randn(n_out, device="cuda")
    res = torch.randn(m, n_out, device="cuda")
    y = ops.q4_gemv_fused(dw, ds, db, dx, gs, row_add=ra, residual=res)
    y2 = ops.q4_gemv_fused(dw, ds, db, dx, gs, row_add=ra, residual=res)
    per = torch.stack([ops.q4_gemv_fused(dw, ds, db, dx[i:i + 1], gs, row_add=ra, residual=res[i:i + 1])[0]
                       for i in range(m)])
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "not deterministic"
    W = oracle.dequant(w, s, b, 0, n_out, gs).astype(np.float64)
    y64 = x.astype(np.float64) @ W.T + ra.double().cpu().numpy() + res.double().cpu().numpy()
    got = y.cpu().numpy()
    assert rel_l2(got, y64) <= TOL, f"vs fp64 {rel_l2(got, y64):.2e}"
    assert rel_l2(got, per.cpu().numpy()) <= TOL
    lib = __import__("hetero_infer_b200._lib", fromlist=["load"]).load()
    assert lib.hq4_device_status(0) & 1 == 0


@pytest.mark.gpu
@pytest.mark.parametrize("silu", [0, 1])
def test_norm_prologue_and_silu_epilogue(cuda, silu):
    """hq4_gemv_norm at 11 tokens (passes of 8 + 3) against one-token calls."""
    import torch
    from hetero_infer_b200 import _lib
    lib = _lib.load()
    n_out, n_in, gs, m, eps = 2 * 1024, 3584, 64, 11, 1e-6
    w, s, b, x = _linear(n_out, n_in, gs, 11 + silu, m)
    dw, ds, db, dx = _dev(w), _dev(s), _dev(b), _dev(x)
    nw = torch.rand(n_in, device="cuda") + 0.5
    n_store = n_out // 2 if silu else n_out
    out = torch.zeros(m, n_store, device="cuda")
    ref = torch.zeros(m, n_store, device="cuda")
    _lib.check(lib.hq4_gemv_norm(dw.data_ptr(), ds.data_ptr(), db.data_ptr(), dx.data_ptr(), out.data_ptr(),
                                 n_out, n_in, gs, m, nw.data_ptr(), eps, silu, None, None, _stream()), "norm")
    for i in range(m):
        _lib.check(lib.hq4_gemv_norm(dw.data_ptr(), ds.data_ptr(), db.data_ptr(), dx[i].data_ptr(),
                                     ref[i].data_ptr(), n_out, n_in, gs, 1, nw.data_ptr(), eps, silu, None, None,
                                     _stream()), "norm m=1")
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= TOL


@pytest.mark.gpu
def test_qkv_rope_tokens_match_one_token_calls(cuda):
    """hq4_qkv_rope at 6 tokens from position 3 against 6 one-token calls at
    positions 3..8: rotated q, and the k / v cache rows."""
    import torch
    from hetero_infer_b200 import _lib
    from hetero_infer_b200.cuda_model import rope_tables
    lib = _lib.load()
    nh, nkv, hd, n_in, gs, m, max_ctx, eps = 4, 2, 64, 512, 64, 6, 32, 1e-6
    n_out = (nh + 2 * nkv) * hd
    w, s, b, x = _linear(n_out, n_in, gs, 21, m)
    dw, ds, db, dx = _dev(w), _dev(s), _dev(b), _dev(x)
    nw = torch.rand(n_in, device="cuda") + 0.5
    bias = torch.randn(n_out, device="cuda") * 0.1
    cos, sin = (torch.from_numpy(np.ascontiguousarray(t)).float().cuda() for t in rope_tables(hd, 1e6, max_ctx))

    def run(tok_ids, pos0):
        q = torch.zeros(m, nh * hd, device="cuda")
        kc = torch.zeros(nkv, max_ctx, hd, device="cuda")
        vc = torch.zeros(nkv, max_ctx, hd, device="cuda")
        for i0, cnt in tok_ids:
            pos = torch.tensor([pos0 + i0], dtype=torch.int32, device="cuda")
            _lib.check(lib.hq4_qkv_rope(dw.data_ptr(), ds.data_ptr(), db.data_ptr(), dx[i0].data_ptr(), nh, nkv,
                                        hd, n_in, gs, cnt, nw.data_ptr(), eps, bias.data_ptr(), pos.data_ptr(),
                                        cos.data_ptr(), sin.data_ptr(), max_ctx, q[i0].data_ptr(), kc.data_ptr(),
                                        vc.data_ptr(), _stream()), "qkv_rope")
            torch.cuda.synchronize()
        return q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()

    got = run([(0, m)], 3)
    ref = run([(i, 1) for i in range(m)], 3)
    for a, r in zip(got, ref):
        assert rel_l2(a, r) <= TOL
    assert np.count_nonzero(got[1][:, 3:3 + m]) > 0 and np.count_nonzero(got[1][:, 3 + m:]) == 0
