"""W4A16 tcgen05 GEMM (hq4_gemm_w4a16) on the GPU.

Four kernels sit behind the entry point (hq4_gemm_plan says which):
* multi-token streaming kernel (2..8 tokens where its x image fits): the
  one-token kernel's exact digit product -- checked against the full-
  precision product (the reference's float path, out = x . (q*s+b)^T,
  hetero/cpu_model.py QLinear, kernel/q4gemv.c:113-139 per token) to 2e-6;
* register path (the other token counts up to 16 bf16 / 8 fp32): weights
  exact, fp32 x as bf16 hi + lo -- checked against the full-precision
  product to 2e-5 (bf16 x) / 5e-5 (fp32 x);
* one token: hq4_gemv's streaming kernel (weights exact, x widened to fp32)
  -- the register path's bars;
* tcgen05 path: weights rounded once to fp16, x to fp16 -- checked against
  that exact fp16-operand product in float64 (<= 1e-5: only fp32
  accumulation order differs) and against the full-precision product at the
  north star's 1e-3 relative L2 (fp16 weight rounding costs ~3e-4).
"""
import numpy as np
import pytest

from hetero_infer_b200 import synth

EXACT_TOL = 1e-5
SPEC_TOL = 1e-3
MT_TOL = 4e-6


def rel_l2(a, b):
    import torch
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def _case(n_out, n_in, m, gs, seed, x_dtype):
    import torch
    rng = np.random.default_rng(seed)
    w, s, b = synth.q4_tensor(rng, n_out, n_in, gs)
    x = torch.from_numpy(rng.standard_normal((m, n_in), dtype=np.float32)).cuda().to(x_dtype)
    dw = torch.from_numpy(w.view(np.int32)).cuda()
    ds = torch.from_numpy(s).cuda()
    db = torch.from_numpy(b).cuda()
    return dw, ds, db, x


def _dequant64(dw, ds, db, gs):
    """(q*s+b) in float64 on the device, [n_out, n_in] (exact)."""
    import torch
    n_out, wpr = dw.shape
    wu = dw.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, device=dw.device, dtype=torch.int64) * 4
    q = ((wu.unsqueeze(-1) >> shifts) & 0xF).reshape(n_out, wpr * 8).double()
    s = ds.double().repeat_interleave(gs, dim=1)
    b = db.double().repeat_interleave(gs, dim=1)
    return q * s + b


def _refs(dw, ds, db, x, gs):
    import torch
    w64 = _dequant64(dw, ds, db, gs)
    x64 = x.double()
    exact = x.float().half().double() @ w64.half().double().T
    spec = x64 @ w64.T
    return exact, spec


SHAPES = [
    # n_out, n_in, m, gs, x dtype
    (128, 64, 1, 64, "bf16"),
    (256, 512, 7, 64, "bf16"),
    (384, 1024, 16, 128, "bf16"),
    (1000, 256, 33, 64, "bf16"),          # ragged row tile
    (512, 3584, 300, 64, "bf16"),         # two token tiles, K split over a cluster
    (18944, 3584, 64, 64, "bf16"),        # gate/up, config 3
    (18944, 3584, 256, 64, "bf16"),       # gate/up, config 3, tensor-bound
    (3584, 18944, 256, 64, "bf16"),       # down, config 3, K split
    (3584, 18944, 4, 64, "bf16"),
    (4608, 3584, 48, 256, "f32"),
    (3584, 3584, 128, 64, "f32"),
    (1024, 2048, 6, 64, "f32"),           # multi-token kernel, fp32 x
    (1024, 2048, 12, 64, "bf16"),         # register path
    (2048, 4096, 32, 64, "bf16"),         # tcgen05 path, 32 tokens
    (3584, 18944, 7, 128, "f32"),         # register path, K split, gs 128
    (18944, 3584, 1, 64, "bf16"),         # one token: the streaming GEMV
    (3584, 18944, 1, 64, "f32"),          # one token, fp32 x
    (512, 1024, 1, 128, "bf16"),          # one token, gs 128
    (18944, 3584, 4, 64, "bf16"),         # multi-token kernel, config 3
    (18944, 3584, 8, 64, "bf16"),         # multi-token kernel, three column tiles
    (3584, 18944, 4, 64, "bf16"),         # multi-token kernel, K split over a cluster
    (3584, 18944, 8, 64, "f32"),
    (4608, 3584, 5, 64, "f32"),
    (1000, 512, 3, 64, "f32"),            # ragged last strip
    (256, 2048, 6, 256, "bf16"),          # scale groups of 256
    (512, 2048, 7, 128, "f32"),           # scale groups of 128
]


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(SHAPES)))
def test_gemm_matches_exact_and_reference(cuda, ci):
    import torch
    from hetero_infer_b200 import ops
    n_out, n_in, m, gs, xd = SHAPES[ci]
    dw, ds, db, x = _case(n_out, n_in, m, gs, seed=100 + ci,
                          x_dtype=torch.bfloat16 if xd == "bf16" else torch.float32)
    y = ops.q4_gemm(dw, ds, db, x, gs)
    torch.cuda.synchronize()
    exact, spec = _refs(dw, ds, db, x, gs)
    plan = ops.gemm_plan(n_out, n_in, m, xd == "f32")
    e1, e2 = rel_l2(y, exact), rel_l2(y, spec)
    if plan["kernel"] == "gemv_mt":
        assert e2 <= MT_TOL, f"{SHAPES[ci]}: vs full precision {e2:.2e} ({plan})"
    elif plan["kernel"] in ("mma.sync", "gemv"):
        assert e2 <= (5e-5 if xd == "f32" else 2e-5), f"{SHAPES[ci]}: vs full precision {e2:.2e} ({plan})"
    else:
        assert e1 <= EXACT_TOL, f"{SHAPES[ci]}: vs fp16-operand product {e1:.2e} ({plan})"
        assert e2 <= SPEC_TOL, f"{SHAPES[ci]}: vs reference {e2:.2e}"
    y2 = ops.q4_gemm(dw, ds, db, x, gs)
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "not deterministic"


@pytest.mark.gpu
@pytest.mark.parametrize("m", [6, 24])
def test_gemm_row_add_residual_and_reference_oracle(cuda, oracle, m):
    """Fused bias + residual in the store, on both kernels; and the full-
    precision reference taken from the C oracle of q4gemv.c's float path
    itself (per token)."""
    import torch
    from hetero_infer_b200 import ops
    n_out, n_in, gs = 640, 1536, 64
    dw, ds, db, x = _case(n_out, n_in, m, gs, seed=7, x_dtype=torch.bfloat16)
    ra = torch.randn(n_out, device="cuda")
    res = torch.randn(m, n_out, device="cuda")
    y = ops.q4_gemm(dw, ds, db, x, gs, row_add=ra, residual=res)
    exact, spec = _refs(dw, ds, db, x, gs)
    if ops.gemm_plan(n_out, n_in, m)["kernel"] in ("mma.sync", "gemv_mt"):
        assert rel_l2(y, spec + ra.double() + res.double()) <= 2e-5
    else:
        assert rel_l2(y, exact + ra.double() + res.double()) <= EXACT_TOL
    w = dw.cpu().numpy().view(np.uint32)
    s = ds.cpu().numpy()
    b = db.cpu().numpy()
    xs = x.float().cpu().numpy()
    ref = oracle.gemv_f32(w, s, b, xs, gs)
    got = (y - ra - res).cpu().numpy()
    assert float(np.linalg.norm(got - ref) / np.linalg.norm(ref)) <= SPEC_TOL


@pytest.mark.gpu
def test_gemm_error_codes(cuda):
    import torch
    from hetero_infer_b200 import _lib
    lib = _lib.load()
    dw, ds, db, x = _case(256, 512, 8, 64, seed=1, x_dtype=torch.bfloat16)
    out = torch.empty(8, 256, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    need = lib.hq4_gemm_workspace_bytes(256, 512, 8)
    assert 0 < need <= 1 << 20
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    call = lambda xp, gs, n_in=512, wsb=need: lib.hq4_gemm_w4a16(
        dw.data_ptr(), ds.data_ptr(), db.data_ptr(), xp, 0, out.data_ptr(), 256, n_in, gs, 8, None, None,
        ws.data_ptr(), wsb, st)
    assert call(x.data_ptr(), 32) == -1          # gs below 64 (q4gemv.c:234-240 AVX2 rule)
    assert call(x.data_ptr(), 96) == -1          # not a power of two
    assert call(x.data_ptr(), 64, n_in=500) == -1
    assert call(x.data_ptr(), 64, wsb=1024) == -1       # workspace too small
    assert call(x.data_ptr() + 2, 64) == -2      # x not 16-byte aligned
    assert call(x.data_ptr(), 64) == 0
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) & 5 == 0


@pytest.mark.gpu
def test_gemm_range_flag(cuda):
    """The tcgen05 path carries x in fp16: bf16 activations beyond fp16 range
    set status bit 2 (no silent inf).  The register and multi-token paths
    keep bf16 and compute such inputs exactly, with no flag."""
    import torch
    from hetero_infer_b200 import _lib, ops
    lib = _lib.load()
    dw, ds, db, x = _case(256, 512, 80, 64, seed=2, x_dtype=torch.bfloat16)
    assert ops.gemm_plan(256, 512, 80)["kernel"] == "tcgen05"
    lib.hq4_device_status(1)
    ops.q4_gemm(dw, ds, db, x, 64)
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) & 4 == 0
    x[3, 100] = 1e6
    ops.q4_gemm(dw, ds, db, x, 64)
    torch.cuda.synchronize()
    assert lib.hq4_device_status(1) & 4
    xs = x[:8].contiguous()
    assert ops.gemm_plan(256, 512, 8)["kernel"] in ("mma.sync", "gemv_mt")
    y = ops.q4_gemm(dw, ds, db, xs, 64)
    torch.cuda.synchronize()
    assert lib.hq4_device_status(1) & 4 == 0
    _, spec = _refs(dw, ds, db, xs, 64)
    assert rel_l2(y, spec) <= 2e-5


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(18944, 3584, 256), (3584, 18944, 256), (2048, 1024, 200), (4096, 2048, 40)])
def test_gemm_back_to_back_calls(cuda, shape):
    """Calls queued back to back on one stream (the next launch overlapping the
    previous one's tail), rotating weights, one shared workspace: every
    output equals its own exact product."""
    import torch
    from hetero_infer_b200 import ops
    n_out, n_in, m = shape
    cases = [_case(n_out, n_in, m, 64, seed=300 + j, x_dtype=torch.bfloat16) for j in range(3)]
    ws = ops.gemm_workspace(n_out, n_in, m, torch.device("cuda"))
    outs = []
    for rep in range(2):
        for dw, ds, db, x in cases:
            outs.append(ops.q4_gemm(dw, ds, db, x, 64, workspace=ws))
    torch.cuda.synchronize()
    small = ops.gemm_plan(n_out, n_in, m)["kernel"] in ("mma.sync", "gemv_mt")
    for j, y in enumerate(outs):
        dw, ds, db, x = cases[j % 3]
        exact, spec = _refs(dw, ds, db, x, 64)
        assert rel_l2(y, spec if small else exact) <= (2e-5 if small else EXACT_TOL), f"call {j}"
