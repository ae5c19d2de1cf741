"""Allocation-free W4A16 GEMM entry point (hq4_gemm_w4a16_static).

The entry point is hq4_gemm_w4a16 with its workspace taken from a static
device area instead of a caller buffer.  Two consecutive calls on one stream
(sharing that area, queued without a synchronisation between them) must each
give exactly the output of the workspace entry point on the same inputs, on
both kernels behind it.  The file sorts last so that it also runs after every
other test has used the library.
"""
import numpy as np
import pytest

from hetero_infer_b200 import synth

STATIC_SCRATCH = 16 << 20  # HQ4_GEMM_STATIC_SCRATCH_BYTES in include/hq4.h


def _case(n_out, n_in, m, gs, seed, x_dtype):
    import torch
    rng = np.random.default_rng(seed)
    w, s, b = synth.q4_tensor(rng, n_out, n_in, gs)
    x = torch.from_numpy(rng.standard_normal((m, n_in), dtype=np.float32)).cuda().to(x_dtype)
    return (torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
            torch.from_numpy(b).cuda(), x)


def _static(lib, dw, ds, db, x, gs, out, row_add=None, residual=None):
    import torch
    n_out, n_in, m = dw.shape[0], x.shape[1], x.shape[0]
    return lib.hq4_gemm_w4a16_static(
        dw.data_ptr(), ds.data_ptr(), db.data_ptr(), x.data_ptr(), int(x.dtype == torch.float32),
        out.data_ptr(), n_out, n_in, gs, m,
        None if row_add is None else row_add.data_ptr(),
        None if residual is None else residual.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


CASES = [
    # n_out, n_in, m, gs, x dtype, fused epilogue
    (2048, 1024, 200, 64, "bf16", False),    # tcgen05 kernel
    (1024, 2048, 12, 64, "bf16", True),      # register-path kernel, bias + residual
    (3584, 18944, 256, 64, "bf16", False),   # down shape, K split, 9.25 MiB of scratch
    (640, 1536, 24, 128, "bf16", True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_static_scratch_two_calls_match_workspace_entry(cuda, ci):
    import torch
    from hetero_infer_b200 import _lib, ops
    lib = _lib.load()
    n_out, n_in, m, gs, xd, fused = CASES[ci]
    assert lib.hq4_gemm_workspace_bytes(n_out, n_in, m) <= STATIC_SCRATCH
    dt = torch.bfloat16 if xd == "bf16" else torch.float32
    cases = [_case(n_out, n_in, m, gs, seed=900 + 10 * ci + j, x_dtype=dt) for j in range(2)]
    extra = []
    for j in range(2):
        if fused:
            extra.append((torch.randn(n_out, device="cuda"), torch.randn(m, n_out, device="cuda")))
        else:
            extra.append((None, None))
    outs = [torch.full((m, n_out), float("nan"), device="cuda") for _ in range(2)]
    lib.hq4_device_status(1)
    for j in range(2):  # two consecutive calls, one stream, no sync in between
        dw, ds, db, x = cases[j]
        _lib.check(_static(lib, dw, ds, db, x, gs, outs[j], *extra[j]), "hq4_gemm_w4a16_static")
    torch.cuda.synchronize()
    assert lib.hq4_device_status(0) & 5 == 0
    for j in range(2):
        dw, ds, db, x = cases[j]
        ra, res = extra[j]
        ref = ops.q4_gemm(dw, ds, db, x, gs, row_add=ra, residual=res)
        torch.cuda.synchronize()
        assert torch.equal(outs[j], ref), f"call {j} differs from hq4_gemm_w4a16"


@pytest.mark.gpu
def test_static_scratch_rejects_oversize_and_bad_input(cuda):
    import torch
    from hetero_infer_b200 import _lib
    lib = _lib.load()
    n_out, n_in, m = 3584, 18944, 512
    assert lib.hq4_gemm_workspace_bytes(n_out, n_in, m) > STATIC_SCRATCH
    dw, ds, db, x = _case(n_out, n_in, m, 64, seed=5, x_dtype=torch.bfloat16)
    out = torch.zeros(m, n_out, device="cuda")
    assert _static(lib, dw, ds, db, x, 64, out) == -1
    xs = x[:8].contiguous()
    small = torch.zeros(8, n_out, device="cuda")
    assert _static(lib, dw, ds, db, xs, 96, small) == -1  # unsupported group size
    assert lib.hq4_gemm_w4a16_static(dw.data_ptr(), ds.data_ptr(), db.data_ptr(), xs.data_ptr() + 2, 0,
                                     small.data_ptr(), n_out, n_in, 64, 8, None, None,
                                     torch.cuda.current_stream().cuda_stream) == -2
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(small) == 0
