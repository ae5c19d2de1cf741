"""Pin the oracle: our C restatement (oracle/q4_oracle.c) must agree bit for bit
with the reference's kernel/q4gemv.c compiled from its own source (float and
AVX2 variants, oracle/_ref/), and with the committed golden vectors that were
produced by the reference itself (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from hetero_infer_b200 import synth
from oracle import q4

CASES = [(64, 512, 64, 1), (300, 3584, 64, 2), (37, 1024, 128, 3), (128, 18944, 64, 4),
         (1, 64, 64, 5), (33, 256, 256, 6)]


def _case(n_out, n_in, gs, seed, general):
    w, s, b = synth.q4_linear(seed, "w", n_out, n_in, gs)
    if general:
        b = (np.random.default_rng(seed).standard_normal(b.shape) * 0.05).astype(np.float16)
    x = synth.activation(seed, "x", (n_in,))
    return w, s, b, x


@pytest.mark.parametrize("n_out,n_in,gs,seed", CASES)
@pytest.mark.parametrize("general", [False, True])
def test_oracle_matches_reference_build(oracle, n_out, n_in, gs, seed, general):
    avail = q4.available_ref_variants()
    if not avail:
        pytest.skip("reference kernel not built here (oracle/_ref); golden tests cover it")
    w, s, b, x = _case(n_out, n_in, gs, seed, general)
    if "float" in avail:
        ref = q4.RefKernel("float").gemv(w, s, b, x, gs)
        assert np.array_equal(oracle.gemv_f32(w, s, b, x, gs), ref)
        assert np.array_equal(oracle.dequant(w, s, b, 0, n_out, gs),
                              q4.RefKernel("float").dequant(w, s, b, 0, n_out, gs))
    if "avx2" in avail:
        ref = q4.RefKernel("avx2").gemv(w, s, b, x, gs)
        assert np.array_equal(oracle.gemv_i16(w, s, b, x, gs, contract=1), ref)
        assert np.array_equal(oracle.dequant(w, s, b, 0, n_out, gs),
                              q4.RefKernel("avx2").dequant(w, s, b, 0, n_out, gs))


def test_oracle_error_codes(oracle):
    w, s, b, x = _case(8, 128, 64, 1, False)
    with pytest.raises(RuntimeError, match="-1"):
        oracle.gemv_f32(w, s, b, x[:128], 48)   # n_in % gs


def test_dequant_is_affine_exact(oracle):
    """q*scale is exact in fp32, so dequant == (q-8)*scale bit for bit when
    bias = -8*scale (the benchmark distribution)."""
    w, s, b, _ = _case(16, 256, 64, 9, False)
    got = oracle.dequant(w, s, b, 0, 16, 64)
    q = ((w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(16, 256)
    want = (q.astype(np.float32) - 8.0) * np.repeat(s.astype(np.float32), 64, axis=1)
    assert np.array_equal(got, want)
