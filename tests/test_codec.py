"""The int8 activation codec (hetero/transport.py:198-225).

The oracle (oracle/codec.py) is pinned to bytes the reference produced
(tests/golden/codec_i8.npz); the device kernels (hq4_act_encode_i8 /
hq4_act_decode_i8) must reproduce those bytes and values exactly."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "codec_i8.npz")


def _golden():
    g = np.load(GOLDEN)
    names = sorted({k.rsplit(".", 1)[0] for k in g.files})
    return [(n, g[f"{n}.x"], g[f"{n}.payload"].tobytes(), g[f"{n}.decoded"]) for n in names]


@pytest.mark.parametrize("case", _golden(), ids=lambda c: c[0])
def test_oracle_matches_reference_bytes(case):
    from oracle import codec
    name, x, payload, decoded = case
    assert codec.encode_i8(x) == payload
    y = codec.decode_i8(payload, x.shape)
    assert y.dtype == np.float16 and np.array_equal(y.view(np.uint16), decoded.view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("case", _golden(), ids=lambda c: c[0])
def test_device_codec_matches_reference_bytes(cuda, case):
    import torch
    from hetero_infer_b200 import ops
    name, x, payload, decoded = case
    cols = x.shape[-1]
    rows = x.size // cols
    p = ops.act_encode_i8(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert p.cpu().numpy().tobytes() == payload
    y16 = ops.act_decode_i8(p, rows, cols).cpu().numpy()
    y32 = ops.act_decode_i8(p, rows, cols, dtype=torch.float32).cpu().numpy()
    ref = decoded.reshape(rows, cols)
    assert np.array_equal(y16.view(np.uint16), ref.view(np.uint16))
    assert np.array_equal(y32, ref.astype(np.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 3584), (37, 513), (1, 18944)])
def test_device_codec_random_matches_oracle(cuda, rows, cols):
    import torch
    from hetero_infer_b200 import ops
    from oracle import codec
    x = (np.random.default_rng(rows * cols).standard_normal((rows, cols)) * 7).astype(np.float32)
    p = ops.act_encode_i8(torch.from_numpy(x).cuda())
    assert p.cpu().numpy().tobytes() == codec.encode_i8(x)
    y = ops.act_decode_i8(p, rows, cols).cpu().numpy()
    assert np.array_equal(y.view(np.uint16), codec.decode_i8(codec.encode_i8(x), x.shape).view(np.uint16))


@pytest.mark.gpu
def test_device_codec_rejects_bad_arguments(cuda):
    import torch
    from hetero_infer_b200 import _lib
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(16, device="cuda")
    p = torch.zeros(64, dtype=torch.uint8, device="cuda")
    assert lib.hq4_act_encode_i8(x.data_ptr(), 0, 16, p.data_ptr(), st) == -1
    assert lib.hq4_act_decode_i8(p.data_ptr(), 1, 16, None, None, st) == -1
    assert lib.hq4_act_encode_i8(x.data_ptr() + 2, 1, 4, p.data_ptr(), st) == -2


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(1, 3584), (6, 513), (2, 256)])
def test_device_wire_encode_rounds_through_fp16(cuda, rows, cols):
    """hq4_act_encode_i8_wire gives the bytes of the reference engine's int8
    frame, transport.encode(backend.to_wire(y), "int8") (hetero/engine.py:97):
    the fp32 state rounded to fp16 first, then the codec.  Values are spread
    so the fp16 rounding changes the scales and some of the int8 digits."""
    import torch
    from hetero_infer_b200 import ops
    from oracle import codec
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-3, 9, (rows, 1)))).astype(np.float32)
    ref = codec.encode_i8(x.astype(np.float16).astype(np.float32))
    assert ref != codec.encode_i8(x)  # the case distinguishes the two encodings
    p = ops.act_encode_i8(torch.from_numpy(x).cuda(), wire=True)
    assert p.cpu().numpy().tobytes() == ref
