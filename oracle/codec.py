"""NumPy restatement of the reference's int8 activation codec -- TEST
INFRASTRUCTURE ONLY (tests/ and the CPU pipeline oracle may use it; the
product path never imports anything under oracle/).

hetero/transport.py:198-225 (encode / decode, codec "int8"):
  encode: per row (last axis) scale = max|x| / 127 in fp32, an all-zero row's
          scale is 1; q = clip(rint(x / scale), -127, 127) as int8; the
          payload is the fp32 scales followed by the int8 rows.
  decode: (q as fp32 * scale) rounded to fp16.
Pinned against bytes the reference itself produced (tests/golden/
codec_i8.npz, written by tests/golden/make_codec_golden.py).
"""
from __future__ import annotations

import numpy as np


def encode_i8(x) -> bytes:
    """Payload of transport.encode(x, "int8") (the header carries the shape)."""
    a = np.asarray(x, dtype=np.float32)
    flat = a.reshape(-1, a.shape[-1])
    scale = np.abs(flat).max(axis=-1, keepdims=True) / np.float32(127.0)
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint(flat / scale), -127, 127).astype(np.int8)
    return scale.tobytes() + q.tobytes()


def decode_i8(payload: bytes, shape) -> np.ndarray:
    """transport.decode for codec "int8": fp16 array of `shape`."""
    shape = tuple(shape)
    rows = int(np.prod(shape[:-1]))
    scale = np.frombuffer(payload[:rows * 4], dtype=np.float32).reshape(rows, 1)
    q = np.frombuffer(payload[rows * 4:], dtype=np.int8).reshape(rows, shape[-1])
    with np.errstate(over="ignore"):  # |q*scale| > 65504 becomes inf, as in the reference
        return (q.astype(np.float32) * scale).reshape(shape).astype(np.float16)
