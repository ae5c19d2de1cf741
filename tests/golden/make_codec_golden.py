"""Golden vectors of the reference's int8 activation codec.

Imports the reference's hetero/transport.py unmodified (build container only:
the reference tree is not on the GPU box) and records, for a set of inputs,
what its encode(x, "int8") payload and decode(...) output are.  The tests
read tests/golden/codec_i8.npz.

  python tests/golden/make_codec_golden.py [REFERENCE_ROOT]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def cases():
    rng = np.random.default_rng(11)
    out = {}
    out["normal_3x3584"] = rng.standard_normal((1, 3, 3584)).astype(np.float32)
    out["wide_range_2x1000"] = (rng.standard_normal((2, 1000)) * np.array([[1e-3], [3e4]])).astype(np.float32)
    z = rng.standard_normal((4, 256)).astype(np.float32)
    z[1] = 0.0                                          # all-zero row: scale 1
    z[2] = 0.0
    z[2, 17] = -5.0                                     # one non-zero element
    out["zero_rows_4x256"] = z
    t = np.zeros((1, 128), np.float32)
    t[0, 0] = 127.0                                     # scale exactly 1: halves tie to even
    t[0, 1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5]
    out["ties_1x128"] = t
    out["tiny_1x64"] = (rng.standard_normal((1, 64)) * 1e-30).astype(np.float32)   # subnormal scale
    out["hidden_7b_like_1x1x3584"] = (rng.standard_normal((1, 1, 3584)) * 40.0).astype(np.float32)
    return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.sep, "root", "reference")
    sys.path.insert(0, ref_root)
    from hetero import transport
    save = {}
    for name, x in cases().items():
        header, payload = transport.encode(x, "int8")
        assert header["shape"] == list(x.shape)
        y = transport.decode(header, payload)
        save[f"{name}.x"] = x
        save[f"{name}.payload"] = np.frombuffer(payload, np.uint8)
        save[f"{name}.decoded"] = y
    np.savez(os.path.join(HERE, "codec_i8.npz"), **save)
    print("wrote", len(save) // 3, "cases")


if __name__ == "__main__":
    main()
