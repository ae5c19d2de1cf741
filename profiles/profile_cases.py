"""One small run of the kernels the ncu summaries in this directory cover
(this script is what those summaries' commands execute):

  layer   the four GEMV launches of a Qwen2-7B-shape layer at batch 1
          (q|k|v 4608x3584, o 3584x3584, gate|up 37888x3584, down 3584x18944),
          two warm-up rounds then one profiled round;
  gemm    hq4_gemm_w4a16 on 18944x3584 at 16 tokens (register-path kernel)
          and 256 tokens (tcgen05 kernel), bf16 activations.

Weights are seeded random int4 with the benchmark's scale/bias law.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from hetero_infer_b200 import _lib, ops  # noqa: E402

LAYER = [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate_up", 37888, 3584), ("down", 3584, 18944)]


def q4(n, k, g, dev):
    w = torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
    s = (torch.randn(n, k // 64, device=dev, generator=g).abs() * 0.01).half()
    return w, s, (s.float() * -8).half()


def main(which):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    if which in ("layer", "all"):
        mats = [(q4(n, k, g, dev), torch.randn(1, k, device=dev, generator=g), torch.empty(1, n, device=dev), n, k)
                for _, n, k in LAYER]
        for _ in range(3):
            for (w, s, b), x, y, n, k in mats:
                _lib.check(lib.hq4_gemv(w.data_ptr(), s.data_ptr(), b.data_ptr(), x.data_ptr(), y.data_ptr(),
                                        n, k, 64, 1, st), "hq4_gemv")
    if which in ("gemm", "all"):
        n, k = 18944, 3584
        w, s, b = q4(n, k, g, dev)
        for m in (16, 256):
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            for _ in range(3):
                ops.q4_gemm(w, s, b, x, 64)
    torch.cuda.synchronize()
    print("ok", lib.hq4_device_status(0))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "all")
