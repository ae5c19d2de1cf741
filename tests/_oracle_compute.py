"""CPU compute for the pipeline runner -- TEST INFRASTRUCTURE ONLY.

``OracleCompute`` has the interface of ``pipeline.DeviceCompute`` and runs a
stage with the NumPy stage oracle (``oracle/stage.py``), so the pipeline
schedule and its communication run under gloo ranks without a GPU.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch


class OracleCompute:
    """The same on the CPU with the NumPy stage oracle (test infrastructure:
    lets the schedule and communication run under gloo without a GPU)."""

    def __init__(self, cfg: dict, start: int, end: int, weights: Dict[str, np.ndarray], head_rows: tuple,
                 embed_rows=None, wire: str = "float16"):
        if wire not in ("float16", "int8"):
            raise ValueError(f"wire must be float16 or int8, not {wire!r}")
        self.wire = wire
        self.wire_dtype = torch.uint8 if wire == "int8" else torch.float16
        from oracle import stage as ost
        self.cfg, self.hidden_dim = cfg, cfg["hidden_size"]
        self.stage = ost.OracleStage(cfg, weights, start, end, start == 0, False, embed_rows=embed_rows)
        lo, hi = head_rows
        self.lo = lo
        self.norm_w = np.asarray(weights["model.norm.weight"], np.float32)
        self.lm = ost.OLinear(self.stage.orc, weights["lm_head.weight"][lo:hi], weights["lm_head.scales"][lo:hi],
                              weights["lm_head.biases"][lo:hi], None, cfg["quantization"]["group_size"])
        self._ost = ost

    def new_cache(self):
        return self.stage.new_caches()

    def embed_forward(self, ids, cache):
        return self.stage(ids, cache, apply_head=False)

    def forward(self, h, cache):
        return self.stage(h, cache, apply_head=False)

    def decode_tick(self, m, cache, src, first: bool, last: bool):
        h = self.embed_forward(src, cache) if first else self.forward(self.from_wire(src), cache)
        return (None if last else self.to_wire(h)), h

    def wire_empty(self, rows: int) -> torch.Tensor:
        if self.wire == "int8":
            return torch.empty(rows * (4 + self.hidden_dim), dtype=torch.uint8)
        return torch.empty((1, rows, self.hidden_dim), dtype=torch.float16)

    def to_wire(self, h):
        if self.wire == "int8":
            from oracle import codec
            # the reference's engine encodes its backend's fp16 wire array (engine.py:97)
            h16 = np.asarray(h, np.float16).astype(np.float32)
            return torch.frombuffer(bytearray(codec.encode_i8(h16)), dtype=torch.uint8)
        return torch.from_numpy(np.ascontiguousarray(np.asarray(h, dtype=np.float16)))

    def from_wire(self, t):
        if self.wire == "int8":
            from oracle import codec
            rows = t.numel() // (4 + self.hidden_dim)
            return codec.decode_i8(t.numpy().tobytes(), (1, rows, self.hidden_dim)).astype(np.float32)
        return t.numpy().astype(np.float32)

    def to_comm32(self, h):
        return torch.from_numpy(np.ascontiguousarray(np.asarray(h, np.float32).reshape(-1, self.hidden_dim)[-1]))

    def head(self, h32):
        x = self._ost.rms_norm(h32.numpy().reshape(1, 1, -1), self.norm_w, self.cfg["rms_norm_eps"])
        z = self.lm(x).reshape(-1)
        i = int(z.argmax())
        return float(z[i]), self.lo + i
