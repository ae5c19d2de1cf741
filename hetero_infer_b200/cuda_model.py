"""The qwen2 stage on the GPU: the device-side counterpart of the reference's
NumPy model (hetero/cpu_model.py).

This module starts with the quantised linear layer, ``QLinear``, whose
constructor and call signature are the reference's
(``hetero/cpu_model.py:84-158``): packed MLX-layout weights in, activations in,
activations out.  Weights are uploaded once to HBM; every product runs in
``libhq4.so``.  Host (NumPy) inputs are staged through pinned memory and come
back as NumPy arrays, so code written against the reference's QLinear runs
unchanged; CUDA tensors in give CUDA tensors out, which is what the device
stage uses.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import ops


def _dev_array(a, dtype=None, device="cuda"):
    """NumPy (or torch) array -> contiguous CUDA tensor; uint32 travels as int32."""
    if isinstance(a, torch.Tensor):
        t = a
    else:
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        t = torch.from_numpy(a)
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device).contiguous()


class _Pinned:
    """Grow-only pinned host buffers keyed by name (host<->device staging)."""

    def __init__(self):
        self.bufs = {}

    def get(self, name: str, shape, dtype) -> torch.Tensor:
        n = int(np.prod(shape))
        b = self.bufs.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(max(n, 1), dtype=dtype, pin_memory=True)
            self.bufs[name] = b
        return b[:n].view(*shape)


class QLinear:
    """Weights stay 4-bit in HBM; the fused int4 GEMV reads them once per token.

    Same constructor as ``hetero/cpu_model.py:96``.  ``bits`` must be 4 (the
    only width the device kernels read); the reference falls back to an fp32
    expansion for other widths, this class raises instead."""

    def __init__(self, w, scales, biases, bias, group_size, bits, device="cuda"):
        if bits != 4:
            raise NotImplementedError("device QLinear reads 4-bit packed weights only")
        self.group_size, self.bits = int(group_size), int(bits)
        self.n_out, self.n_in = int(w.shape[0]), int(w.shape[1]) * (32 // bits)
        self.device = torch.device(device)
        self.w = _dev_array(w, device=self.device)
        self.scales = _dev_array(scales, torch.float16, self.device)
        self.biases = _dev_array(biases, torch.float16, self.device)
        self.bias = None if bias is None else _dev_array(bias, torch.float32, self.device)
        self._pinned = _Pinned()

    def forward_device(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                       residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """CUDA fp32 [..., n_in] -> CUDA fp32 [..., n_out] (+ bias, + residual)."""
        return ops.q4_gemv_fused(self.w, self.scales, self.biases, x.contiguous(),
                                 self.group_size, self.bias, residual, out)

    def __call__(self, x):
        if isinstance(x, torch.Tensor) and x.is_cuda:
            return self.forward_device(x)
        # host path: NumPy in, NumPy out (the reference's calling convention)
        xa = np.asarray(x, dtype=np.float32)
        lead = xa.shape[:-1]
        flat = xa.reshape(-1, self.n_in)
        h_in = self._pinned.get("x", flat.shape, torch.float32)
        h_in.numpy()[...] = flat
        d_in = h_in.to(self.device, non_blocking=True)
        d_out = self.forward_device(d_in)
        h_out = self._pinned.get("y", (flat.shape[0], self.n_out), torch.float32)
        h_out.copy_(d_out, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return h_out.numpy().copy().reshape(*lead, self.n_out)
