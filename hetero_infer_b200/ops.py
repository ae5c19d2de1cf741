"""Torch-facing wrappers of the hq4 kernels.

PyTorch provides device memory and the current CUDA stream; the arithmetic is
all in ``libhq4.so``.  Every op checks that its tensors are CUDA, contiguous and
of the dtype the C ABI expects, and raises instead of computing anything on the
CPU.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(t: torch.Tensor, name: str, dtype=None) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (no CPU fallback)")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")


def q4_gemv(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor,
            group_size: int = 64, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[m, n_out] = x[m, n_in] @ dequant(w).T`` on the GPU (hq4_gemv).

    w: uint32/int32 [n_out, n_in/8]; scales, biases: fp16 [n_out, n_in/gs];
    x: fp32 [..., n_in]."""
    lib = _lib.load()
    _need_cuda(w, "w")
    if w.dtype not in (torch.int32, torch.uint32):
        raise RuntimeError("w must hold packed uint32 words")
    _need_cuda(scales, "scales", torch.float16)
    _need_cuda(biases, "biases", torch.float16)
    n_out, n_in = w.shape[0], w.shape[1] * 8
    xf = x.reshape(-1, n_in)
    _need_cuda(xf, "x", torch.float32)
    m = xf.shape[0]
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.float32, device=x.device)
    _need_cuda(out, "out", torch.float32)
    rc = lib.hq4_gemv(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), xf.data_ptr(),
                      out.data_ptr(), n_out, n_in, group_size, m, _stream_ptr(x.device))
    _lib.check(rc, "hq4_gemv")
    return out.reshape(*x.shape[:-1], n_out)


def q4_gemv_fused(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor,
                  group_size: int = 64, row_add: Optional[torch.Tensor] = None,
                  residual: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GEMV with the bias / residual add fused into its store (hq4_gemv_fused).

    ``out`` may alias ``residual`` (in-place residual update) but not ``x``."""
    lib = _lib.load()
    _need_cuda(w, "w")
    _need_cuda(scales, "scales", torch.float16)
    _need_cuda(biases, "biases", torch.float16)
    n_out, n_in = w.shape[0], w.shape[1] * 8
    xf = x.reshape(-1, n_in)
    _need_cuda(xf, "x", torch.float32)
    m = xf.shape[0]
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.float32, device=x.device)
    _need_cuda(out, "out", torch.float32)
    ra = 0
    if row_add is not None:
        _need_cuda(row_add, "row_add", torch.float32)
        ra = row_add.data_ptr()
    rs = 0
    if residual is not None:
        _need_cuda(residual, "residual", torch.float32)
        rs = residual.data_ptr()
    rc = lib.hq4_gemv_fused(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), xf.data_ptr(),
                            out.data_ptr(), n_out, n_in, group_size, m, ra or None, rs or None,
                            _stream_ptr(x.device))
    _lib.check(rc, "hq4_gemv_fused")
    return out.reshape(*x.shape[:-1], n_out)


def q4_dequant(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, row0: int, row1: int,
               group_size: int = 64, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 expansion of rows [row0, row1) (hq4_dequant)."""
    lib = _lib.load()
    _need_cuda(w, "w")
    _need_cuda(scales, "scales", torch.float16)
    _need_cuda(biases, "biases", torch.float16)
    n_in = w.shape[1] * 8
    rows = max(row1 - row0, 0)
    if out is None:
        out = torch.empty((rows, n_in), dtype=torch.float32, device=w.device)
    _need_cuda(out, "out", torch.float32)
    rc = lib.hq4_dequant(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), out.data_ptr(),
                         row0, row1, n_in, group_size, _stream_ptr(w.device))
    _lib.check(rc, "hq4_dequant")
    return out


_WORKSPACES = {}


def gemm_workspace(n_out: int, n_in: int, m: int, device: torch.device) -> torch.Tensor:
    """A grow-only per-device workspace large enough for hq4_gemm_w4a16 on
    this shape.  Callers that capture CUDA graphs should take it before
    capturing and pass it explicitly."""
    lib = _lib.load()
    need = int(lib.hq4_gemm_workspace_bytes(n_out, n_in, m))
    if need < 0:
        raise RuntimeError(f"hq4_gemm_workspace_bytes({n_out}, {n_in}, {m}) = {need}")
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", key))
        _WORKSPACES[key] = ws
    return ws


def q4_gemm(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor,
            group_size: int = 64, row_add: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None,
            workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """W4A16 GEMM on the tcgen05 tensor cores (hq4_gemm_w4a16):
    ``out[m, n_out] = x[m, n_in] @ dequant(w).T`` with x bf16 or fp32 and an
    fp32 result, for token counts where the product is a dense contraction."""
    lib = _lib.load()
    _need_cuda(w, "w")
    if w.dtype not in (torch.int32, torch.uint32):
        raise RuntimeError("w must hold packed uint32 words")
    _need_cuda(scales, "scales", torch.float16)
    _need_cuda(biases, "biases", torch.float16)
    n_out, n_in = w.shape[0], w.shape[1] * 8
    xf = x.reshape(-1, n_in)
    _need_cuda(xf, "x")
    if xf.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"x must be bfloat16 or float32, got {xf.dtype}")
    m = xf.shape[0]
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.float32, device=x.device)
    _need_cuda(out, "out", torch.float32)
    ra = 0
    if row_add is not None:
        _need_cuda(row_add, "row_add", torch.float32)
        ra = row_add.data_ptr()
    rs = 0
    if residual is not None:
        _need_cuda(residual, "residual", torch.float32)
        rs = residual.data_ptr()
    if workspace is None:
        workspace = gemm_workspace(n_out, n_in, m, x.device)
    _need_cuda(workspace, "workspace", torch.uint8)
    rc = lib.hq4_gemm_w4a16(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), xf.data_ptr(),
                            1 if xf.dtype == torch.float32 else 0, out.data_ptr(), n_out, n_in,
                            group_size, m, ra or None, rs or None, workspace.data_ptr(), workspace.numel(),
                            _stream_ptr(x.device))
    _lib.check(rc, "hq4_gemm_w4a16")
    return out.reshape(*x.shape[:-1], n_out)


def gemm_plan(n_out: int, n_in: int, m: int, x_is_f32: bool = False) -> dict:
    """The launch plan hq4_gemm_w4a16 uses for a shape (host only)."""
    import ctypes
    lib = _lib.load()
    info = (ctypes.c_int * 8)()
    _lib.check(lib.hq4_gemm_plan(n_out, n_in, m, 1 if x_is_f32 else 0, info), "hq4_gemm_plan")
    keys = ("row_tiles", "ksplit", "token_tiles", "tile_tokens", "stages", "smem", "weight_slots", "kernel")
    d = dict(zip(keys, list(info)))
    d["kernel"] = {0: "tcgen05", 1: "mma.sync", 2: "gemv", 3: "gemv_mt"}[d["kernel"]]
    return d


def act_encode_i8(x: torch.Tensor, payload: Optional[torch.Tensor] = None, wire: bool = False) -> torch.Tensor:
    """int8 wire payload of fp32 activations [..., cols] (hetero/transport.py:198-211):
    the rows' fp32 scales then the int8 rows, as a uint8 tensor.  wire=True
    rounds every value to fp16 first, as the reference's engine encodes the
    fp16 array its backend's to_wire made (hetero/engine.py:97)."""
    xs = x.contiguous()
    cols = int(xs.shape[-1])
    rows = xs.numel() // cols
    if payload is None:
        payload = torch.empty(rows * (4 + cols), dtype=torch.uint8, device=xs.device)
    lib = _lib.load()
    fn, name = (lib.hq4_act_encode_i8_wire, "hq4_act_encode_i8_wire") if wire else \
        (lib.hq4_act_encode_i8, "hq4_act_encode_i8")
    _lib.check(fn(xs.data_ptr(), rows, cols, payload.data_ptr(), torch.cuda.current_stream(xs.device).cuda_stream),
               name)
    return payload


def act_decode_i8(payload: torch.Tensor, rows: int, cols: int, dtype=torch.float16,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Activations [rows, cols] from an int8 wire payload (hetero/transport.py:214-225):
    fp16(q * scale), or that value widened to fp32 when dtype is float32."""
    if out is None:
        out = torch.empty((rows, cols), dtype=dtype, device=payload.device)
    lib = _lib.load()
    f16 = out.data_ptr() if out.dtype == torch.float16 else None
    f32 = out.data_ptr() if out.dtype == torch.float32 else None
    _lib.check(lib.hq4_act_decode_i8(payload.data_ptr(), rows, cols, f16, f32,
                                     torch.cuda.current_stream(payload.device).cuda_stream), "hq4_act_decode_i8")
    return out
