"""ctypes binding of ``libhq4.so`` (the C ABI declared in ``include/hq4.h``).

The binding mirrors how the reference binds its own kernel
(``hetero/cpu_model.py:33-45``: ``ctypes.CDLL`` plus argtypes of ``c_void_p`` and
``c_int``).  There is no fallback: if the library is missing the import of any
op fails with an error naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import re

from . import build as _build

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_Z = ctypes.c_size_t
_F = ctypes.c_float

HEADER = os.path.join(_build.INCLUDE, "hq4.h")

# name -> (restype, argtypes); kept in the order of include/hq4.h
SIGNATURES = {
    "hq4_version": (_I, []),
    "hq4_device_status": (_I, [_I]),
    "hq4_gemv": (_I, [_P] * 5 + [_I] * 4 + [_P]),
    "hq4_gemv_fused": (_I, [_P] * 5 + [_I] * 4 + [_P] * 3),
    "hq4_gemv_ex": (_I, [_P] * 5 + [_I] * 4 + [_P] * 2 + [_I, _P]),
    "hq4_gemv_host": (_I, [_P] * 6 + [_I] * 4 + [_P] * 3),
    "hq4_dequant": (_I, [_P] * 4 + [_I] * 4 + [_P]),
    "hq4_embed_f16": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "hq4_gemm_w4a16": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P, _P, _P, _LL, _P]),
    "hq4_gemm_workspace_bytes": (_LL, [_I, _I, _I]),
    "hq4_gemm_plan": (_I, [_I, _I, _I, _I, _P]),
    "hq4_gemm_w4a16_static": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P, _P, _P]),
    "hq4_gemv_norm": (_I, [_P] * 5 + [_I] * 4 + [_P, _F, _I, _P, _P, _P]),
    "hq4_qkv_rope": (_I, [_P] * 4 + [_I] * 6 + [_P, _F, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    "hq4_attention": (_I, [_P] * 4 + [_I] * 4 + [_P, _I, _F, _P]),
    "hq4_act_encode_i8": (_I, [_P, _I, _I, _P, _P]),
    "hq4_act_decode_i8": (_I, [_P, _I, _I, _P, _P, _P]),
    "hq4_act_encode_i8_wire": (_I, [_P, _I, _I, _P, _P]),
    "hq4_argmax": (_I, [_P, _I, _P, _P, _I, _P, _P, _P]),
    "hq4_sample": (_I, [_P, _I, _F, _F, ctypes.c_double, _P, _P]),
    "hq4_synth_embed_f16": (_I, [ctypes.c_longlong, _I, _I, _F, _P, _P]),
    "hq4_argmax_pair": (_I, [_P, _I, _I, _P, _P]),
    "hq4_pick_token": (_I, [_P, _I, _P, _P, _I, _P]),
    "hq4_pick_token_next": (_I, [_P, _I, _P, _P, _P, _I, _P]),
    "hq4_advance_position": (_I, [_P, _I, _P]),
    "hq4_decode_plan_create": (_I, [_P] + [_I] * 7 + [_F, _F, _P, _P, _I] + [_P] * 6),
    "hq4_decode_plan_run": (_I, [_P, _P]),
    "hq4_decode_plan_info": (_I, [_P, _P]),
    "hq4_decode_plan_fault": (_I, [_P, _I, _LL]),
    "hq4_decode_plan_destroy": (None, [_P]),
}

ERRORS = {
    -1: "bad shape (n_in % gs, unsupported gs, or a non-positive size)",
    -2: "misaligned pointer",
    -4: "CUDA launch failed",
    -5: "current device is not sm_100 (B200)",
}

_lib = None

# HQ4_CHECKS=1: every call made through `checked()` validates its tensors
# (device, minimum size, alignment) before the launch.
CHECKS = os.environ.get("HQ4_CHECKS", "0") == "1"


def expect(t, nbytes: int, what: str, align: int = 4):
    """Raise unless tensor t is on the current CUDA device, holds at least
    nbytes from its data pointer on, and is `align`-byte aligned."""
    if not CHECKS or t is None:
        return
    import torch
    if not t.is_cuda or t.device.index != torch.cuda.current_device():
        raise RuntimeError(f"{what}: tensor on {t.device}, current device {torch.cuda.current_device()}")
    have = (t.untyped_storage().nbytes() - t.storage_offset() * t.element_size())
    if have < nbytes:
        raise RuntimeError(f"{what}: needs {nbytes} bytes, tensor holds {have}")
    if t.data_ptr() % align:
        raise RuntimeError(f"{what}: pointer not {align}-byte aligned")


def declared_symbols(header: str = HEADER):
    """Function names declared in include/hq4.h."""
    text = open(header).read()
    return re.findall(r"^\s*(?:int|size_t|void|long long)\s+(hq4_\w+)\s*\(", text, flags=re.M)


def load(path: str = None) -> ctypes.CDLL:
    """Load libhq4.so and attach argtypes; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or _build.LIB
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m hetero_infer_b200.build` "
                           "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with {rc}: {ERRORS.get(rc, 'unknown error')}")
