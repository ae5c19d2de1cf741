"""ctypes front end of the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only to check or time against; the product
path (``hetero_infer_b200``) never imports anything under ``oracle/``.

Two kinds of checker live here:

* ``Oracle``: our own C restatement of the reference arithmetic
  (``oracle/q4_oracle.c``), for the float semantics of
  ``kernel/q4gemv.c:113-139`` and the AVX2 int16 semantics of
  ``kernel/q4gemv.c:80-111,252-272``, plus ``q4_dequant`` (``:316-379``).
* ``RefKernel``: the reference's own ``kernel/q4gemv.c`` compiled from its
  source into ``oracle/_ref/`` by ``oracle/Makefile`` -- the same C ABI the
  reference binds in ``hetero/cpu_model.py:33-45``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle_q4.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_VARIANTS = {"avx2": "libq4gemv_avx2.so", "float": "libq4gemv_float.so"}

_P = ctypes.c_void_p
_I = ctypes.c_int


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (our restatement, plus the reference build when the
    reference tree is present)."""
    out = subprocess.run(["make", "-C", HERE, "all"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")
    if not quiet:
        print(out.stdout)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _check_packed(w, scales, biases, gs):
    w = np.ascontiguousarray(w, dtype=np.uint32)
    scales = np.ascontiguousarray(scales).view(np.uint16)
    biases = np.ascontiguousarray(biases).view(np.uint16)
    n_out, n_in = w.shape[0], w.shape[1] * 8
    return w, scales, biases, n_out, n_in


class Oracle:
    """Our C restatement (oracle/q4_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.oracle_q4_gemv_f32.argtypes = [_P] * 5 + [_I] * 3
        lib.oracle_q4_gemv_i16.argtypes = [_P] * 5 + [_I] * 4
        lib.oracle_q4_dequant.argtypes = [_P] * 4 + [_I] * 4
        lib.oracle_quantise_x_i16.argtypes = [_P, _I, _P]
        lib.oracle_quantise_x_i16.restype = ctypes.c_float
        for f in ("oracle_q4_gemv_f32", "oracle_q4_gemv_i16", "oracle_q4_dequant"):
            getattr(lib, f).restype = _I
        self.lib = lib

    def gemv_f32(self, w, scales, biases, x, gs: int = 64) -> np.ndarray:
        w, scales, biases, n_out, n_in = _check_packed(w, scales, biases, gs)
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
        out = np.empty((x.shape[0], n_out), np.float32)
        for m in range(x.shape[0]):
            rc = self.lib.oracle_q4_gemv_f32(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x[m]),
                                             _ptr(out[m]), n_out, n_in, gs)
            if rc != 0:
                raise RuntimeError(f"oracle_q4_gemv_f32 failed with {rc}")
        return out

    def gemv_i16(self, w, scales, biases, x, gs: int = 64, contract: int = 1) -> np.ndarray:
        w, scales, biases, n_out, n_in = _check_packed(w, scales, biases, gs)
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
        out = np.empty((x.shape[0], n_out), np.float32)
        for m in range(x.shape[0]):
            rc = self.lib.oracle_q4_gemv_i16(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x[m]),
                                             _ptr(out[m]), n_out, n_in, gs, contract)
            if rc != 0:
                raise RuntimeError(f"oracle_q4_gemv_i16 failed with {rc}")
        return out

    def quantise_x_i16(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        xq = np.empty(x.shape, np.int16)
        scale = self.lib.oracle_quantise_x_i16(_ptr(x), x.size, _ptr(xq))
        return xq, np.float32(scale)

    def dequant(self, w, scales, biases, row0: int, row1: int, gs: int = 64) -> np.ndarray:
        w, scales, biases, n_out, n_in = _check_packed(w, scales, biases, gs)
        out = np.empty((max(row1 - row0, 0), n_in), np.float32)
        rc = self.lib.oracle_q4_dequant(_ptr(w), _ptr(scales), _ptr(biases), _ptr(out),
                                        row0, row1, n_in, gs)
        if rc != 0:
            raise RuntimeError(f"oracle_q4_dequant failed with {rc}")
        return out


class RefKernel:
    """The reference's own q4gemv.c, built from source into oracle/_ref/."""

    def __init__(self, variant: str = "avx2"):
        path = os.path.join(REF_DIR, REF_VARIANTS[variant])
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run make -C oracle ref)")
        lib = ctypes.CDLL(path)
        # argtypes as the reference binds them (hetero/cpu_model.py:41-44)
        lib.q4_gemv.argtypes = [_P] * 5 + [_I] * 4
        lib.q4_gemv.restype = _I
        lib.q4_dequant.argtypes = [_P] * 4 + [_I] * 5
        lib.q4_dequant.restype = _I
        self.lib, self.variant, self.path = lib, variant, path

    def gemv(self, w, scales, biases, x, gs: int = 64, nthreads: int = 1) -> np.ndarray:
        w, scales, biases, n_out, n_in = _check_packed(w, scales, biases, gs)
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
        out = np.empty((x.shape[0], n_out), np.float32)
        for m in range(x.shape[0]):
            rc = self.lib.q4_gemv(_ptr(w), _ptr(scales), _ptr(biases), _ptr(x[m]), _ptr(out[m]),
                                  n_out, n_in, gs, nthreads)
            if rc != 0:
                raise RuntimeError(f"q4_gemv failed with {rc}")
        return out

    def dequant(self, w, scales, biases, row0, row1, gs: int = 64, nthreads: int = 1):
        w, scales, biases, n_out, n_in = _check_packed(w, scales, biases, gs)
        out = np.empty((max(row1 - row0, 0), n_in), np.float32)
        rc = self.lib.q4_dequant(_ptr(w), _ptr(scales), _ptr(biases), _ptr(out),
                                 row0, row1, n_in, gs, nthreads)
        if rc != 0:
            raise RuntimeError(f"q4_dequant failed with {rc}")
        return out


def available_ref_variants():
    return [v for v, f in REF_VARIANTS.items() if os.path.exists(os.path.join(REF_DIR, f))]
