"""The C ABI library loads without a GPU and exports every symbol include/hq4.h
declares; the ctypes signatures cover exactly those symbols."""
import ctypes
import os

import pytest

from hetero_infer_b200 import _lib, build


def test_library_built():
    assert os.path.exists(build.LIB), "run python -m hetero_infer_b200.build (or __graft_entry__.build())"


def test_exports_every_declared_symbol():
    names = _lib.declared_symbols()
    assert len(names) >= 3
    lib = ctypes.CDLL(build.LIB)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/hq4.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_version_without_gpu():
    lib = _lib.load()
    assert lib.hq4_version() >= 1


def test_error_table_matches_header():
    text = open(_lib.HEADER).read()
    for code in _lib.ERRORS:
        assert f"({code})" in text
