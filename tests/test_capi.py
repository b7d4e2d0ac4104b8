"""The C ABI library: it loads without a GPU, exports every entry point the header
declares with the signatures the Python layer binds, and rejects bad arguments
before touching the device.  CPU only (no compute calls)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from int8_linear import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "int8_linear_b200.h"


def header_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(i8l_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.load()
    declared = header_functions()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"
    assert set(declared) == set(_native.SIGNATURES), "the Python bindings and the header differ"


def test_header_declares_cplusplus_guard_and_no_torch_types():
    code = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    assert 'extern "C"' in code
    for banned in ("torch", "at::", "Tensor", "c10"):
        assert banned not in code


def test_version_and_error_string():
    lib = _native.load()
    assert lib.i8l_version().decode().endswith("sm_100a")
    assert isinstance(lib.i8l_last_error(), bytes)


def test_argument_errors_need_no_gpu():
    lib = _native.load()
    # an unsupported output dtype is refused before any CUDA call
    rc = lib.i8l_w8a8_mm(None, 16, None, 16, None, 0, None, 0, None, 0, None, 99, 16,
                         4, 4, 16, None, None, 0, None)
    assert rc == _native.ENOTSUP and b"dtype" in lib.i8l_last_error()
    with pytest.raises(_native.NotSupported):
        _native.check(rc)
    # empty problems are a no-op
    assert lib.i8l_w8a8_mm(None, 16, None, 16, None, 0, None, 0, None, 0, None, 0, 16,
                           0, 4, 16, None, None, 0, None) == _native.OK
    rc = lib.i8l_w8a8_mm(None, 16, None, 16, None, 0, None, 0, None, 0, None, 0, 16,
                         -1, 4, 16, None, None, 0, None)
    assert rc == _native.EINVAL
    with pytest.raises(ValueError):
        _native.check(rc)
    assert lib.i8l_silu_mul_quant(None, 0, 7, None, 0, None, 1, 8, 1, 0, None) == _native.ENOTSUP
    assert lib.i8l_quant_rows(None, 0, 0, None, 0, None, 0, 8, 1, None) == _native.OK
    assert lib.i8l_add_rmsnorm_quant(None, 0, None, 0, None, 0, 9, None, 0, None, None, 0,
                                     1, 8, ctypes.c_float(1e-6), 1, None) == _native.ENOTSUP


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError, match="int8_linear.build"):
        _native.load(tmp_path / "nope.so")
