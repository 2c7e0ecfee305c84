"""The C-ABI library loads without a GPU and exports every symbol include/moss_w8.h declares."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from moss_image_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "moss_w8.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moss_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for required in ("moss_w8_quantize", "moss_w8a16_gemm_fwd", "moss_w8a16_gemm_dx", "moss_offload_pack",
                     "moss_offload_prefetch", "moss_offload_wait", "moss_strided_gather"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_exported_dynamic_symbols_are_exactly_the_c_abi():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    moss = {name for name in exported if name.startswith("moss_")}
    assert moss == set(declared_functions())


def test_version_and_argument_validation_need_no_gpu():
    lib = _lib.library()
    assert lib.moss_version() >= 100
    rc = lib.moss_w8_quantize(None, 7, 4, 4, None, None, None, None)
    assert rc == _lib.MOSS_ERR_UNSUPPORTED
    assert "dtype" in _lib.last_error()
    rc = lib.moss_w8a16_gemm_fwd(None, 2, 4, 4, None, None, 1, 4, None, 0, None, None, 0, 0, 1.0, None, 1, None, 0,
                                 None, None)
    assert rc == _lib.MOSS_ERR_UNSUPPORTED  # f32 compute dtype is refused up front
    rc = lib.moss_strided_gather(None, 3, 1, (ctypes.c_int64 * 1)(4), (ctypes.c_int64 * 1)(1), None, None)
    assert rc in (_lib.MOSS_ERR_INVALID_ARGUMENT, _lib.MOSS_ERR_UNSUPPORTED)
    rc = lib.moss_offload_ring_create(0, 0, 0, None, None, ctypes.byref(ctypes.c_void_p()))
    assert rc == _lib.MOSS_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(rc, "moss_offload_ring_create")


def test_empty_problems_are_no_ops_without_device_work():
    lib = _lib.library()
    assert lib.moss_w8a16_gemm_fwd(None, 1, 0, 16, None, None, 1, 8, None, 0, None, None, 0, 0, 1.0, None, 1,
                                   None, 0, None, None) == _lib.MOSS_OK
    assert lib.moss_w8a16_gemm_dx(None, 1, 0, 8, None, None, 1, 16, None, None, 0, 0, 1.0, None, 1,
                                  None, 0, None, None) == _lib.MOSS_OK
    size = ctypes.c_size_t(123)
    assert lib.moss_w8a16_gemm_workspace_bytes(0, 8, 16, ctypes.byref(size)) == _lib.MOSS_OK and size.value == 0
    assert lib.moss_w8_quantize(None, 1, 0, 16, None, None, None, None) == _lib.MOSS_OK
