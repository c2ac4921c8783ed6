"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and argument validation fails with the documented status codes
before any device work."""
import ctypes
import os
import re

import numpy as np
import pytest

import mold_b200
from mold_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mold_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^MB_API\s+[\w\s\*]+?\b(mb_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "mb_qlinear" in syms and "mb_attention" in syms and "mb_flux_denoise" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in include/mold_b200.h but not exported"


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_no_cpu_fallback_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.lib()


def test_invalid_arguments_report_status():
    lib = mold_b200.lib()
    out = ctypes.c_void_p()
    data = np.zeros(144, np.uint8)
    # unsupported ggml type (Q2_K = 10)
    rc = lib.mb_weight_create(10, 1, 256, data.ctypes.data_as(ctypes.c_void_p), 144, 0, ctypes.byref(out))
    assert rc == _lib.MB_ERR_UNSUPPORTED
    assert b"unsupported ggml type" in lib.mb_last_error()
    # n_cols not a multiple of the Q4_K block
    rc = lib.mb_weight_create(12, 1, 100, data.ctypes.data_as(ctypes.c_void_p), 144, 0, ctypes.byref(out))
    assert rc == _lib.MB_ERR_INVALID
    # byte count mismatch
    rc = lib.mb_weight_create(12, 2, 256, data.ctypes.data_as(ctypes.c_void_p), 144, 0, ctypes.byref(out))
    assert rc == _lib.MB_ERR_INVALID and b"nbytes" in lib.mb_last_error()
    # NULL handles
    assert lib.mb_dequant(None, None, 0, None) == _lib.MB_ERR_INVALID
    assert lib.mb_qlinear(None, None, 0, 0, 0, None, 0, 0, None, 0, 0, None, None, 0, None) == _lib.MB_ERR_INVALID
    assert lib.mb_attention(None, None, None, 1, 1, 1, 1, None, 128, None) == _lib.MB_ERR_INVALID
    assert lib.mb_flux_forward(None, None, None, 0, None, None, 0, 0.0, None, 0.0, None, None) == _lib.MB_ERR_INVALID


def test_flux_config_rejects_bad_head_dim():
    lib = mold_b200.lib()
    cfg = mold_b200.FluxConfig(hidden_size=3000, num_heads=24).to_c()
    h = ctypes.c_void_p()
    rc = lib.mb_flux_create(ctypes.byref(cfg), 512, 4096, ctypes.byref(h))
    assert rc == _lib.MB_ERR_UNSUPPORTED and b"head_dim" in lib.mb_last_error()
