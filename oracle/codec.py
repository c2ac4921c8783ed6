"""ctypes front of oracle/codec.c (test infrastructure only; see oracle/__init__.py)."""
import ctypes
import os
import subprocess

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16 = 0, 1, 8, 12, 30
GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q5_K, GGML_Q6_K = 2, 3, 6, 7, 13, 14
_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144),
          GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20), GGML_Q5_0: (32, 22), GGML_Q5_1: (32, 24),
          GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}

_HERE = os.path.dirname(os.path.abspath(__file__))
lib_path = os.path.join(_HERE, "liboracle.so")
_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(lib_path) or os.path.getmtime(lib_path) < os.path.getmtime(os.path.join(_HERE, "codec.c")):
            subprocess.check_call(["make", "-s", "-C", _HERE])
        _lib = ctypes.CDLL(lib_path)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        _lib.or_dequantize.argtypes = [ctypes.c_int, P, I64, P]
        _lib.or_dequantize.restype = ctypes.c_int
        _lib.or_quantize_q8_0.argtypes = [P, I64, P]
        _lib.or_quantize_q4_k.argtypes = [P, I64, P]
        _lib.or_quantize_q4q5.argtypes = [P, I64, P, ctypes.c_int, ctypes.c_int]
        _lib.or_quantize_q5_k.argtypes = [P, I64, P]
        _lib.or_quantize_q6_k.argtypes = [P, I64, P]
        _lib.or_lora_merge.argtypes = [ctypes.c_int, P, I64, I64, I64, I64, P, P, ctypes.c_int, ctypes.c_float, P]
        _lib.or_lora_merge.restype = ctypes.c_int
        _lib.or_randn.argtypes = [ctypes.c_uint64, I64, ctypes.c_float, P]
        _lib.or_round_bf16.argtypes = [P, I64, P]
    return _lib


def block_elems(t):
    return _BLOCK[t][0]


def block_bytes(t):
    return _BLOCK[t][1]


def row_bytes(t, k):
    be, bb = _BLOCK[t]
    assert k % be == 0
    return k // be * bb


def randn(seed, shape, std=1.0):
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    _load().or_randn(ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), n, std, out.ctypes.data)
    return out.reshape(shape)


def round_bf16(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _load().or_round_bf16(x.ctypes.data, x.size, out.ctypes.data)
    return out


def to_bf16_bits(x):
    """f32 array -> uint16 bf16 bit patterns (RNE)."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def quantize(x, t):
    """f32 [.., K] -> raw GGML bytes [.., row_bytes]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    if t == GGML_F32:
        return x.view(np.uint8).reshape(x.shape[:-1] + (k * 4,)).copy()
    if t == GGML_F16:
        return x.astype(np.float16).view(np.uint8).reshape(x.shape[:-1] + (k * 2,)).copy()
    if t == GGML_BF16:
        return to_bf16_bits(x).view(np.uint8).reshape(x.shape[:-1] + (k * 2,)).copy()
    out = np.empty(x.shape[:-1] + (row_bytes(t, k),), dtype=np.uint8)
    if t == GGML_Q8_0:
        _load().or_quantize_q8_0(x.ctypes.data, x.size, out.ctypes.data)
    elif t == GGML_Q4_K:
        _load().or_quantize_q4_k(x.ctypes.data, x.size, out.ctypes.data)
    elif t in (GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1):
        bits = 4 if t in (GGML_Q4_0, GGML_Q4_1) else 5
        _load().or_quantize_q4q5(x.ctypes.data, x.size, out.ctypes.data, bits, int(t in (GGML_Q4_1, GGML_Q5_1)))
    elif t == GGML_Q5_K:
        _load().or_quantize_q5_k(x.ctypes.data, x.size, out.ctypes.data)
    elif t == GGML_Q6_K:
        _load().or_quantize_q6_k(x.ctypes.data, x.size, out.ctypes.data)
    else:
        raise ValueError(f"no quantizer for ggml type {t}")
    return out


def dequantize(raw, t, shape):
    """raw GGML bytes -> f32 array of `shape` (last dim = K)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    rc = _load().or_dequantize(t, raw.ctypes.data, n, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"dequantize failed rc={rc} type={t}")
    return out.reshape(shape)


def lora_merge(raw, t, shape, row0, nrows, A, B, scale):
    """Raw GGUF bytes of a [rows, cols] weight with rows [row0, row0 + nrows) replaced by
    quantize(dequant + fl(fl(B @ A) * scale)) (dot products by fmaf in ascending k)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    rows, cols = shape
    assert A.shape == (B.shape[1], cols) and B.shape[0] == nrows
    out = np.empty_like(raw)
    rc = _load().or_lora_merge(t, raw.ctypes.data, rows, cols, row0, nrows, A.ctypes.data, B.ctypes.data, B.shape[1],
                               float(scale), out.ctypes.data)
    if rc != 0:
        raise ValueError(f"lora_merge failed rc={rc}")
    return out
