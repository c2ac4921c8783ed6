"""mb_qlinear_f32_static: the f32-input quantized linear that allocates nothing.

Callers that cannot let the library call cudaMalloc (callers that hand out device
memory from their own pool, hosts that forbid allocation after start-up) use this entry point; it stages the bf16 copy of x in a
fixed 8 MiB array compiled into the library instead of a grown scratch buffer.
Its results must equal mb_qlinear's on the same f32 input and match the oracle's
x W^T. This file is collected last so that a run stopping at the first failure has
run every other test first.
"""
import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref
from mold_b200 import _lib
from tests.conftest import ROOT, rel_l2


def _static(w, x, y, bias=None, epilogue=mb.EPI_NONE, gelu_from=0, M=None):
    P = ctypes.c_void_p
    return mb.lib().mb_qlinear_f32_static(
        w.handle, P(x.data_ptr()), x.shape[0] if M is None else M, x.stride(0), P(y.data_ptr()),
        _lib.DT_BF16 if y.dtype == torch.bfloat16 else _lib.DT_F32, y.stride(0),
        P(bias.data_ptr()) if bias is not None else None, epilogue, gelu_from, None, None, 0,
        P(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize("t,M,N,K", [(oracle.GGML_Q4_K, 300, 512, 1024), (oracle.GGML_Q8_0, 1024, 384, 4096)])
def test_static_matches_qlinear_twice(cuda, t, M, N, K):
    raw = oracle.quantize(oracle.randn(41, (N, K), 0.02), t)
    w = mb.QMatMul.from_weights(mb.QTensor(t, (N, K), raw))
    wf = oracle.dequantize(raw, t, (N, K)).astype(np.float64)
    b_np = oracle.randn(42, (N,), 0.02)
    bias = torch.from_numpy(b_np).to(cuda)
    for call, seed in enumerate((43, 44)):  # two calls in a row; the array keeps the previous call's data
        x_np = oracle.randn(seed, (M, K))
        x = torch.from_numpy(x_np).to(cuda)
        ref = w.forward(x, bias=bias, epilogue=mb.EPI_GELU_TANH, gelu_from=N // 2)  # mb_qlinear, f32 in/out
        y = torch.empty((M, N), device=cuda, dtype=torch.float32)
        _lib.check(_static(w, x, y, bias, mb.EPI_GELU_TANH, N // 2))
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert rel_l2(got, ref.cpu().numpy()) < 1e-6, f"call {call} vs mb_qlinear"
        # Oracle: f64 product of the exact GGML decode, GELU-tanh on the columns >= gelu_from.
        o = x_np.astype(np.float64) @ wf.T + b_np
        o[:, N // 2:] = flux_ref.gelu_tanh(o[:, N // 2:])
        assert rel_l2(got, o) < 4e-3, f"call {call} vs oracle"
    assert mb.device_status() == 0


@pytest.mark.gpu
def test_static_rejects_oversize(cuda):
    K, N = 4096, 128
    raw = oracle.quantize(oracle.randn(45, (N, K), 0.02), oracle.GGML_Q4_K)
    w = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q4_K, (N, K), raw))
    M = (4 << 20) // K + 1
    x = torch.zeros((M, K), device=cuda)
    y = torch.empty((M, N), device=cuda)
    rc = _static(w, x, y)
    assert rc == _lib.MB_ERR_INVALID
    assert b"exceed the fixed staging buffer" in mb.lib().mb_last_error()
    # A row count whose product with K wraps 64 bits is rejected as well, not staged.
    rc = _static(w, x, y, M=(1 << 58))
    assert rc == _lib.MB_ERR_INVALID


_FRESH = textwrap.dedent("""
    import ctypes, sys, torch
    sys.path.insert(0, {root!r})
    import mold_b200 as mb, oracle
    from mold_b200 import _lib
    mb.init(0)
    K, N = 3072, 1024
    raw = oracle.quantize(oracle.randn(46, (N, K), 0.02), oracle.GGML_Q4_K)
    w = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q4_K, (N, K), raw))
    P = ctypes.c_void_p
    def call(M):
        x = xs[M]; y = ys[M]
        _lib.check(mb.lib().mb_qlinear_f32_static(w.handle, P(x.data_ptr()), M, K, P(y.data_ptr()), _lib.DT_F32, N,
                                                  None, 0, 0, None, None, 0, None))
    xs = {{M: torch.randn(M, K, device="cuda") for M in (64, 1024, 1365)}}
    ys = {{M: torch.empty(M, N, device="cuda") for M in xs}}
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for M in (64, 1024, 1365, 64):
        call(M)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    print("FREE", free0, free1)
    assert free1 == free0, f"device free memory changed by {{free0 - free1}} bytes"
""")


@pytest.mark.gpu
def test_static_first_calls_allocate_nothing(cuda):
    """In a fresh process (device modules loaded eagerly, so the library's own code and
    the fixed array are resident from context creation), the first calls of the entry
    point, at several sizes, leave the device's free memory unchanged."""
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _FRESH.format(root=ROOT)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
