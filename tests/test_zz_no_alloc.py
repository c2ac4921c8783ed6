"""mb_qlinear_f32_static: the f32-input quantized linear that allocates nothing.

Callers that cannot let the library call cudaMalloc (callers that hand out device
memory from their own pool, hosts that forbid allocation after start-up) use this entry point; it stages the bf16 copy of x in a
fixed 8 MiB array compiled into the library instead of a grown scratch buffer.
Its results must equal mb_qlinear's on the same f32 input. This file is collected
last so that a run stopping at the first failure has run every other test first.
"""
import ctypes

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from mold_b200 import _lib
from tests.conftest import rel_l2


def _static(w, x, y, bias=None, epilogue=mb.EPI_NONE, gelu_from=0):
    P = ctypes.c_void_p
    return mb.lib().mb_qlinear_f32_static(
        w.handle, P(x.data_ptr()), x.shape[0], x.stride(0), P(y.data_ptr()),
        _lib.DT_BF16 if y.dtype == torch.bfloat16 else _lib.DT_F32, y.stride(0),
        P(bias.data_ptr()) if bias is not None else None, epilogue, gelu_from, None, None, 0,
        P(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize("t,M,N,K", [(oracle.GGML_Q4_K, 300, 512, 1024), (oracle.GGML_Q8_0, 1024, 384, 4096)])
def test_static_matches_qlinear_twice(cuda, t, M, N, K):
    raw = oracle.quantize(oracle.randn(41, (N, K), 0.02), t)
    w = mb.QMatMul.from_weights(mb.QTensor(t, (N, K), raw))
    bias = torch.from_numpy(oracle.randn(42, (N,), 0.02)).to(cuda)
    for call, seed in enumerate((43, 44)):  # two calls in a row; the array keeps the previous call's data
        x = torch.from_numpy(oracle.randn(seed, (M, K))).to(cuda)
        ref = w.forward(x, bias=bias, epilogue=mb.EPI_GELU_TANH, gelu_from=N // 2)  # mb_qlinear, f32 in/out
        y = torch.empty((M, N), device=cuda, dtype=torch.float32)
        _lib.check(_static(w, x, y, bias, mb.EPI_GELU_TANH, N // 2))
        torch.cuda.synchronize()
        assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < 1e-6, f"call {call}"
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
    assert b"exceeds the fixed staging buffer" in mb.lib().mb_last_error()
