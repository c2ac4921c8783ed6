"""Edge cases of the C-ABI kernels: empty inputs (M = 0 rows) are no-ops that succeed, single
rows and single keys, one valid key (softmax over one key returns that key's value row), and the
documented size limits rejected with MB_ERR_INVALID before any kernel runs."""
import ctypes

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from mold_b200 import _lib
from oracle import flux_ref as F
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


def qmat(x, t):
    raw = oracle.quantize(x, t)
    return mb.QMatMul.from_weights(mb.QTensor(t, x.shape, raw)), raw


@pytest.mark.parametrize("t", [oracle.GGML_Q4_K, oracle.GGML_Q8_0])
def test_empty_rows_are_noops(cuda, t):
    N, K = 256, 512
    w, _ = qmat(oracle.randn(1, (N, K), 0.02), t)
    x = torch.zeros((1, K), device=cuda, dtype=torch.bfloat16)
    y = torch.full((1, N), 7.0, device=cuda)
    assert mb.lib().mb_qlinear(w.handle, P(x.data_ptr()), _lib.DT_BF16, 0, K, P(y.data_ptr()), _lib.DT_F32, N,
                               None, 0, 0, None, None, 0, None) == _lib.MB_OK
    xf = torch.zeros((1, 3072), device=cuda)
    sh = torch.zeros(3072, device=cuda)
    yb = torch.zeros((1, 3072), device=cuda, dtype=torch.bfloat16)
    assert mb.lib().mb_ln_modulate(P(xf.data_ptr()), 0, 3072, 3072, P(sh.data_ptr()), P(sh.data_ptr()),
                                   P(yb.data_ptr()), 3072, None) == _lib.MB_OK
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing was written
    assert mb.device_status() == 0


def test_single_row_gemm_and_gemv(cuda):
    N, K = 33, 256  # N not a multiple of the 32-row GEMV block or the 128-row GEMM tile
    w, raw = qmat(oracle.randn(2, (N, K), 0.02), oracle.GGML_Q4_K)
    wd = oracle.dequantize(raw, oracle.GGML_Q4_K, (N, K)).astype(np.float64)
    x = oracle.randn(3, (1, K))
    ref = x.astype(np.float64) @ wd.T
    y = w.forward(torch.from_numpy(x).to(cuda))
    assert rel_l2(y.cpu().numpy(), ref) < 4e-3
    yv = mb.qgemv(w, torch.from_numpy(x[0]).to(cuda))
    assert rel_l2(yv.cpu().numpy(), ref[0]) < 1e-5


def test_attention_one_valid_key_returns_its_value(cuda):
    H, Lq, Lk = 2, 130, 256
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = (torch.randn((H, L, 128), device="cuda", generator=g).bfloat16() for L in (Lq, Lk, Lk))
    out = mb.attention(q, k, v, n_valid_keys=1).float()  # [Lq, H * 128]
    want = v[:, 0, :].float().reshape(1, H * 128).expand(Lq, -1)
    assert torch.allclose(out, want, atol=1e-30, rtol=0)


def test_attention_single_query(cuda):
    H, Lk = 3, 300
    qn = oracle.round_bf16(oracle.randn(5, (H, 1, 128)))
    kn = oracle.round_bf16(oracle.randn(6, (H, Lk, 128)))
    vn = oracle.round_bf16(oracle.randn(7, (H, Lk, 128)))
    ref = F.sdpa(qn, kn, vn).transpose(1, 0, 2).reshape(1, H * 128)
    t = lambda a: torch.from_numpy(a).to(cuda).bfloat16()
    got = mb.attention(t(qn), t(kn), t(vn)).float().cpu().numpy()
    assert rel_l2(got, ref) < 1e-2


def test_size_limits_rejected(cuda):
    w, _ = qmat(oracle.randn(8, (64, 8192), 0.02), oracle.GGML_Q8_0)
    x = torch.zeros(8192, device=cuda)
    y = torch.zeros(64, device=cuda)
    assert mb.lib().mb_qgemv(w.handle, P(x.data_ptr()), 0, None, P(y.data_ptr()), None) == _lib.MB_ERR_INVALID
    assert b"K <= 4096" in mb.lib().mb_last_error()
    # the GEMM's K must be a multiple of 64 (bf16) / 256 (quantized)
    w2, _ = qmat(oracle.randn(9, (64, 288), 0.02), oracle.GGML_BF16)
    xb = torch.zeros((4, 288), device=cuda, dtype=torch.bfloat16)
    yb = torch.zeros((4, 64), device=cuda)
    rc = mb.lib().mb_qlinear(w2.handle, P(xb.data_ptr()), _lib.DT_BF16, 4, 288, P(yb.data_ptr()), _lib.DT_F32, 64,
                             None, 0, 0, None, None, 0, None)
    assert rc == _lib.MB_ERR_INVALID
    assert mb.device_status() == 0


@pytest.mark.parametrize("t", [oracle.GGML_Q4_K, oracle.GGML_Q8_0])
def test_gemv_nonfinite_input_propagates(cuda, t):
    """The GEMV stages x as fixed point; a non-finite input must still give non-finite outputs."""
    w, _ = qmat(oracle.randn(10, (64, 512), 0.02), t)
    x = torch.from_numpy(oracle.randn(11, (512,))).to(cuda)
    x[7] = float("inf")
    y = mb.qgemv(w, x)
    assert not torch.isfinite(y).any()
    x[7] = float("nan")
    assert not torch.isfinite(mb.qgemv(w, x)).any()
