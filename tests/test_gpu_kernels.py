"""GPU parity of the single kernels against the CPU oracle, through the C ABI."""
import ctypes
import math

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from mold_b200 import _lib
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "codec_golden.npz"))


def qmat(x, t, device=0):
    raw = oracle.quantize(x, t)
    return mb.QMatMul.from_weights(mb.QTensor(t, x.shape, raw), device), raw


# ------------------------------------------------------------------ K1 dequant
@pytest.mark.parametrize("t", [oracle.GGML_Q4_K, oracle.GGML_Q8_0, oracle.GGML_BF16])
@pytest.mark.parametrize("shape", [(1, 256), (37, 512), (300, 3072)])
def test_dequant_bit_exact(cuda, t, shape):
    x = oracle.randn(11, shape, 0.02)
    w, raw = qmat(x, t)
    ref = oracle.dequantize(raw, t, shape)
    got = mb.dequantize(w, torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    gb = mb.dequantize(w, torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(gb.view(np.uint32), oracle.round_bf16(ref).view(np.uint32))


def test_dequant_golden_q4k_random_blocks(cuda):
    blocks = GOLD["q4k_blocks"]
    w = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q4_K, (blocks.shape[0], 256), blocks))
    got = mb.dequantize(w, torch.float32).cpu().numpy()
    ref = GOLD["q4k_deq"].astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_golden_q8(cuda):
    blocks = GOLD["q8_blocks"]
    w = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q8_0, GOLD["q8_in"].shape, blocks))
    got = mb.dequantize(w, torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), GOLD["q8_deq"].astype(np.float32).view(np.uint32))


# ------------------------------------------------------------------ K2 quantized GEMM
GEMM_CASES = [
    (oracle.GGML_Q4_K, 128, 128, 256),
    (oracle.GGML_Q4_K, 1, 64, 256),
    (oracle.GGML_Q4_K, 300, 200, 512),
    (oracle.GGML_Q4_K, 1536, 3072, 3072),
    (oracle.GGML_Q8_0, 128, 128, 256),
    (oracle.GGML_Q8_0, 257, 384, 768),
    (oracle.GGML_Q8_0, 1536, 1024, 3072),
    (oracle.GGML_BF16, 200, 3072, 64),
    (oracle.GGML_BF16, 130, 256, 320),
]


@pytest.mark.parametrize("t,M,N,K", GEMM_CASES)
def test_qgemm_matches_oracle(cuda, t, M, N, K):
    w_f = oracle.randn(5, (N, K), 0.02)
    w, raw = qmat(w_f, t)
    x = oracle.round_bf16(oracle.randn(6, (M, K)))
    bias = oracle.randn(7, (N,), 0.02)
    wd = oracle.dequantize(raw, t, (N, K)).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T + bias
    xt = torch.from_numpy(x).to(cuda).bfloat16()
    bt = torch.from_numpy(bias).to(cuda)
    y = w.forward(xt, bias=bt, out_dtype=torch.float32)
    torch.cuda.synchronize()
    err = rel_l2(y.cpu().numpy(), ref)
    # bf16 weights operand (one rounding of the exact GGML decode) -> ~2^-9 relative
    assert err < 1e-2, err
    assert err < 4e-3, err
    # tighter: against the bf16-rounded dequantized weight the only difference is f32 accumulation order
    ref_bf = x.astype(np.float64) @ oracle.round_bf16(wd.astype(np.float32)).astype(np.float64).T + bias
    assert rel_l2(y.cpu().numpy(), ref_bf) < 1e-5
    assert mb.device_status() == 0


def test_qgemm_bf16_out_and_gelu_from(cuda):
    N, K, M = 512, 256, 256
    w, raw = qmat(oracle.randn(8, (N, K), 0.02), oracle.GGML_Q4_K)
    x = oracle.round_bf16(oracle.randn(9, (M, K)))
    b = oracle.randn(10, (N,), 0.02)
    ref = x.astype(np.float64) @ oracle.dequantize(raw, 12, (N, K)).astype(np.float64).T + b
    ref[:, 200:] = F.gelu_tanh(ref[:, 200:].astype(np.float32))
    y = w.forward(torch.from_numpy(x).to(cuda).bfloat16(), bias=torch.from_numpy(b).to(cuda),
                  epilogue=mb.EPI_GELU_TANH, gelu_from=200)
    assert y.dtype == torch.bfloat16
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-2


def test_qgemm_gate_residual_strided(cuda):
    """y = res + gate * (x W^T + b) with x read through a row stride (as the fused
    single-block layout does) and y aliasing the residual."""
    N, K, M, ld = 384, 512, 200, 1024
    w, raw = qmat(oracle.randn(12, (N, K), 0.02), oracle.GGML_Q8_0)
    xfull = oracle.round_bf16(oracle.randn(13, (M, ld)))
    x = xfull[:, 256:256 + K]
    b = oracle.randn(14, (N,), 0.02)
    g = oracle.randn(15, (N,))
    res = oracle.randn(16, (M, N))
    ref = res + g * (x.astype(np.float64) @ oracle.dequantize(raw, 8, (N, K)).astype(np.float64).T + b)
    xt = torch.from_numpy(xfull).to(cuda).bfloat16()[:, 256:256 + K]
    rt = torch.from_numpy(res).to(cuda)
    w.forward(xt, bias=torch.from_numpy(b).to(cuda), epilogue=mb.EPI_GATE_RESIDUAL, gate=torch.from_numpy(g).to(cuda),
              residual=rt, out=rt)
    # the update gate*(xW^T+b) is rounded once to bf16 before the f32 residual add
    assert rel_l2(rt.cpu().numpy(), ref) < 4e-3
    assert rel_l2(rt.cpu().numpy() - res, ref - res) < 4e-3


def test_qlinear_f32_input(cuda):
    N, K, M = 256, 512, 64
    w, raw = qmat(oracle.randn(17, (N, K), 0.02), oracle.GGML_Q4_K)
    x = oracle.randn(18, (M, K))
    ref = x.astype(np.float64) @ oracle.dequantize(raw, 12, (N, K)).astype(np.float64).T
    y = w.forward(torch.from_numpy(x).to(cuda))
    assert y.dtype == torch.float32
    assert rel_l2(y.cpu().numpy(), ref) < 1e-2


def test_qlinear_f32_unaligned_rejected(cuda):
    """An f32 x that is not 16-byte aligned, or whose row stride is not a multiple of 4,
    is rejected with MB_ERR_INVALID before any kernel runs."""
    N, K, M = 256, 512, 8
    w, _ = qmat(oracle.randn(19, (N, K), 0.02), oracle.GGML_Q4_K)
    buf = torch.zeros(M * (K + 4) + 4, device=cuda)
    y = torch.empty((M, N), device=cuda)
    P = ctypes.c_void_p
    for off, ld in ((1, K), (0, K + 1)):  # 4-byte offset base; odd row stride
        rc = mb.lib().mb_qlinear(w.handle, P(buf.data_ptr() + 4 * off), _lib.DT_F32, M, ld, P(y.data_ptr()),
                                 _lib.DT_F32, N, None, 0, 0, None, None, 0, None)
        assert rc == _lib.MB_ERR_INVALID, (off, ld)
        assert b"16-byte aligned" in mb.lib().mb_last_error()


# ------------------------------------------------------------------ K3 GEMV
@pytest.mark.parametrize("t", [oracle.GGML_Q4_K, oracle.GGML_Q8_0])
@pytest.mark.parametrize("K,xs", [(3072, 1.0), (256, 1.0), (768, 1.0), (4096, 1.0), (3072, 1e3), (3072, 1e-3)])
def test_qgemv_silu(cuda, t, K, xs):
    N = 1000
    w, raw = qmat(oracle.randn(19, (N, K), 0.02), t)
    x = oracle.randn(20, (K,)) * np.float32(xs)
    b = oracle.randn(21, (N,), 0.02)
    ref = F.silu(x.astype(np.float64)) @ oracle.dequantize(raw, t, (N, K)).astype(np.float64).T + b
    y = mb.qgemv(w, torch.from_numpy(x).to(cuda), apply_silu=True, bias=torch.from_numpy(b).to(cuda))
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5


# ------------------------------------------------------------------ K5 / K6 / rope / euler
@pytest.mark.parametrize("C,offset", [(3072, 1.0), (3072, 1000.0), (2304, 1.0), (1536, 50.0), (6144, 1.0)])
def test_ln_modulate(cuda, C, offset):
    """Widths whose blocks have a power-of-two number of warps (one-pass merged statistics) and
    not (2304: three warps, two passes); a row mean far above the spread checks the stability of
    the variance."""
    M = 300
    x = (oracle.randn(22, (M, C)) * 3 + offset).astype(np.float32)
    sh, sc = oracle.randn(23, (C,)), oracle.randn(24, (C,))
    ref = F.modulate(x, sh, sc)
    y = mb.ln_modulate(torch.from_numpy(x).to(cuda), torch.from_numpy(sh).to(cuda), torch.from_numpy(sc).to(cuda))
    assert rel_l2(y.float().cpu().numpy(), ref) < 4e-3


def test_rope_table(cuda):
    ids = np.concatenate([np.zeros((16, 3), np.float32), F.img_ids(8, 12)])
    ref = F.embed_nd(ids, (16, 56, 56), 10000)
    pe = mb.rope_table(torch.from_numpy(ids).to(cuda)).cpu().numpy()
    assert np.abs(pe - ref).max() < 2e-6


def test_qk_norm_rope(cuda):
    H, Lt, Li = 3, 40, 96
    L = Lt + Li
    ids = np.concatenate([np.zeros((Lt, 3), np.float32), F.img_ids(8, 12)])
    pe = F.embed_nd(ids, (16, 56, 56), 10000)
    qkv = oracle.round_bf16(oracle.randn(25, (Li, 3 * H * 128)))
    qs, ks = 1 + oracle.randn(26, (128,), 0.1), 1 + oracle.randn(27, (128,), 0.1)
    q, k, v = F.split_qkv(qkv, H)
    qr = F.apply_rope(F.rms_norm(q, qs), pe[Lt:])
    kr = F.apply_rope(F.rms_norm(k, ks), pe[Lt:])
    pet = torch.from_numpy(pe).to(cuda)
    gq, gk, gv = mb.qk_norm_rope(torch.from_numpy(qkv).to(cuda).bfloat16(), H, torch.from_numpy(qs).to(cuda),
                                 torch.from_numpy(ks).to(cuda), pet, row_offset=Lt, L_total=L)
    assert rel_l2(gq[:, Lt:].float().cpu().numpy(), qr) < 4e-3
    assert rel_l2(gk[:, Lt:].float().cpu().numpy(), kr) < 4e-3
    assert np.array_equal(gv[:, Lt:].float().cpu().numpy(), v)


def test_euler(cuda):
    a = torch.randn(1000, device=cuda)
    p = torch.randn(1000, device=cuda)
    ref = a + p * -0.125
    mb.euler_step(a, p, -0.125)
    assert torch.allclose(a, ref)


# ------------------------------------------------------------------ K4 attention
@pytest.mark.parametrize("H,Lq,Lk,valid", [(2, 128, 128, None), (3, 256, 384, None), (2, 200, 200, None),
                                           (24, 1536, 1536, None), (2, 384, 512, 300), (1, 1000, 1000, None)])
def test_attention(cuda, H, Lq, Lk, valid):
    q = oracle.round_bf16(oracle.randn(30, (H, Lq, 128)))
    k = oracle.round_bf16(oracle.randn(31, (H, Lk, 128)))
    v = oracle.round_bf16(oracle.randn(32, (H, Lk, 128)))
    mask = None
    if valid is not None:
        mask = np.arange(Lk) < valid
    ref = F.sdpa(q, k, v, mask).transpose(1, 0, 2).reshape(Lq, H * 128)
    out = mb.attention(*(torch.from_numpy(a).to(cuda).bfloat16() for a in (q, k, v)), n_valid_keys=valid)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert rel_l2(out.float().cpu().numpy(), ref) < 1e-2


def test_attention_peaky_scores_rescale(cuda):
    """Scores that grow along the key axis force the lazy O rescale path."""
    H, L = 2, 512
    q = oracle.round_bf16(oracle.randn(33, (H, L, 128)) * 2)
    k = oracle.randn(34, (H, L, 128))
    k *= np.linspace(0.1, 4.0, L, dtype=np.float32)[None, :, None]
    k = oracle.round_bf16(k)
    v = oracle.round_bf16(oracle.randn(35, (H, L, 128)))
    ref = F.sdpa(q, k, v).transpose(1, 0, 2).reshape(L, H * 128)
    out = mb.attention(*(torch.from_numpy(a).to(cuda).bfloat16() for a in (q, k, v)))
    assert rel_l2(out.float().cpu().numpy(), ref) < 1e-2
