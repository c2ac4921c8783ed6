"""The GGUF types beyond Q4_K / Q8_0 (Q4_0, Q4_1, Q5_0, Q5_1, Q5_K, Q6_K) through dequant (K1),
the tensor-core GEMM (K2) and the GEMV (K3), against the oracle's decode (pinned bit-exact to
gguf 0.19.0 in test_oracle_codec.py)."""
import os

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "codec_golden.npz"))
TYPES = [("q4_0", oracle.GGML_Q4_0), ("q4_1", oracle.GGML_Q4_1), ("q5_0", oracle.GGML_Q5_0),
         ("q5_1", oracle.GGML_Q5_1), ("q5_k", oracle.GGML_Q5_K), ("q6_k", oracle.GGML_Q6_K)]


def qmat(x, t):
    raw = oracle.quantize(x, t)
    return mb.QMatMul.from_weights(mb.QTensor(t, x.shape, raw)), raw


@pytest.mark.parametrize("name,t", TYPES)
def test_dequant_golden_random_blocks(cuda, name, t):
    blocks = GOLD[name + "_blocks"]
    ref = GOLD[name + "_deq"].reshape(-1)
    K = 256 if ref.size % 1024 else 1024
    shape = (ref.size // K, K)
    w = mb.QMatMul.from_weights(mb.QTensor(t, shape, blocks.reshape(shape[0], -1)))
    got = mb.dequantize(w, torch.float32).cpu().numpy().reshape(-1)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("name,t", TYPES)
@pytest.mark.parametrize("shape", [(1, 256), (37, 512), (300, 3072)])
def test_dequant_bit_exact(cuda, name, t, shape):
    x = oracle.randn(31, shape, 0.02)
    w, raw = qmat(x, t)
    ref = oracle.dequantize(raw, t, shape)
    got = mb.dequantize(w, torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    gb = mb.dequantize(w, torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(gb.view(np.uint32), oracle.round_bf16(ref).view(np.uint32))


@pytest.mark.parametrize("name,t", TYPES)
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (300, 200, 512), (1536, 1024, 3072)])
def test_qgemm(cuda, name, t, M, N, K):
    w, raw = qmat(oracle.randn(32, (N, K), 0.02), t)
    x = oracle.round_bf16(oracle.randn(33, (M, K)))
    bias = oracle.randn(34, (N,), 0.02)
    wd = oracle.dequantize(raw, t, (N, K)).astype(np.float64)
    y = w.forward(torch.from_numpy(x).to(cuda).bfloat16(), bias=torch.from_numpy(bias).to(cuda),
                  out_dtype=torch.float32).cpu().numpy()
    ref = x.astype(np.float64) @ wd.T + bias
    assert rel_l2(y, ref) < 4e-3
    # the in-GEMM operand is the exact decode rounded once to bf16
    ref_bf = x.astype(np.float64) @ oracle.round_bf16(wd.astype(np.float32)).astype(np.float64).T + bias
    assert rel_l2(y, ref_bf) < 1e-5
    assert mb.device_status() == 0


@pytest.mark.parametrize("name,t", TYPES)
@pytest.mark.parametrize("K", [256, 3072])
def test_qgemv(cuda, name, t, K):
    N = 333
    w, raw = qmat(oracle.randn(35, (N, K), 0.02), t)
    x = oracle.randn(36, (K,))
    b = oracle.randn(37, (N,), 0.02)
    ref = F.silu(x.astype(np.float64)) @ oracle.dequantize(raw, t, (N, K)).astype(np.float64).T + b
    y = mb.qgemv(w, torch.from_numpy(x).to(cuda), apply_silu=True, bias=torch.from_numpy(b).to(cuda))
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5


def test_tiny_flux_forward_q6k_q4_1_mix(cuda):
    """A FLUX model whose linears mix Q6_K and Q4_1 (as K_M files mix types) against the oracle."""
    from tests.test_gpu_flux import TINY, inputs, to_model
    W = F.synth_weights(TINY, seed=6, qtype=oracle.GGML_Q6_K)
    W2 = F.synth_weights(TINY, seed=6, qtype=oracle.GGML_Q4_1)
    for n in W:
        if "single_blocks" in n and n.endswith("weight") and W[n].ggml_type == oracle.GGML_Q6_K:
            W[n] = W2[n]
    m = to_model(TINY, W, 64, 256)
    img, ids, txt, tids, y = inputs(TINY, 40, 12, 10)
    ref = F.forward(W, TINY, img, ids, txt, tids, 0.7, y, 3.5)
    t = lambda a: torch.from_numpy(a).to(cuda)
    pred = m.forward(t(img), t(ids), t(txt), t(tids), 0.7, t(y), 3.5).cpu().numpy()
    assert rel_l2(pred, ref) < 2e-2


def test_tiny_flux_forward_gemv_kinds_mixed(cuda):
    """Q4_K linears with Q6_K / Q5_K modulation weights: the step's modulation GEMVs then need both
    GEMV kernels (Q4_K / Q8_0 / plain rows, and the decode_unit types) in the same batch."""
    from tests.test_gpu_flux import TINY, inputs, to_model
    W = F.synth_weights(TINY, seed=12, qtype=oracle.GGML_Q4_K)
    W6 = F.synth_weights(TINY, seed=12, qtype=oracle.GGML_Q6_K)
    W5 = F.synth_weights(TINY, seed=12, qtype=oracle.GGML_Q5_K)
    swapped = 0
    for n in W:
        if n.endswith("weight") and ("_mod.lin" in n or "modulation.lin" in n):
            src = W6 if swapped % 2 == 0 else W5
            if src[n].ggml_type in (oracle.GGML_Q6_K, oracle.GGML_Q5_K):
                W[n] = src[n]
                swapped += 1
    assert swapped >= 2
    m = to_model(TINY, W, 64, 256)
    img, ids, txt, tids, y = inputs(TINY, 40, 12, 10)
    ref = F.forward(W, TINY, img, ids, txt, tids, 0.7, y, 3.5)
    t = lambda a: torch.from_numpy(a).to(cuda)
    pred = m.forward(t(img), t(ids), t(txt), t(tids), 0.7, t(y), 3.5).cpu().numpy()
    assert mb.device_status() == 0
    assert rel_l2(pred, ref) < 2e-2
