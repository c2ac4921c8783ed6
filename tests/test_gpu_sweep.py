"""BASELINE config 2 (the Q4_K dequant-GEMM microbenchmark over the FLUX linear shapes):
every M x (K -> N) of the sweep through mb_qlinear, checked against the oracle. Weights are
N(0, 0.02) quantized by the oracle's Q4_K quantizer, activations bf16 N(0, 1); the reference
is the oracle's exact GGML decode multiplied in fp32 on the GPU (TF32 off; the numpy product
is too slow at these sizes), so the decode under test is never the product's own.
The linears are those of flux/offload.rs:191-226 (qkv, proj, mlp) and :377-396 (linear2)."""
import numpy as np
import pytest
import torch

import bench
import mold_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("name,K,N", bench.SWEEP_KN, ids=[s[0] for s in bench.SWEEP_KN])
def test_sweep_shape_matches_oracle(cuda, name, K, N):
    raw = oracle.quantize(oracle.randn(K * 7 + N, (N, K), 0.02), oracle.GGML_Q4_K)
    w = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q4_K, (N, K), raw))
    wf = torch.from_numpy(oracle.dequantize(raw, oracle.GGML_Q4_K, (N, K))).to(cuda)
    assert torch.equal(mb.dequantize(w, torch.float32), wf)  # bit-exact device decode
    for M in bench.SWEEP_M:
        g = torch.Generator(device="cuda").manual_seed(M + K)
        x = torch.randn((M, K), device="cuda", generator=g).bfloat16()
        y = w.forward(x, out_dtype=torch.float32)
        ref = x.float() @ wf.t()
        err = ((y - ref).norm() / ref.norm()).item()
        assert err < 4e-3, (M, err)
        # the tensor core multiplies the decode rounded to bf16: against that product the error is
        # only the fp32 summation order
        refb = x.float() @ wf.bfloat16().float().t()
        errb = ((y - refb).norm() / refb.norm()).item()
        assert errb < 1e-4, (M, errb)
    assert mb.device_status() == 0
