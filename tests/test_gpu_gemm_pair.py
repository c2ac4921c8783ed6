"""The CTA-pair GEMM (tcgen05.mma.cta_group::2, the default) against the one-CTA-per-tile
kernel (MB_GEMM_PAIR=0, run in a child process since the mode is read once per process):
bit-identical outputs for every weight type, ragged M / N (pair tiles whose second half lies
past N, activation halves past M) and every epilogue."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = [(oracle.GGML_Q4_K, 1024, 3072, 3072), (oracle.GGML_Q8_0, 512, 640, 3072), (oracle.GGML_Q6_K, 300, 384, 512),
         (oracle.GGML_BF16, 100, 64, 256), (oracle.GGML_Q5_K, 257, 320, 768), (oracle.GGML_Q4_0, 64, 640, 512),
         (oracle.GGML_Q4_1, 700, 896, 256), (oracle.GGML_Q5_0, 33, 128, 256), (oracle.GGML_Q5_1, 513, 384, 512)]


def run_cases():
    """Every case with four epilogues; returns {name: host array}."""
    mb.init(0)
    out = {}
    for i, (qt, M, N, K) in enumerate(CASES):
        rng = np.random.default_rng(i)
        w = mb.QMatMul.from_weights(
            mb.QTensor(qt, (N, K), oracle.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), qt)))
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda().bfloat16()
        bias = torch.from_numpy((rng.standard_normal(N) * 0.02).astype(np.float32)).cuda()
        gate = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda()
        res = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).cuda()
        out[f"{i}_f32"] = w.forward(x, bias=bias, out_dtype=torch.float32)
        out[f"{i}_bf16"] = w.forward(x, out_dtype=torch.bfloat16)
        out[f"{i}_gelu"] = w.forward(x, bias=bias, epilogue=mb.EPI_GELU_TANH, gelu_from=N // 2, out_dtype=torch.bfloat16)
        out[f"{i}_res"] = w.forward(x, bias=bias, epilogue=mb.EPI_GATE_RESIDUAL, gate=gate, residual=res,
                                    out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    return {k: v.float().cpu().numpy() for k, v in out.items()}


def test_pair_gemm_matches_single_cta_gemm(cuda, tmp_path):
    ref_file = tmp_path / "single.npz"
    env = dict(os.environ, MB_GEMM_PAIR="0", PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, os.path.abspath(__file__), str(ref_file)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    single = np.load(ref_file)
    assert os.environ.get("MB_GEMM_PAIR", "1") != "0"
    pair = run_cases()
    assert sorted(pair) == sorted(single.files)
    bad = [k for k in pair if not np.array_equal(pair[k], single[k])]
    assert not bad, bad


if __name__ == "__main__":
    np.savez(sys.argv[1], **run_cases())
