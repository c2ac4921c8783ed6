"""LoRA merge on the device (mb_weight_lora_merge / mb_flux_lora_merge) against the oracle's merge,
byte for byte, and a FLUX model patched on the GPU against one built from oracle-merged bytes."""
import os

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from mold_b200.lora import LoraAdapter, apply_lora, plan_patches
from oracle import flux_ref as F
from tests.test_gpu_flux import TINY, inputs, to_model

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "codec_golden.npz"))

ALL_TYPES = [oracle.GGML_F32, oracle.GGML_F16, oracle.GGML_BF16, oracle.GGML_Q8_0, oracle.GGML_Q4_0, oracle.GGML_Q4_1,
             oracle.GGML_Q5_0, oracle.GGML_Q5_1, oracle.GGML_Q4_K, oracle.GGML_Q5_K, oracle.GGML_Q6_K]
SUPER = (oracle.GGML_Q4_K, oracle.GGML_Q5_K, oracle.GGML_Q6_K)


def merge_on_gpu(raw, t, shape, row0, A, B, scale, cuda):
    w = mb.QMatMul.from_weights(mb.QTensor(t, shape, raw))
    w.lora_merge(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), scale, row_offset=row0)
    torch.cuda.synchronize()
    return w.download()


@pytest.mark.parametrize("t", ALL_TYPES)
@pytest.mark.parametrize("shape,row0,rows,rank", [((48, 256), 8, 16, 4), ((20, 800), 3, 17, 16), ((300, 3072), 0, 300, 32)])
def test_merge_bit_exact_vs_oracle(cuda, t, shape, row0, rows, rank):
    if t in SUPER and shape[1] % 256:
        pytest.skip("super-block types need 256-value rows")
    w = oracle.randn(80, shape, 0.05)
    raw = oracle.quantize(w, t).reshape(-1)
    A = oracle.randn(81, (rank, shape[1]), 0.1)
    B = oracle.randn(82, (rows, rank), 0.1)
    want = oracle.lora_merge(raw, t, shape, row0, rows, A, B, 0.625)
    got = merge_on_gpu(raw, t, shape, row0, A, B, 0.625, cuda)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("name,t", [("q8_0", oracle.GGML_Q8_0), ("q4_0", oracle.GGML_Q4_0), ("q4_1", oracle.GGML_Q4_1),
                                    ("q5_0", oracle.GGML_Q5_0), ("q5_1", oracle.GGML_Q5_1), ("bf16", oracle.GGML_BF16)])
def test_merge_matches_gguf_requantize_fixture(cuda, name, t):
    """Rank-1 merge against gguf-py's dequantize + add + quantize (ggml's reference quantizers)."""
    raw = GOLD["lora_" + name + "_raw"].reshape(-1)
    got = merge_on_gpu(raw, t, (48, 256), int(GOLD["lora_row0"]), GOLD["lora_A"], GOLD["lora_B"],
                       float(GOLD["lora_scale"]), cuda)
    assert np.array_equal(got, GOLD["lora_" + name + "_out"].reshape(-1))


def test_merge_zero_rows_and_bounds(cuda):
    w = oracle.randn(83, (16, 256), 0.05)
    raw = oracle.quantize(w, oracle.GGML_Q8_0).reshape(-1)
    q = mb.QMatMul.from_weights(mb.QTensor(oracle.GGML_Q8_0, (16, 256), raw))
    A = torch.zeros((2, 256), device=cuda)
    q.lora_merge(A, torch.zeros((0, 2), device=cuda), 1.0, row_offset=16)
    torch.cuda.synchronize()
    assert np.array_equal(q.download(), raw)
    with pytest.raises(mb.MoldError, match="outside"):
        q.lora_merge(A, torch.zeros((4, 2), device=cuda), 1.0, row_offset=14)
    assert mb.device_status() == 0


def adapter_for(cfg, seed=90, rank=8):
    h, m = cfg.hidden_size, int(cfg.hidden_size * cfg.mlp_ratio)
    specs = {
        "transformer.transformer_blocks.0.attn.to_q": (h, h, 16.0),
        "transformer.transformer_blocks.0.attn.add_v_proj": (h, h, None),
        "transformer.transformer_blocks.1.attn.to_out.0": (h, h, 4.0),
        "transformer.transformer_blocks.1.ff.net.2": (h, m, None),
        "transformer.transformer_blocks.0.norm1.linear": (6 * h, h, None),
        "transformer.single_transformer_blocks.0.proj_mlp": (m, h, 8.0),
        "transformer.single_transformer_blocks.1.attn.to_k": (h, h, None),
        "transformer.single_transformer_blocks.1.proj_out": (h, h + m, None),
        "transformer.single_transformer_blocks.1.unknown": (h, h, None),
    }
    tensors = {}
    for i, (k, (o, inp, alpha)) in enumerate(specs.items()):
        tensors[k + ".lora_A.weight"] = oracle.randn(seed + 3 * i, (rank, inp), 0.05)
        tensors[k + ".lora_B.weight"] = oracle.randn(seed + 3 * i + 1, (o, rank), 0.05)
        if alpha is not None:
            tensors[k + ".alpha"] = np.array(alpha, np.float32)
    return LoraAdapter.from_tensors(tensors)


@pytest.mark.parametrize("qtype", [oracle.GGML_Q8_0, oracle.GGML_Q4_K])
def test_flux_lora_on_gpu_equals_oracle_merged_model(cuda, qtype):
    W = F.synth_weights(TINY, seed=11, qtype=qtype)
    ad = adapter_for(TINY)
    rows = {n: qt.shape[0] for n, qt in W.items() if len(qt.shape) == 2}
    patches, skipped = plan_patches(ad, 0.8, rows)
    assert skipped == ["transformer.single_transformer_blocks.1.unknown"]
    W2 = dict(W)
    for name, off, a, b, eff in patches:
        qt = W2[name]
        raw = oracle.lora_merge(qt.raw.reshape(-1), qt.ggml_type, qt.shape, off, b.shape[0], a, b, eff)
        W2[name] = F.QTensorRef(qt.ggml_type, qt.shape, raw.reshape(qt.raw.shape))

    img, ids, txt, tids, y = inputs(TINY, 40, 12, 10)
    t = lambda a: torch.from_numpy(a).to(cuda)
    run = lambda m: m.forward(t(img), t(ids), t(txt), t(tids), 0.7, t(y), 3.5)

    m = to_model(TINY, W, 64, 256)
    base = run(m)  # merge after the first forward: the captured work must read the new bytes
    n, sk = apply_lora(m, ad, 0.8)
    assert n == len(patches) and sk == skipped
    got = run(m)
    want = run(to_model(TINY, W2, 64, 256))
    assert torch.equal(got, want)
    assert not torch.equal(got, base)
    # and the merged model is the reference block math on the merged weights
    ref = F.forward(W2, TINY, img, ids, txt, tids, 0.7, y, 3.5)
    from tests.conftest import rel_l2
    assert rel_l2(got.cpu().numpy(), ref) < 2e-2
    assert mb.device_status() == 0
