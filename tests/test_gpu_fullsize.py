"""The headline workload's own shapes (FLUX.1-dev at 1024x1024: 4608 tokens, hidden 3072, 24
heads) through the C ABI, checked against plain PyTorch fp32 references of the same op on the
GPU (the oracle's numpy path is too slow at these sizes): the single-block linear1 GEMM in Q4_K
and Q8_0, and the joint attention."""
import pytest
import torch

import bench
import mold_b200 as mb
import oracle

pytestmark = pytest.mark.gpu

M, N, K = 4608, 21504, 3072


def weight(qt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((N, K), device="cuda", generator=g) * 0.02
    raw = bench.q4k_quantize_torch(x) if qt == mb.GGML_Q4_K else bench.q8_0_quantize_torch(x)
    return mb.QMatMul.from_weights(mb.QTensor(qt, (N, K), raw.cpu().numpy()))


@pytest.mark.parametrize("qt", [mb.GGML_Q4_K, mb.GGML_Q8_0])
def test_linear1_full_size(cuda, qt):
    w = weight(qt, 1)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn((M, K), device="cuda", generator=g).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g) * 0.02
    y = w.forward(x, bias=bias, out_dtype=torch.float32)
    # the oracle's decode of the same GGUF bytes (C, on the host), bit-equal to the device decode
    wf = torch.from_numpy(oracle.dequantize(w.download(), qt, (N, K))).cuda()
    assert torch.equal(mb.dequantize(w, torch.float32), wf)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        # fp32 reference on the bf16 operands the tensor core sees (the exact decode rounded to bf16)
        ref = x.float() @ wf.bfloat16().float().t() + bias
        err = ((y - ref).norm() / ref.norm()).item()
        assert err < 1e-4, err
        # and against the unrounded decode (what the GGML weights mean)
        ref32 = x.float() @ wf.t() + bias
        assert ((y - ref32).norm() / ref32.norm()).item() < 4e-3
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert mb.device_status() == 0


def test_linear1_full_size_gelu_epilogue(cuda):
    w = weight(mb.GGML_Q4_K, 3)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn((M, K), device="cuda", generator=g).bfloat16()
    y = w.forward(x, epilogue=mb.EPI_GELU_TANH, gelu_from=9216, out_dtype=torch.float32)
    pre = x.float() @ mb.dequantize(w, torch.bfloat16).float().t()
    ref = torch.cat([pre[:, :9216], torch.nn.functional.gelu(pre[:, 9216:], approximate="tanh")], dim=1)
    assert ((y - ref).norm() / ref.norm()).item() < 2e-3


def test_joint_attention_full_size(cuda):
    H, L = 24, 4608
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn((H, L, 128), device="cuda", generator=g).bfloat16() for _ in range(3))
    out = mb.attention(q, k, v).float()  # [L, H * 128]
    ref = torch.nn.functional.scaled_dot_product_attention(q.float()[None], k.float()[None], v.float()[None])[0]
    ref = ref.transpose(0, 1).reshape(L, H * 128)
    assert ((out - ref).norm() / ref.norm()).item() < 1e-2
    assert mb.device_status() == 0


def test_flux_full_size_denoise_deterministic_and_finite(cuda):
    """The headline configuration end to end (FLUX.1-dev Q4_K 1024x1024, 4096 + 512 tokens, the
    28-step schedule): two denoise calls from the same latent give bit-identical results, and the
    result is finite. (No reference run at this size exists here; the block math is checked
    against the oracle at smaller sizes.)"""
    model, cfg, _ = bench.build_flux("q4_k", 0)
    g = torch.Generator(device="cuda").manual_seed(7)
    latent = torch.randn((16, bench.LAT_H, bench.LAT_W), generator=g, device="cuda")
    img0 = mb.sampling.patchify(latent).contiguous()
    img_ids = mb.sampling.img_ids(bench.LAT_H // 2, bench.LAT_W // 2, device="cuda")
    txt = torch.randn((bench.L_TXT, cfg.context_in_dim), generator=g, device="cuda")
    txt_ids = mb.sampling.txt_ids(bench.L_TXT, device="cuda")
    y = torch.randn((cfg.vec_in_dim,), generator=g, device="cuda")
    sched = mb.sampling.get_schedule(28, bench.L_IMG)
    outs = []
    for _ in range(2):
        img = img0.clone()
        model.denoise(img, img_ids, txt, txt_ids, y, sched, bench.GUIDANCE)
        torch.cuda.synchronize()
        outs.append(img)
    assert mb.device_status() == 0
    assert torch.isfinite(outs[0]).all()
    assert torch.equal(outs[0], outs[1])
    assert not torch.equal(outs[0], img0)
