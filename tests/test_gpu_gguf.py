"""Models loaded from GGUF files (mb_flux_load_gguf / mb_qwen_load_gguf) give the same result
as models fed tensor by tensor, including the city96 embedding patch."""
import dataclasses

import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from oracle import qwen_ref as Q
from tests.gguf_util import write_gguf
from tests.test_gpu_flux import TINY, inputs, to_model

pytestmark = pytest.mark.gpu

EMB = ("img_in.", "time_in.", "vector_in.", "guidance_in.")


def flux_cfg(c):
    return mb.FluxConfig(in_channels=c.in_channels, vec_in_dim=c.vec_in_dim, context_in_dim=c.context_in_dim,
                         hidden_size=c.hidden_size, mlp_ratio=c.mlp_ratio, num_heads=c.num_heads, depth=c.depth,
                         depth_single_blocks=c.depth_single_blocks, axes_dim=c.axes_dim, theta=c.theta,
                         guidance_embed=c.guidance_embed)


def run_flux(m, cuda):
    img, ids, txt, tids, y = inputs(TINY, 40, 12, 10)
    t = lambda a: torch.from_numpy(a).to(cuda)
    return m.forward(t(img), t(ids), t(txt), t(tids), 0.7, t(y), 3.5)


def test_flux_from_gguf_equals_set_tensor(cuda, tmp_path):
    W = F.synth_weights(TINY, seed=7, qtype=oracle.GGML_Q4_K)
    path = tmp_path / "flux.gguf"
    write_gguf(path, W)
    ref = run_flux(to_model(TINY, W, 64, 256), cuda)
    m = mb.FluxTransformer(flux_cfg(TINY), max_txt=64, max_img=256)
    assert m.load_gguf(path) == len(W)
    assert m.missing() == []
    assert torch.equal(run_flux(m, cuda), ref)


def test_flux_city96_embedding_patch(cuda, tmp_path):
    W = F.synth_weights(TINY, seed=8, qtype=oracle.GGML_Q6_K)
    main = {n: v for n, v in W.items() if not n.startswith(EMB)}
    emb = {n: v for n, v in W.items() if n.startswith(EMB)}
    write_gguf(tmp_path / "finetune.gguf", main)
    write_gguf(tmp_path / "dev.gguf", {**emb, "double_blocks.0.img_mod.lin.bias": W["double_blocks.0.img_mod.lin.bias"]})
    m = mb.FluxTransformer(flux_cfg(TINY), max_txt=64, max_img=256)
    m.load_gguf(tmp_path / "finetune.gguf")
    assert set(m.missing()) == set(emb)
    m2 = mb.FluxTransformer(flux_cfg(TINY), max_txt=64, max_img=256)
    assert m2.load_gguf(tmp_path / "finetune.gguf", embeddings_path=tmp_path / "dev.gguf") == len(W)
    assert m2.missing() == []
    assert torch.equal(run_flux(m2, cuda), run_flux(to_model(TINY, W, 64, 256), cuda))


def test_qwen_from_gguf_equals_set_tensor(cuda, tmp_path):
    cfg_o = Q.QwenConfig(joint_attention_dim=256, hidden_size=256, num_heads=2, num_layers=2, mlp_hidden=1024)
    W = Q.synth_weights(cfg_o, seed=9, qtype=oracle.GGML_Q5_K)
    write_gguf(tmp_path / "qwen.gguf", W, arch="qwen_image")
    cfg = mb.QwenConfig(**dataclasses.asdict(cfg_o))
    a = mb.QwenTransformer(cfg, max_txt=32, max_img=64, max_batch=1)
    for n, qt in W.items():
        a.set_tensor(n, mb.QTensor(qt.ggml_type, qt.shape, qt.raw))
    b = mb.QwenTransformer(cfg, max_txt=32, max_img=64, max_batch=1)
    assert b.load_gguf(tmp_path / "qwen.gguf") == len(W)
    x = torch.from_numpy(oracle.randn(1, (1, 64, 64))).to(cuda)
    txt = torch.from_numpy(oracle.randn(2, (1, 24, 256))).to(cuda)
    assert torch.equal(a.forward(x, 500.0, txt, None, 8, 8), b.forward(x, 500.0, txt, None, 8, 8))
