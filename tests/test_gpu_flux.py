"""FLUX forward / denoise through the C ABI (mb_flux_*) against the numpy oracle."""
import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


def to_model(cfg_o, W, max_txt, max_img):
    cfg = mb.FluxConfig(in_channels=cfg_o.in_channels, vec_in_dim=cfg_o.vec_in_dim,
                        context_in_dim=cfg_o.context_in_dim, hidden_size=cfg_o.hidden_size,
                        mlp_ratio=cfg_o.mlp_ratio, num_heads=cfg_o.num_heads, depth=cfg_o.depth,
                        depth_single_blocks=cfg_o.depth_single_blocks, axes_dim=cfg_o.axes_dim,
                        theta=cfg_o.theta, guidance_embed=cfg_o.guidance_embed)
    m = mb.FluxTransformer(cfg, max_txt=max_txt, max_img=max_img)
    for name, qt in W.items():
        m.set_tensor(name, mb.QTensor(qt.ggml_type, qt.shape, qt.raw))
    assert m.missing() == []
    return m


def inputs(cfg, lt, hh, ww, seed=100):
    img = oracle.randn(seed, (hh * ww, cfg.in_channels))
    ids = F.img_ids(hh, ww)
    txt = oracle.randn(seed + 1, (lt, cfg.context_in_dim))
    tids = np.zeros((lt, 3), np.float32)
    y = oracle.randn(seed + 2, (cfg.vec_in_dim,))
    return img, ids, txt, tids, y


TINY = F.FluxConfig(hidden_size=256, num_heads=2, mlp_ratio=4.0, depth=2, depth_single_blocks=2,
                    context_in_dim=256, vec_in_dim=256)


@pytest.mark.parametrize("qtype", [oracle.GGML_Q4_K, oracle.GGML_Q8_0])
def test_tiny_flux_forward(cuda, qtype):
    W = F.synth_weights(TINY, seed=1, qtype=qtype)
    m = to_model(TINY, W, 64, 256)
    img, ids, txt, tids, y = inputs(TINY, 40, 12, 10)
    ref = F.forward(W, TINY, img, ids, txt, tids, 0.7, y, 3.5)
    t = lambda a: torch.from_numpy(a).to(cuda)
    pred = m.forward(t(img), t(ids), t(txt), t(tids), 0.7, t(y), 3.5).cpu().numpy()
    assert mb.device_status() == 0
    assert rel_l2(pred, ref) < 2e-2


def test_tiny_flux_denoise_cosine(cuda):
    W = F.synth_weights(TINY, seed=2, qtype=oracle.GGML_Q4_K)
    m = to_model(TINY, W, 64, 256)
    img, ids, txt, tids, y = inputs(TINY, 32, 8, 8, seed=200)
    ts = mb.sampling.get_schedule(6, 64)  # the product's schedule (equal to the oracle's, tests/test_sampling.py)
    ref = F.denoise(W, TINY, img, ids, txt, tids, y, ts, 3.5)
    t = lambda a: torch.from_numpy(a).to(cuda)
    gi = t(img).clone()
    m.denoise(gi, t(ids), t(txt), t(tids), t(y), ts, 3.5)
    got = gi.cpu().numpy()
    cos = float(np.dot(got.ravel(), ref.ravel()) / np.linalg.norm(got) / np.linalg.norm(ref))
    assert cos >= 0.999, cos
    # a second call replays the captured step graph and must give the same result
    gi2 = t(img).clone()
    m.denoise(gi2, t(ids), t(txt), t(tids), t(y), ts, 3.5)
    assert torch.equal(gi2, gi) or rel_l2(gi2.cpu().numpy(), got) < 1e-6


def test_config1_single_block_q8(cuda):
    """one FLUX single-stream block, 512 txt + 1024 img tokens,
    hidden 3072, Q8_0 linears, seed 0, through the model API (stems + 1 single block + final)."""
    cfg = F.FluxConfig(depth=0, depth_single_blocks=1)
    W = F.synth_weights(cfg, seed=0, qtype=oracle.GGML_Q8_0)
    m = to_model(cfg, W, 512, 1024)
    img, ids, txt, tids, y = inputs(cfg, 512, 32, 32, seed=0)
    ref = F.forward(W, cfg, img, ids, txt, tids, 0.5, y, 3.5)
    t = lambda a: torch.from_numpy(a).to(cuda)
    pred = m.forward(t(img), t(ids), t(txt), t(tids), 0.5, t(y), 3.5).cpu().numpy()
    assert rel_l2(pred, ref) < 1e-2


def test_config1_single_block_ops(cuda):
    """Per-layer check of the single block itself (rel-L2 <= 1e-2 of the block output),
    composing the C-ABI ops in the order the model runs them."""
    cfg = F.FluxConfig(depth=0, depth_single_blocks=1)
    h, H = 3072, 24
    W = F.synth_weights(cfg, seed=0, qtype=oracle.GGML_Q8_0, only=lambda n: n.startswith("single_blocks.0."))
    p = "single_blocks.0."
    Lt, Li = 512, 1024
    x = oracle.randn(1, (Lt + Li, h))
    vec = oracle.randn(2, (h,))
    ids = np.concatenate([np.zeros((Lt, 3), np.float32), F.img_ids(32, 32)])
    pe = F.embed_nd(ids, cfg.axes_dim, cfg.theta)
    ref = F.single_block(W, p, cfg, x, vec, pe)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    qm = {n: mb.QMatMul.from_weights(mb.QTensor(W[n].ggml_type, W[n].shape, W[n].raw))
          for n in W if n.endswith("weight")}
    vecs = {n: t(W[n].f32()) for n in W if not n.endswith("weight")}
    mods = mb.qgemv(qm[p + "modulation.lin.weight"], t(vec), apply_silu=True, bias=vecs[p + "modulation.lin.bias"])
    shift, scale, gate = mods[:h], mods[h:2 * h], mods[2 * h:]
    xg = t(x)
    xm = mb.ln_modulate(xg, shift, scale)
    Y = qm[p + "linear1.weight"].forward(xm, bias=vecs[p + "linear1.bias"], epilogue=mb.EPI_GELU_TANH,
                                         gelu_from=3 * h)
    q, k, v = mb.qk_norm_rope(Y, H, vecs[p + "norm.query_norm.scale"], vecs[p + "norm.key_norm.scale"], t(pe))
    mb.attention(q, k, v, out=Y[:, 2 * h:3 * h])
    qm[p + "linear2.weight"].forward(Y[:, 2 * h:], bias=vecs[p + "linear2.bias"], epilogue=mb.EPI_GATE_RESIDUAL,
                                     gate=gate, residual=xg, out=xg)
    err = rel_l2(xg.cpu().numpy() - x, ref - x)  # error relative to the block's update
    assert err < 1e-2, err
    assert rel_l2(xg.cpu().numpy(), ref) < 1e-2


def test_tiny_flux_denoise_inpaint_and_progress(cuda):
    """FluxTransformer::denoise with an inpaint context and progress events
    (flux/transformer.rs:79-93) through mb_flux_denoise_ex: the blend runs inside the replayed
    step graph, the callback reports steps 1..n in order, and the result matches the oracle."""
    W = F.synth_weights(TINY, seed=2, qtype=oracle.GGML_Q4_K)
    m = to_model(TINY, W, 64, 256)
    img, ids, txt, tids, y = inputs(TINY, 32, 8, 8, seed=210)
    ts = mb.sampling.get_schedule(6, 64)
    mask = (np.random.default_rng(3).random((64, 1)) < 0.5).astype(np.float32) * np.ones((1, 64), np.float32)
    orig = oracle.randn(211, img.shape)
    noise = img.copy()
    ref = F.denoise(W, TINY, img, ids, txt, tids, y, ts, 3.5, inpaint=(mask, orig, noise))
    t = lambda a: torch.from_numpy(a).to(cuda)
    seen = []
    gi = t(img).clone()
    m.denoise(gi, t(ids), t(txt), t(tids), t(y), ts, 3.5, inpaint=(t(mask), t(orig), t(noise)),
              on_step=lambda step, total: seen.append((step, total)))
    torch.cuda.synchronize()
    got = gi.cpu().numpy()
    assert seen == [(i, 6) for i in range(1, 7)]
    cos = float(np.dot(got.ravel(), ref.ravel()) / np.linalg.norm(got) / np.linalg.norm(ref))
    assert cos >= 0.999, cos
    # preserved tokens hold exactly the re-noised original at the last t (0): the original
    keep = mask[:, 0] == 0
    assert np.allclose(got[keep], orig[keep], atol=1e-6)
    assert rel_l2(got[~keep], ref[~keep]) < 2e-2
