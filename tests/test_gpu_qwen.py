"""Qwen-Image path through the C ABI (mb_qwen_*, mb_rms_norm, mb_cfg_euler_step,
mb_qk_norm_rope_ex, mb_attention_ex) against the numpy oracle."""
import dataclasses

import numpy as np
import pytest
import torch

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from oracle import qwen_ref as Q
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TINY = Q.QwenConfig(joint_attention_dim=256, hidden_size=256, num_heads=2, num_layers=2, mlp_hidden=1024)


def to_model(cfg_o, W, max_txt, max_img, max_batch=2):
    m = mb.QwenTransformer(mb.QwenConfig(**dataclasses.asdict(cfg_o)), max_txt=max_txt, max_img=max_img,
                           max_batch=max_batch)
    for name, qt in W.items():
        m.set_tensor(name, mb.QTensor(qt.ggml_type, qt.shape, qt.raw))
    assert m.missing() == []
    return m


def t(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def masks(lt):
    m0 = np.zeros(lt, np.uint8)
    m0[: lt - 11] = 1                                   # tokenizer-style padding at the end
    rng = np.random.default_rng(5)
    m1 = (rng.random(lt) < 0.6).astype(np.uint8)        # arbitrary pattern
    return np.stack([m0, m1])


# ------------------------------------------------------------------ single kernels
def test_rms_norm(cuda):
    x = oracle.randn(31, (300, 3584))
    w = 1.0 + oracle.randn(32, (3584,), 0.02)
    ref = F.rms_norm(x, w)
    got = mb.rms_norm(t(x, cuda), t(w, cuda)).float().cpu().numpy()
    assert rel_l2(got, ref) < 5e-3


@pytest.mark.parametrize("g", [1.0, 4.0])
def test_cfg_euler_step(cuda, g):
    hh, ww = 12, 10
    cond = oracle.randn(41, (16, hh, ww))
    unc = oracle.randn(42, (16, hh, ww))
    img = oracle.randn(43, (16, hh, ww))
    dt = -0.0371
    ref = img + Q.cfg_combine(cond, unc, g) * np.float32(dt)
    gi = t(F.patchify(img), cuda)
    mb.cfg_euler_step(gi, t(F.patchify(cond), cuda), t(F.patchify(unc), cuda), g, dt)
    got = F.unpack(gi.cpu().numpy(), hh, ww)
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("lt,li", [(70, 200), (256, 1024), (5, 130)])
def test_masked_joint_attention(cuda, lt, li):
    """QK-RMSNorm + RoPE with the kept-keys-first order, then attention over the kept prefix
    with the output split into text / image rows, against masked SDPA on cat[txt, img]."""
    H, D = 3, 128
    L = lt + li
    rng = np.random.default_rng(lt)
    mask = (rng.random(lt) < 0.55).astype(np.uint8)
    mask[0] = 1
    qkv = oracle.round_bf16(oracle.randn(lt + 7, (L, 3 * H * D)))
    qs = 1.0 + oracle.randn(2, (D,), 0.02)
    ks = 1.0 + oracle.randn(3, (D,), 0.02)
    ids_img, ids_txt = Q.rope_ids(1, li // 10, 10, lt) if li % 10 == 0 else Q.rope_ids(1, li, 1, lt)
    pe = F.embed_nd(np.concatenate([ids_txt, ids_img]), (16, 56, 56), 10000)
    q, k, v = F.split_qkv(qkv, H)
    q = F.apply_rope(F.rms_norm(q, qs), pe)
    k = F.apply_rope(F.rms_norm(k, ks), pe)
    keep = np.concatenate([mask.astype(bool), np.ones(li, bool)])
    ref = F.sdpa(q, k, v, keep).transpose(1, 0, 2).reshape(L, H * D)
    pos, nv = mb.key_order(torch.from_numpy(mask), li)
    gq, gk, gv = mb.qk_norm_rope(t(qkv, cuda).bfloat16(), H, t(qs, cuda), t(ks, cuda), t(pe, cuda),
                                 kv_pos=pos.to(cuda))
    ot, oi = mb.attention(gq, gk, gv, n_valid_keys=nv, split_row=lt)
    got = np.concatenate([ot.float().cpu().numpy(), oi.float().cpu().numpy()])
    assert rel_l2(got, ref) < 1e-2
    assert mb.device_status() == 0


# ------------------------------------------------------------------ model
@pytest.mark.parametrize("qtype", [oracle.GGML_Q4_K, oracle.GGML_Q8_0])
def test_tiny_qwen_forward_batch2_masked(cuda, qtype):
    W = Q.synth_weights(TINY, seed=3, qtype=qtype)
    m = to_model(TINY, W, 64, 256)
    hh, ww, lt = 9, 13, 40                                  # odd grid: centred positions
    li = hh * ww
    x = oracle.randn(50, (2, li, TINY.in_channels))
    txt = oracle.randn(51, (2, lt, TINY.joint_attention_dim))
    mk = masks(lt)
    got = m.forward(t(x, cuda), 512.0, t(txt, cuda), t(mk, cuda), hh, ww).cpu().numpy()
    for b in range(2):
        ref = Q.forward(W, TINY, x[b], 512.0, txt[b], mk[b].astype(bool), hh, ww)
        assert rel_l2(got[b], ref) < 2e-2, b
    assert mb.device_status() == 0


def test_tiny_qwen_forward_no_mask_equals_all_ones(cuda):
    W = Q.synth_weights(TINY, seed=4, qtype=oracle.GGML_Q4_K)
    m = to_model(TINY, W, 64, 256, max_batch=1)
    x = oracle.randn(60, (1, 64, TINY.in_channels))
    txt = oracle.randn(61, (1, 24, TINY.joint_attention_dim))
    a = m.forward(t(x, cuda), 900.0, t(txt, cuda), None, 8, 8)
    b = m.forward(t(x, cuda), 900.0, t(txt, cuda), torch.ones((1, 24), dtype=torch.uint8, device=cuda), 8, 8)
    assert torch.equal(a, b)


@pytest.mark.parametrize("cfg_batch", [True, False])
def test_tiny_qwen_denoise_cosine(cuda, cfg_batch):
    W = Q.synth_weights(TINY, seed=5, qtype=oracle.GGML_Q4_K)
    m = to_model(TINY, W, 64, 256)
    hh, ww, lt = 8, 10, 32
    latent = oracle.randn(70, (TINY.out_channels, 2 * hh, 2 * ww))
    txt = oracle.randn(71, (2, lt, TINY.joint_attention_dim))
    mk = masks(lt)
    sig = Q.scheduler_sigmas(4, hh * ww)
    if cfg_batch:
        ref = Q.denoise(W, TINY, latent, txt[0], mk[0].astype(bool), sig, txt[1], mk[1].astype(bool), 4.0)
        gt, gm = t(txt, cuda), t(mk, cuda)
    else:
        ref = Q.denoise(W, TINY, latent, txt[0], mk[0].astype(bool), sig)
        gt, gm = t(txt[:1], cuda), t(mk[:1], cuda)
    gi = t(F.patchify(latent), cuda)
    m.denoise(gi, gt, gm, hh, ww, sig, 4.0)
    got = F.unpack(gi.cpu().numpy(), 2 * hh, 2 * ww)
    cos = float(np.dot(got.ravel(), ref.ravel()) / np.linalg.norm(got) / np.linalg.norm(ref))
    assert cos >= 0.999, cos
    gi2 = t(F.patchify(latent), cuda)                      # replay of the captured graph
    m.denoise(gi2, gt, gm, hh, ww, sig, 4.0)
    assert rel_l2(F.unpack(gi2.cpu().numpy(), 2 * hh, 2 * ww), got) < 1e-6


def test_config5_one_block_q4k(cuda):
    """Config 5 widths (hidden 3072, 24 heads, text width 3584, Q4_K) with one block:
    256 text tokens of which 200 are kept, a 32 x 32 token image, seed 0."""
    cfg = Q.QwenConfig(num_layers=1)
    W = Q.synth_weights(cfg, seed=0, qtype=oracle.GGML_Q4_K)
    m = to_model(cfg, W, 256, 1024, max_batch=1)
    hh = ww = 32
    x = oracle.randn(80, (1, hh * ww, cfg.in_channels))
    txt = oracle.randn(81, (1, 256, cfg.joint_attention_dim))
    mk = np.zeros((1, 256), np.uint8)
    mk[0, :200] = 1
    ref = Q.forward(W, cfg, x[0], 700.0, txt[0], mk[0].astype(bool), hh, ww)
    got = m.forward(t(x, cuda), 700.0, t(txt, cuda), t(mk, cuda), hh, ww).cpu().numpy()[0]
    assert rel_l2(got, ref) < 1e-2


def test_tiny_qwen_denoise_inpaint_and_progress(cuda):
    """The Qwen step loop with the flow-matching inpaint blend at sigma_next and per-step
    progress (qwen_image/pipeline.rs:2708-2724) through mb_qwen_denoise_ex, CFG batch 2."""
    W = Q.synth_weights(TINY, seed=6, qtype=oracle.GGML_Q4_K)
    m = to_model(TINY, W, 64, 256)
    hh, ww, lt = 8, 10, 32
    latent = oracle.randn(72, (TINY.out_channels, 2 * hh, 2 * ww))
    orig = oracle.randn(73, latent.shape)
    mask = np.broadcast_to((np.random.default_rng(4).random((1, 2 * hh, 2 * ww)) < 0.5), latent.shape)
    mask = np.ascontiguousarray(mask, dtype=np.float32)
    txt = oracle.randn(74, (2, lt, TINY.joint_attention_dim))
    mk = masks(lt)
    sig = Q.scheduler_sigmas(4, hh * ww)
    ref = Q.denoise(W, TINY, latent, txt[0], mk[0].astype(bool), sig, txt[1], mk[1].astype(bool), 4.0,
                    inpaint=(mask, orig, latent))
    seen = []
    gi = t(F.patchify(latent), cuda)
    m.denoise(gi, t(txt, cuda), t(mk, cuda), hh, ww, sig, 4.0,
              inpaint=(t(F.patchify(mask), cuda), t(F.patchify(orig), cuda), t(F.patchify(latent), cuda)),
              on_step=lambda step, total: seen.append(step))
    torch.cuda.synchronize()
    got = F.unpack(gi.cpu().numpy(), 2 * hh, 2 * ww)
    assert seen == [1, 2, 3, 4]
    assert rel_l2(got, ref) < 2e-2
    keep = mask == 0  # the last sigma is 0: preserved pixels hold the original exactly
    assert np.allclose(got[keep], orig[keep], atol=1e-6)
