"""Qwen-Image quantized-transformer math in numpy — TEST INFRASTRUCTURE ONLY.

A restatement of mold's quantized Qwen-Image transformer on its CPU path
(working dtype F32) and of the Qwen sampling glue:

  QwenLinear::forward          crates/mold-inference/src/qwen_image/quantized_transformer.rs:54-77
  DynamicRmsNorm               qwen_image/quantized_transformer.rs:96-108 (eps from config, 1e-6)
  LayerNormNoParams            qwen_image/quantized_transformer.rs:123-151 (eps 1e-6)
  QwenRopeEmbedder             qwen_image/quantized_transformer.rs:211-435 (axes 16/56/56, theta 10000:
                               frame index from 0, height/width centred with the negative half
                               first, text positions start at max(h/2, w/2) on every axis)
  TimestepProjEmbeddings       qwen_image/quantized_transformer.rs:577-602 (cos first, no x1000:
                               the caller passes t = sigma * 1000)
  FeedForward (GELU-tanh)      qwen_image/quantized_transformer.rs:604-641
  JointAttention::forward      qwen_image/quantized_transformer.rs:695-781 (key mask :799-816)
  QwenImageTransformerBlock    qwen_image/quantized_transformer.rs:856-959
  OutputLayer                  qwen_image/quantized_transformer.rs:962-989 (chunk order scale, shift)
  model forward                qwen_image/quantized_transformer.rs:1048-1139
  QwenImageScheduler           qwen_image/sampling.rs:19-129
  CFG + norm rescale           qwen_image/pipeline.rs:2693-2698

apply_rotary_emb (candle-transformers-mold 0.9.10 z_image, not vendored) is
taken as the rotation of interleaved pairs (x[2i], x[2i+1]) by the (seq, 64)
cos/sin tables, the form restated in-repo at ltx2/model/video_transformer.rs:811-833.
Block math is parity unpinned beyond this restatement; the scheduler is pinned
against qwen_image/sampling.rs:136-240.

The reference's CUDA path runs the transformer in bf16 (including the timestep
value and the residual stream); this oracle follows its f32 CPU path.
"""
import math
from dataclasses import dataclass

import numpy as np

from . import codec
from .flux_ref import (QTensorRef, embed_nd, gelu_tanh, layer_norm, linear, pick_type, rms_norm, sdpa, silu,
                       tensor_seed)


@dataclass
class QwenConfig:
    in_channels: int = 64        # 16 latent channels x 2 x 2 patch
    out_channels: int = 16
    patch_size: int = 2
    joint_attention_dim: int = 3584
    hidden_size: int = 3072
    num_heads: int = 24
    num_layers: int = 60
    mlp_hidden: int = 12288
    axes_dim: tuple = (16, 56, 56)
    theta: int = 10000

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads


def qwen_image_config():
    return QwenConfig()


ATTN_LINEARS = ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out")
NORMS = ("norm_q", "norm_k", "norm_added_q", "norm_added_k")


def weight_names(cfg: QwenConfig):
    """(name, shape, is_matrix) in the GGUF naming of the quantized transformer; matrices [out, in]."""
    h, m, hd = cfg.hidden_size, cfg.mlp_hidden, cfg.head_dim
    out = []

    def lin(n, o, i):
        out.extend([(n + ".weight", (o, i), True), (n + ".bias", (o,), False)])

    lin("time_text_embed.timestep_embedder.linear_1", h, 256)
    lin("time_text_embed.timestep_embedder.linear_2", h, h)
    lin("img_in", h, cfg.in_channels)
    lin("txt_in", h, cfg.joint_attention_dim)
    out.append(("txt_norm.weight", (cfg.joint_attention_dim,), False))
    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        for n in ATTN_LINEARS:
            lin(p + "attn." + n, h, h)
        for n in NORMS:
            out.append((p + "attn." + n + ".weight", (hd,), False))
        for s in ("img", "txt"):
            lin(p + f"{s}_mlp.net.0.proj", m, h)
            lin(p + f"{s}_mlp.net.2", h, m)
            lin(p + f"{s}_mod.1", 6 * h, h)
    lin("norm_out.linear", 2 * h, h)
    lin("proj_out", cfg.patch_size * cfg.patch_size * cfg.out_channels, h)
    return out


def synth_tensor(name, shape, is_matrix, seed, index, qtype):
    """Seeded synthetic tensor: matrices N(0, 0.02) quantized to `qtype`; biases N(0, 0.02);
    norm weights 1 + 0.02 N(0, 1)."""
    s = tensor_seed(seed, index)
    if is_matrix:
        x = codec.randn(s, shape, 0.02)
        t = pick_type(qtype, shape)
        return QTensorRef(t, shape, codec.quantize(x, t))
    if "norm" in name and name.endswith(".weight"):
        x = 1.0 + codec.randn(s, shape, 0.02)
    else:
        x = codec.randn(s, shape, 0.02)
    return QTensorRef(codec.GGML_F32, shape, codec.quantize(x.astype(np.float32), codec.GGML_F32))


def synth_weights(cfg: QwenConfig, seed=0, qtype=codec.GGML_Q4_K, only=None):
    w = {}
    for i, (name, shape, is_matrix) in enumerate(weight_names(cfg)):
        if only is not None and not only(name):
            continue
        w[name] = synth_tensor(name, shape, is_matrix, seed, i, qtype)
    return w


# ---------------------------------------------------------------- positions
def rope_ids(frame, h_tokens, w_tokens, txt_len):
    """Per-row RoPE positions (frame, row, col) of QwenRopeEmbedder::forward as an ids array.

    Image rows (f, y, x) in raster order: f from 0; y in [-(h - h//2), h//2), x likewise
    (centred_axis_freqs takes the last h - h//2 rows of the negative table, then h//2 rows
    of the positive one). Text row i: max(h//2, w//2) + i on all three axes."""
    hn, wn = h_tokens - h_tokens // 2, w_tokens - w_tokens // 2
    f = np.repeat(np.arange(frame, dtype=np.float32), h_tokens * w_tokens)
    y = np.tile(np.repeat(np.arange(h_tokens, dtype=np.float32) - hn, w_tokens), frame)
    x = np.tile(np.arange(w_tokens, dtype=np.float32) - wn, frame * h_tokens)
    img = np.stack([f, y, x], axis=1).astype(np.float32)
    s = max(h_tokens // 2, w_tokens // 2)
    t = (s + np.arange(txt_len, dtype=np.float32))
    txt = np.stack([t, t, t], axis=1).astype(np.float32)
    return img, txt


# ---------------------------------------------------------------- ops
def timestep_embedding(t, dim=256):
    """TimestepProjEmbeddings: freqs = exp(-ln(10000) i / half), cat[cos(t f), sin(t f)]."""
    half = dim // 2
    freqs = np.exp(np.arange(half, dtype=np.float32) * np.float32(-math.log(10000.0) / half)).astype(np.float32)
    args = np.float32(t) * freqs
    return np.concatenate([np.cos(args), np.sin(args)]).astype(np.float32)


def time_embed(W, t):
    p = "time_text_embed.timestep_embedder."
    e = timestep_embedding(t)[None, :]
    h = silu(linear(e, W[p + "linear_1.weight"], W.get(p + "linear_1.bias")))
    return linear(h, W[p + "linear_2.weight"], W.get(p + "linear_2.bias"))[0]


def apply_rope_lhd(x, pe):
    """x [L, H, D] interleaved pairs rotated by pe [L, D/2, 2, 2]."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    o0 = pe[:, None, :, 0, 0] * x0 + pe[:, None, :, 0, 1] * x1
    o1 = pe[:, None, :, 1, 0] * x0 + pe[:, None, :, 1, 1] * x1
    out = np.empty_like(x)
    out[..., 0::2] = o0
    out[..., 1::2] = o1
    return out


def modulate(x, shift, scale):
    return (layer_norm(x) * (1.0 + scale) + shift).astype(np.float32)


def block(W, p, cfg, img, txt, txt_mask, temb, pe_img, pe_txt):
    """QwenImageTransformerBlock::forward for one batch element: img [Li, h], txt [Lt, h],
    txt_mask [Lt] bool (True = attend), temb [h]."""
    H, D = cfg.num_heads, cfg.head_dim
    st = silu(temb)[None, :]
    im = np.split(linear(st, W[p + "img_mod.1.weight"], W.get(p + "img_mod.1.bias"))[0], 6)
    tm = np.split(linear(st, W[p + "txt_mod.1.weight"], W.get(p + "txt_mod.1.bias"))[0], 6)
    a = p + "attn."

    def proj(x, n):
        return linear(x, W[a + n + ".weight"], W.get(a + n + ".bias"))

    def heads(x):
        return x.reshape(x.shape[0], H, D)

    ii, ti = modulate(img, im[0], im[1]), modulate(txt, tm[0], tm[1])
    qi = apply_rope_lhd(rms_norm(heads(proj(ii, "to_q")), W[a + "norm_q.weight"].f32()), pe_img)
    ki = apply_rope_lhd(rms_norm(heads(proj(ii, "to_k")), W[a + "norm_k.weight"].f32()), pe_img)
    vi = heads(proj(ii, "to_v"))
    qt = apply_rope_lhd(rms_norm(heads(proj(ti, "add_q_proj")), W[a + "norm_added_q.weight"].f32()), pe_txt)
    kt = apply_rope_lhd(rms_norm(heads(proj(ti, "add_k_proj")), W[a + "norm_added_k.weight"].f32()), pe_txt)
    vt = heads(proj(ti, "add_v_proj"))
    q = np.concatenate([qt, qi], 0).transpose(1, 0, 2)
    k = np.concatenate([kt, ki], 0).transpose(1, 0, 2)
    v = np.concatenate([vt, vi], 0).transpose(1, 0, 2)
    key_mask = np.concatenate([np.asarray(txt_mask, bool), np.ones(img.shape[0], bool)])
    o = sdpa(np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v), key_mask)
    o = np.ascontiguousarray(o.transpose(1, 0, 2)).reshape(q.shape[1], H * D)
    lt = txt.shape[0]
    img = img + im[2] * proj(o[lt:], "to_out.0")
    txt = txt + tm[2] * proj(o[:lt], "to_add_out")

    def ff(x, s):
        g = gelu_tanh(linear(x, W[p + f"{s}_mlp.net.0.proj.weight"], W.get(p + f"{s}_mlp.net.0.proj.bias")))
        return linear(g, W[p + f"{s}_mlp.net.2.weight"], W.get(p + f"{s}_mlp.net.2.bias"))

    img = img + im[5] * ff(modulate(img, im[3], im[4]), "img")
    txt = txt + tm[5] * ff(modulate(txt, tm[3], tm[4]), "txt")
    return img.astype(np.float32), txt.astype(np.float32)


def output_layer(W, img, temb):
    mod = linear(silu(temb)[None, :], W["norm_out.linear.weight"], W.get("norm_out.linear.bias"))[0]
    scale, shift = np.split(mod, 2)
    return linear(modulate(img, shift, scale), W["proj_out.weight"], W.get("proj_out.bias"))


def forward(W, cfg, x_packed, t, txt, txt_mask, h_tokens, w_tokens, n_layers=None):
    """One batch element: x_packed [Li, 64] (patchified latent), t = sigma * 1000,
    txt [Lt, joint_attention_dim] encoder states, txt_mask [Lt] -> [Li, 64]."""
    temb = time_embed(W, t)
    img = linear(x_packed, W["img_in.weight"], W.get("img_in.bias"))
    txt = linear(rms_norm(txt, W["txt_norm.weight"].f32()), W["txt_in.weight"], W.get("txt_in.bias"))
    ids_img, ids_txt = rope_ids(1, h_tokens, w_tokens, txt.shape[0])
    pe_img = embed_nd(ids_img, cfg.axes_dim, cfg.theta)
    pe_txt = embed_nd(ids_txt, cfg.axes_dim, cfg.theta)
    for i in range(cfg.num_layers if n_layers is None else n_layers):
        img, txt = block(W, f"transformer_blocks.{i}.", cfg, img, txt, txt_mask, temb, pe_img, pe_txt)
    return output_layer(W, img, temb)


# ---------------------------------------------------------------- scheduler + CFG
NUM_TRAIN_TIMESTEPS = 1000
BASE_IMAGE_SEQ_LEN, MAX_IMAGE_SEQ_LEN = 256, 8192
BASE_SHIFT, MAX_SHIFT, SHIFT_TERMINAL = 0.5, 0.9, 0.02


def calculate_shift(image_seq_len):
    m = (MAX_SHIFT - BASE_SHIFT) / (MAX_IMAGE_SEQ_LEN - BASE_IMAGE_SEQ_LEN)
    return image_seq_len * m + (BASE_SHIFT - m * BASE_IMAGE_SEQ_LEN)


def time_shift_exponential(mu, sigma, t):
    return math.exp(mu) / (math.exp(mu) + (1.0 / t - 1.0) ** sigma)


def stretch_shift_to_terminal(sigmas):
    one_minus_z = 1.0 - sigmas[-1]
    if abs(one_minus_z) < 1e-12:
        return list(sigmas)
    scale = one_minus_z / (1.0 - SHIFT_TERMINAL)
    return [1.0 - (1.0 - s) / scale for s in sigmas]


def scheduler_sigmas(num_steps, image_seq_len):
    """QwenImageScheduler::new: linspace(1, 1/N, N), exponential shift, terminal stretch, append 0."""
    if num_steps == 1:
        s = [1.0]
    else:
        step = (1.0 / num_steps - 1.0) / (num_steps - 1)
        s = [1.0 + step * i for i in range(num_steps)]
    mu = calculate_shift(image_seq_len)
    s = [time_shift_exponential(mu, 1.0, x) for x in s]
    return stretch_shift_to_terminal(s) + [0.0]


def cfg_combine(cond, uncond, guidance):
    """pipeline.rs:2693-2698 on [C, H, W] latents (dim 1 of [B, C, H, W] is C here):
    comb = u + g (c - u), rescaled per pixel by ||c|| / max(||comb||, 1e-8) over channels."""
    c = cond.astype(np.float32)
    u = uncond.astype(np.float32)
    comb = u + (c - u) * np.float32(guidance)
    cn = np.sqrt((c.astype(np.float64) ** 2).sum(0, keepdims=True))
    bn = np.maximum(np.sqrt((comb.astype(np.float64) ** 2).sum(0, keepdims=True)), 1e-8)
    return (comb * (cn / bn)).astype(np.float32)


def denoise(W, cfg, latent, txt_c, mask_c, sigmas, txt_u=None, mask_u=None, guidance=1.0, n_layers=None,
            inpaint=None):
    """The Qwen denoise loop on a [C, H, W] latent: t = sigma * 1000, CFG when an unconditional
    prompt is given, Euler x += pred * (sigma_next - sigma) in f32."""
    from .flux_ref import patchify, unpack
    c, hh, ww = latent.shape
    x = latent.astype(np.float32).copy()
    for s, s_next in zip(sigmas[:-1], sigmas[1:]):
        t = s * NUM_TRAIN_TIMESTEPS
        xp = patchify(x)
        pc = unpack(forward(W, cfg, xp, t, txt_c, mask_c, hh // 2, ww // 2, n_layers), hh, ww)
        if txt_u is not None:
            pu = unpack(forward(W, cfg, xp, t, txt_u, mask_u, hh // 2, ww // 2, n_layers), hh, ww)
            pred = cfg_combine(pc, pu, guidance)
        else:
            pred = pc
        x = (x + pred * np.float32(s_next - s)).astype(np.float32)
        if inpaint is not None:  # pipeline.rs:2708-2715 at sigmas[step + 1], [C, H, W] operands
            from .flux_ref import inpaint_blend
            x = inpaint_blend(x, inpaint, s_next)
    return x
