"""FLUX.1 quantized-transformer math in numpy — TEST INFRASTRUCTURE ONLY.

A restatement of the block math mold runs through candle's
`flux::quantized_model::Flux` (third-party, candle-transformers-mold 0.9.10).
mold's own in-repo copy of that math is the spec followed here:

  timestep_embedding      crates/mold-inference/src/flux/offload.rs:21-38
  scaled_dot_product_attn flux/offload.rs:40-54
  apply_rope / attention  flux/offload.rs:56-72
  Modulation1/2           flux/offload.rs:102-156 (silu(vec) -> lin -> chunk)
  SelfAttention.qkv       flux/offload.rs:191-201 ((b,l,3,H,D) split, RMSNorm eps 1e-6)
  Mlp                     flux/offload.rs:222-224 (lin1 -> gelu -> lin2)
  DoubleBlock.forward     flux/offload.rs:275-323
  SingleBlock.forward     flux/offload.rs:377-396
  FinalLayer.forward      flux/offload.rs:421-429
  Flux forward order      flux/offload.rs:525-580
  rope / EmbedNd          flux2/transformer.rs:99-118,170-184 (FLUX.1: theta 10000, axes 16/56/56)
  Euler step              flux/transformer.rs:84  img += pred * (t_prev - t_curr)
  get_schedule            candle flux::sampling::get_schedule, called at flux/pipeline.rs:2044-2048
                          (shift (seq_len, 0.5, 1.15); same form as qwen_image/sampling.rs:19-27)
  State::new / unpack     flux2/sampling.rs:37-72,149-159 (FLUX.1 ids are (0, row, col))

Precision: f32 storage, BLAS f32 matmuls, f64 for norm statistics. Weights
are dequantized with the bit-exact GGML decode in codec.c. Open points
(unpinned): candle's `Tensor::gelu` is taken as the tanh form; candle's CPU
QMatMul may quantize activations to 8 bits before its integer dot products,
this oracle does not (f32 x f32, closer to the true linear).
"""
import math
from dataclasses import dataclass, field

import numpy as np

from . import codec


@dataclass
class FluxConfig:
    in_channels: int = 64
    vec_in_dim: int = 768
    context_in_dim: int = 4096
    hidden_size: int = 3072
    mlp_ratio: float = 4.0
    num_heads: int = 24
    depth: int = 19
    depth_single_blocks: int = 38
    axes_dim: tuple = (16, 56, 56)
    theta: int = 10000
    qkv_bias: bool = True
    guidance_embed: bool = True

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads

    @property
    def mlp_hidden(self):
        return int(self.hidden_size * self.mlp_ratio)


def flux_dev_config():
    return FluxConfig()


# ---------------------------------------------------------------- weights
@dataclass
class QTensorRef:
    """A GGUF tensor: ggml type, logical shape (rows=N out, cols=K in), raw bytes."""
    ggml_type: int
    shape: tuple
    raw: np.ndarray = field(repr=False)

    def f32(self):
        return codec.dequantize(self.raw, self.ggml_type, self.shape)


def weight_names(cfg: FluxConfig):
    """(name, shape, is_matrix) in GGUF naming; matrices are [out, in]."""
    h, m, hd = cfg.hidden_size, cfg.mlp_hidden, cfg.head_dim
    out = [("img_in.weight", (h, cfg.in_channels), True), ("img_in.bias", (h,), False),
           ("txt_in.weight", (h, cfg.context_in_dim), True), ("txt_in.bias", (h,), False)]
    for stem, k in (("time_in", 256), ("vector_in", cfg.vec_in_dim), ("guidance_in", 256)):
        if stem == "guidance_in" and not cfg.guidance_embed:
            continue
        out += [(f"{stem}.in_layer.weight", (h, k), True), (f"{stem}.in_layer.bias", (h,), False),
                (f"{stem}.out_layer.weight", (h, h), True), (f"{stem}.out_layer.bias", (h,), False)]
    for i in range(cfg.depth):
        p = f"double_blocks.{i}."
        for s in ("img", "txt"):
            out += [(p + f"{s}_mod.lin.weight", (6 * h, h), True), (p + f"{s}_mod.lin.bias", (6 * h,), False),
                    (p + f"{s}_attn.qkv.weight", (3 * h, h), True), (p + f"{s}_attn.qkv.bias", (3 * h,), False),
                    (p + f"{s}_attn.norm.query_norm.scale", (hd,), False),
                    (p + f"{s}_attn.norm.key_norm.scale", (hd,), False),
                    (p + f"{s}_attn.proj.weight", (h, h), True), (p + f"{s}_attn.proj.bias", (h,), False),
                    (p + f"{s}_mlp.0.weight", (m, h), True), (p + f"{s}_mlp.0.bias", (m,), False),
                    (p + f"{s}_mlp.2.weight", (h, m), True), (p + f"{s}_mlp.2.bias", (h,), False)]
    for i in range(cfg.depth_single_blocks):
        p = f"single_blocks.{i}."
        out += [(p + "linear1.weight", (3 * h + m, h), True), (p + "linear1.bias", (3 * h + m,), False),
                (p + "linear2.weight", (h, h + m), True), (p + "linear2.bias", (h,), False),
                (p + "norm.query_norm.scale", (hd,), False), (p + "norm.key_norm.scale", (hd,), False),
                (p + "modulation.lin.weight", (3 * h, h), True), (p + "modulation.lin.bias", (3 * h,), False)]
    out += [("final_layer.linear.weight", (cfg.in_channels, h), True),
            ("final_layer.linear.bias", (cfg.in_channels,), False),
            ("final_layer.adaLN_modulation.1.weight", (2 * h, h), True),
            ("final_layer.adaLN_modulation.1.bias", (2 * h,), False)]
    return out


def tensor_seed(seed, index):
    return (seed * 1000003 + index * 7919 + 17) & 0xFFFFFFFF


def pick_type(qtype, shape):
    """GGUF files keep tensors whose row length is not a multiple of the block as BF16."""
    k = shape[-1]
    if k % codec.block_elems(qtype) == 0:
        return qtype
    return codec.GGML_BF16


def synth_tensor(name, shape, is_matrix, seed, index, qtype):
    """Seeded synthetic tensor: matrices N(0, 0.02) quantized to `qtype`;
    biases N(0, 0.02) f32; RMSNorm scales 1 + 0.02 N(0,1) f32."""
    s = tensor_seed(seed, index)
    if is_matrix:
        x = codec.randn(s, shape, 0.02)
        t = pick_type(qtype, shape)
        return QTensorRef(t, shape, codec.quantize(x, t))
    if name.endswith(".scale"):
        x = 1.0 + codec.randn(s, shape, 0.02)
    else:
        x = codec.randn(s, shape, 0.02)
    return QTensorRef(codec.GGML_F32, shape, codec.quantize(x.astype(np.float32), codec.GGML_F32))


def synth_weights(cfg: FluxConfig, seed=0, qtype=codec.GGML_Q4_K, only=None):
    w = {}
    for i, (name, shape, is_matrix) in enumerate(weight_names(cfg)):
        if only is not None and not only(name):
            continue
        w[name] = synth_tensor(name, shape, is_matrix, seed, i, qtype)
    return w


# ---------------------------------------------------------------- ops
def silu(x):
    return x / (1.0 + np.exp(-x))


def gelu_tanh(x):
    x64 = x.astype(np.float64)
    return (0.5 * x64 * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x64 + 0.044715 * x64 ** 3)))).astype(np.float32)


def linear(x, w: QTensorRef, b: QTensorRef = None):
    y = np.asarray(x, dtype=np.float32) @ w.f32().T
    if b is not None:
        y = y + b.f32()
    return y.astype(np.float32)


def layer_norm(x, eps=1e-6):
    x64 = x.astype(np.float64)
    mu = x64.mean(-1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(-1, keepdims=True)
    return ((x64 - mu) / np.sqrt(var + eps)).astype(np.float32)


def rms_norm(x, scale, eps=1e-6):
    x64 = x.astype(np.float64)
    r = np.sqrt((x64 * x64).mean(-1, keepdims=True) + eps)
    return (x64 / r * scale.astype(np.float64)).astype(np.float32)


def modulate(x, shift, scale):
    return (layer_norm(x) * (1.0 + scale) + shift).astype(np.float32)


def timestep_embedding(t, dim=256):
    half = dim // 2
    freqs = np.exp(np.arange(half, dtype=np.float32) * np.float32(-math.log(10000.0) / half)).astype(np.float32)
    args = np.float32(t * 1000.0) * freqs
    return np.concatenate([np.cos(args), np.sin(args)]).astype(np.float32)


def rope(pos, dim, theta):
    """pos [L] -> [L, dim/2, 2, 2] = [[cos, -sin], [sin, cos]] (flux2/transformer.rs:99-118)."""
    inv = np.array([np.float32(1.0) / np.float32(float(theta) ** (i / dim)) for i in range(0, dim, 2)], dtype=np.float32)
    f = pos.astype(np.float32)[:, None] * inv[None, :]
    c, s = np.cos(f), np.sin(f)
    return np.stack([c, -s, s, c], axis=-1).reshape(pos.shape[0], dim // 2, 2, 2).astype(np.float32)


def embed_nd(ids, axes_dim, theta):
    """ids [L, n_axes] -> pe [L, sum(axes)/2, 2, 2]."""
    return np.concatenate([rope(ids[:, i], axes_dim[i], theta) for i in range(ids.shape[1])], axis=1)


def apply_rope(x, pe):
    """x [H, L, D]; pairs (2i, 2i+1): out0 = pe00*x0 + pe01*x1, out1 = pe10*x0 + pe11*x1."""
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    o0 = pe[None, :, :, 0, 0] * x0 + pe[None, :, :, 0, 1] * x1
    o1 = pe[None, :, :, 1, 0] * x0 + pe[None, :, :, 1, 1] * x1
    out = np.empty_like(x)
    out[..., 0::2] = o0
    out[..., 1::2] = o1
    return out


def sdpa(q, k, v, key_mask=None):
    """q,k,v [H, L, D] f32 -> [H, Lq, D]; optional key_mask [Lk] bool (True = keep)."""
    d = q.shape[-1]
    out = np.empty((q.shape[0], q.shape[1], v.shape[2]), dtype=np.float32)
    scale = np.float32(1.0 / math.sqrt(d))
    for h in range(q.shape[0]):
        s = (q[h] @ k[h].T) * scale
        if key_mask is not None:
            s = np.where(key_mask[None, :], s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[h] = p @ v[h]
    return out


def split_qkv(qkv, n_heads):
    """[L, 3*H*D] -> q, k, v each [H, L, D] (flux/offload.rs:193-197)."""
    L = qkv.shape[0]
    r = qkv.reshape(L, 3, n_heads, -1)
    return (np.ascontiguousarray(r[:, 0].transpose(1, 0, 2)), np.ascontiguousarray(r[:, 1].transpose(1, 0, 2)),
            np.ascontiguousarray(r[:, 2].transpose(1, 0, 2)))


def attention(q, k, v, pe):
    """flux/offload.rs:67-72: rope(q), rope(k), sdpa, (H,L,D)->(L,H*D)."""
    x = sdpa(apply_rope(q, pe), apply_rope(k, pe), v)
    return np.ascontiguousarray(x.transpose(1, 0, 2)).reshape(q.shape[1], -1)


def modulation(vec, w, b, n):
    ys = linear(silu(vec)[None, :], w, b)[0]
    return np.split(ys, n)


def double_block(W, p, cfg, img, txt, vec, pe):
    H = cfg.num_heads
    i_s1, i_c1, i_g1, i_s2, i_c2, i_g2 = modulation(vec, W[p + "img_mod.lin.weight"], W[p + "img_mod.lin.bias"], 6)
    t_s1, t_c1, t_g1, t_s2, t_c2, t_g2 = modulation(vec, W[p + "txt_mod.lin.weight"], W[p + "txt_mod.lin.bias"], 6)

    def qkv(x, s):
        q, k, v = split_qkv(linear(x, W[p + f"{s}_attn.qkv.weight"], W.get(p + f"{s}_attn.qkv.bias")), H)
        q = rms_norm(q, W[p + f"{s}_attn.norm.query_norm.scale"].f32())
        k = rms_norm(k, W[p + f"{s}_attn.norm.key_norm.scale"].f32())
        return q, k, v

    iq, ik, iv = qkv(modulate(img, i_s1, i_c1), "img")
    tq, tk, tv = qkv(modulate(txt, t_s1, t_c1), "txt")
    q = np.concatenate([tq, iq], axis=1)
    k = np.concatenate([tk, ik], axis=1)
    v = np.concatenate([tv, iv], axis=1)
    attn = attention(q, k, v, pe)
    lt = txt.shape[0]
    t_attn, i_attn = attn[:lt], attn[lt:]

    def mlp(x, s):
        h = gelu_tanh(linear(x, W[p + f"{s}_mlp.0.weight"], W[p + f"{s}_mlp.0.bias"]))
        return linear(h, W[p + f"{s}_mlp.2.weight"], W[p + f"{s}_mlp.2.bias"])

    img = img + i_g1 * linear(i_attn, W[p + "img_attn.proj.weight"], W[p + "img_attn.proj.bias"])
    img = img + i_g2 * mlp(modulate(img, i_s2, i_c2), "img")
    txt = txt + t_g1 * linear(t_attn, W[p + "txt_attn.proj.weight"], W[p + "txt_attn.proj.bias"])
    txt = txt + t_g2 * mlp(modulate(txt, t_s2, t_c2), "txt")
    return img.astype(np.float32), txt.astype(np.float32)


def single_block(W, p, cfg, x, vec, pe):
    h, H = cfg.hidden_size, cfg.num_heads
    shift, scale, gate = modulation(vec, W[p + "modulation.lin.weight"], W[p + "modulation.lin.bias"], 3)
    xm = linear(modulate(x, shift, scale), W[p + "linear1.weight"], W[p + "linear1.bias"])
    q, k, v = split_qkv(xm[:, :3 * h], H)
    mlp = xm[:, 3 * h:]
    q = rms_norm(q, W[p + "norm.query_norm.scale"].f32())
    k = rms_norm(k, W[p + "norm.key_norm.scale"].f32())
    attn = attention(q, k, v, pe)
    out = linear(np.concatenate([attn, gelu_tanh(mlp)], axis=1), W[p + "linear2.weight"], W[p + "linear2.bias"])
    return (x + gate * out).astype(np.float32)


def final_layer(W, x, vec):
    shift, scale = np.split(linear(silu(vec)[None, :], W["final_layer.adaLN_modulation.1.weight"],
                                   W["final_layer.adaLN_modulation.1.bias"])[0], 2)
    return linear(modulate(x, shift, scale), W["final_layer.linear.weight"], W["final_layer.linear.bias"])


def mlp_embedder(W, stem, x):
    h = silu(linear(x[None, :], W[stem + ".in_layer.weight"], W[stem + ".in_layer.bias"]))
    return linear(h, W[stem + ".out_layer.weight"], W[stem + ".out_layer.bias"])[0]


def vec_embedding(W, cfg, t, y, guidance):
    vec = mlp_embedder(W, "time_in", timestep_embedding(t))
    if cfg.guidance_embed and guidance is not None:
        vec = vec + mlp_embedder(W, "guidance_in", timestep_embedding(guidance))
    return (vec + mlp_embedder(W, "vector_in", y)).astype(np.float32)


def forward(W, cfg, img, img_ids, txt, txt_ids, t, y, guidance):
    """Batch-1 FLUX forward: img [Li, C], ids [L, 3], txt [Lt, ctx], y [vec_in]."""
    pe = embed_nd(np.concatenate([txt_ids, img_ids], axis=0), cfg.axes_dim, cfg.theta)
    txt = linear(txt, W["txt_in.weight"], W["txt_in.bias"])
    img = linear(img, W["img_in.weight"], W["img_in.bias"])
    vec = vec_embedding(W, cfg, t, y, guidance)
    for i in range(cfg.depth):
        img, txt = double_block(W, f"double_blocks.{i}.", cfg, img, txt, vec, pe)
    x = np.concatenate([txt, img], axis=0)
    for i in range(cfg.depth_single_blocks):
        x = single_block(W, f"single_blocks.{i}.", cfg, x, vec, pe)
    return final_layer(W, x[txt.shape[0]:], vec)


def get_schedule(num_steps, image_seq_len=None, base_shift=0.5, max_shift=1.15):
    ts = [v / num_steps for v in range(num_steps + 1)][::-1]
    if image_seq_len is None:
        return ts
    m = (max_shift - base_shift) / (4096.0 - 256.0)
    b = base_shift - m * 256.0
    mu = m * image_seq_len + b

    def shift(t):
        if t <= 0.0:
            return 0.0
        e = math.exp(mu)
        return e / (e + (1.0 / t - 1.0))
    return [shift(t) for t in ts]


def inpaint_blend(img, inpaint, t):
    """flux/transformer.rs:79-87 and img2img.rs:36-42,79-98: the original re-noised to t,
    orig * (1 - t) + noise * t (f64 scalars rounded to f32), restored where mask = 0:
    img * mask + preserved * (1 - mask); every operand in the same (packed) layout."""
    mask, orig, noise = (np.asarray(a, np.float32) for a in inpaint)
    keep = (orig * np.float32(1.0 - t)).astype(np.float32) + (noise * np.float32(t)).astype(np.float32)
    return ((img * mask).astype(np.float32) + (keep * (np.float32(1.0) - mask)).astype(np.float32)).astype(np.float32)


def denoise(W, cfg, img, img_ids, txt, txt_ids, y, timesteps, guidance, inpaint=None):
    """flux/transformer.rs:50-95: img += pred * (t_prev - t_curr), then the inpaint blend at
    t_prev when inpaint = (mask, original, noise) is given."""
    img = img.astype(np.float32).copy()
    for t_curr, t_prev in zip(timesteps[:-1], timesteps[1:]):
        pred = forward(W, cfg, img, img_ids, txt, txt_ids, t_curr, y, guidance)
        img = (img + pred * np.float32(t_prev - t_curr)).astype(np.float32)
        if inpaint is not None:
            img = inpaint_blend(img, inpaint, t_prev)
    return img


def img_ids(h_tokens, w_tokens):
    """State::new ids for FLUX.1: (0, row, col) per 2x2 patch (flux2/sampling.rs:52-72, 3 axes)."""
    r = np.repeat(np.arange(h_tokens, dtype=np.float32), w_tokens)
    c = np.tile(np.arange(w_tokens, dtype=np.float32), h_tokens)
    return np.stack([np.zeros_like(r), r, c], axis=1).astype(np.float32)


def patchify(latent):
    """[C, H, W] -> [(H/2)(W/2), C*4] (flux2/sampling.rs:45-48)."""
    c, h, w = latent.shape
    return latent.reshape(c, h // 2, 2, w // 2, 2).transpose(1, 3, 0, 2, 4).reshape(h // 2 * w // 2, c * 4)


def unpack(x, h, w):
    """[(h/2)(w/2), C*4] -> [C, h, w] (flux2/sampling.rs:149-159, latent dims)."""
    c4 = x.shape[1]
    return x.reshape(h // 2, w // 2, c4 // 4, 2, 2).transpose(2, 0, 3, 1, 4).reshape(c4 // 4, h, w)
