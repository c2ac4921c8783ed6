"""FluxTransformer — the FLUX.1 GGUF transformer behind the C ABI.

Mirrors the reference's `FluxTransformer` enum arm (crates/mold-inference/src/flux/transformer.rs:17-98):
`forward(img, img_ids, txt, txt_ids, timesteps, y, guidance)` is candle's
`WithForward::forward` for the quantized model, and `denoise(...)` is the Euler
loop of `FluxTransformer::denoise`. Weights are handed over by GGUF tensor name
(as `quantized_var_builder::VarBuilder::from_gguf` reads them, flux/pipeline.rs:976).
"""
import ctypes
from dataclasses import dataclass

import torch

from ._lib import FluxConfigC, check, lib
from .ops import QTensor, _lora_operands, _ptr, _stream, denoise_extras, init


@dataclass
class FluxConfig:
    """candle flux::model::Config (FLUX.1-dev values by default)."""
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
    def mlp_hidden(self):
        return int(self.hidden_size * self.mlp_ratio)

    def to_c(self):
        c = FluxConfigC()
        c.in_channels, c.vec_in_dim, c.context_in_dim = self.in_channels, self.vec_in_dim, self.context_in_dim
        c.hidden_size, c.mlp_hidden, c.num_heads = self.hidden_size, self.mlp_hidden, self.num_heads
        c.depth, c.depth_single = self.depth, self.depth_single_blocks
        c.axes_dim[0], c.axes_dim[1], c.axes_dim[2] = self.axes_dim
        c.theta, c.guidance_embed = self.theta, int(self.guidance_embed)
        return c


def tensor_specs(cfg: FluxConfig):
    """(GGUF name, shape) of every tensor the model reads (flux/pipeline.rs:255-276 naming;
    matrices are [out, in])."""
    h, m, hd = cfg.hidden_size, cfg.mlp_hidden, cfg.hidden_size // cfg.num_heads
    out = []

    def lin(n, o, i):
        out.append((n + ".weight", (o, i)))
        out.append((n + ".bias", (o,)))
    lin("img_in", h, cfg.in_channels)
    lin("txt_in", h, cfg.context_in_dim)
    lin("time_in.in_layer", h, 256)
    lin("time_in.out_layer", h, h)
    lin("vector_in.in_layer", h, cfg.vec_in_dim)
    lin("vector_in.out_layer", h, h)
    if cfg.guidance_embed:
        lin("guidance_in.in_layer", h, 256)
        lin("guidance_in.out_layer", h, h)
    for i in range(cfg.depth):
        p = f"double_blocks.{i}."
        for s in ("img", "txt"):
            lin(p + f"{s}_mod.lin", 6 * h, h)
            lin(p + f"{s}_attn.qkv", 3 * h, h)
            out.append((p + f"{s}_attn.norm.query_norm.scale", (hd,)))
            out.append((p + f"{s}_attn.norm.key_norm.scale", (hd,)))
            lin(p + f"{s}_attn.proj", h, h)
            lin(p + f"{s}_mlp.0", m, h)
            lin(p + f"{s}_mlp.2", h, m)
    for i in range(cfg.depth_single_blocks):
        p = f"single_blocks.{i}."
        lin(p + "linear1", 3 * h + m, h)
        lin(p + "linear2", h, h + m)
        out.append((p + "norm.query_norm.scale", (hd,)))
        out.append((p + "norm.key_norm.scale", (hd,)))
        lin(p + "modulation.lin", 3 * h, h)
    lin("final_layer.linear", cfg.in_channels, h)
    lin("final_layer.adaLN_modulation.1", 2 * h, h)
    return out


def step_flops(cfg: FluxConfig, l_txt, l_img):
    """Algorithmic FLOPs of one transformer forward (2 per MAC): linears + attention."""
    h, m, H = cfg.hidden_size, cfg.mlp_hidden, cfg.num_heads
    L = l_txt + l_img
    dbl = 2 * L * h * (3 * h + h + m + m) + 4 * L * L * h
    sgl = 2 * L * h * (3 * h + m) + 2 * L * (h + m) * h + 4 * L * L * h
    stems = 2 * l_txt * cfg.context_in_dim * h + 2 * l_img * cfg.in_channels * h + 2 * l_img * h * cfg.in_channels
    return cfg.depth * dbl + cfg.depth_single_blocks * sgl + stems


class FluxTransformer:
    def __init__(self, cfg: FluxConfig, max_txt=512, max_img=4096, device=0):
        init(device)
        self.cfg, self.device = cfg, device
        self._cc = cfg.to_c()
        h = ctypes.c_void_p()
        check(lib().mb_flux_create(ctypes.byref(self._cc), max_txt, max_img, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().mb_flux_destroy(h)
            except Exception:
                pass
            self._h = None

    def set_tensor(self, name, qt):
        """qt: QTensor (host bytes) or a CUDA uint8 tensor with (ggml_type, shape) attributes."""
        if isinstance(qt, QTensor):
            n_rows = qt.n_rows if len(qt.shape) > 1 else 1
            check(lib().mb_flux_set_tensor(self._h, name.encode(), qt.ggml_type, n_rows, qt.n_cols,
                                           qt.raw.ctypes.data_as(ctypes.c_void_p), qt.raw.size, 0))
        else:
            raw, ggml_type, shape = qt
            n_rows = shape[0] if len(shape) > 1 else 1
            check(lib().mb_flux_set_tensor(self._h, name.encode(), ggml_type, n_rows, shape[-1], _ptr(raw),
                                           raw.numel(), 1))

    def load(self, tensors):
        for name, qt in tensors.items():
            self.set_tensor(name, qt)
        return self

    def load_gguf(self, path, embeddings_path=None):
        """Load a FLUX GGUF file (VarBuilder::from_gguf, flux/pipeline.rs:976); embeddings_path
        supplies img_in / time_in / vector_in / guidance_in when the file lacks them (city96)."""
        n = ctypes.c_int(0)
        check(lib().mb_flux_load_gguf(self._h, str(path).encode(),
                                      None if embeddings_path is None else str(embeddings_path).encode(),
                                      ctypes.byref(n)))
        return n.value

    def lora_merge(self, name, A, B, scale, row_offset=0):
        """Merge scale * (B @ A) into rows [row_offset, row_offset + B.shape[0]) of tensor `name`
        in its own GGML type (mb_flux_lora_merge). A [rank, in], B [rows, rank] (CUDA)."""
        A, B = _lora_operands(A, B)
        check(lib().mb_flux_lora_merge(self._h, name.encode(), int(row_offset), B.shape[0], _ptr(A), _ptr(B),
                                       A.shape[0], float(scale), _stream()))

    def missing(self):
        buf = ctypes.create_string_buffer(1 << 16)
        check(lib().mb_flux_missing(self._h, buf, len(buf)))
        return [s for s in buf.value.decode().split("\n") if s]

    def forward(self, img, img_ids, txt, txt_ids, t, y, guidance):
        """img [L_img, C], ids [L, 3], txt [L_txt, ctx], y [vec_in] (f32 CUDA) -> pred [L_img, C]."""
        img, img_ids, txt, txt_ids, y = (a.contiguous().float() for a in (img, img_ids, txt, txt_ids, y))
        pred = torch.empty_like(img)
        check(lib().mb_flux_forward(self._h, _ptr(img), _ptr(img_ids), img.shape[0], _ptr(txt), _ptr(txt_ids),
                                    txt.shape[0], float(t), _ptr(y), float(guidance), _ptr(pred), _stream()))
        return pred

    def denoise(self, img, img_ids, txt, txt_ids, y, timesteps, guidance, inpaint=None, on_step=None):
        """In-place Euler loop over `timesteps` (list of floats); returns img. inpaint =
        (mask, original, noise) packed like img blends the preserved region back after every
        step; on_step(step, total) reports progress (FluxTransformer::denoise's inpaint_ctx and
        DenoiseStep events, flux/transformer.rs:79-93)."""
        assert img.dtype == torch.float32 and img.is_contiguous()
        ts = (ctypes.c_double * len(timesteps))(*[float(t) for t in timesteps])
        txt, txt_ids, img_ids, y = (a.contiguous().float() for a in (txt, txt_ids, img_ids, y))
        if inpaint is None and on_step is None:
            self._keep = (txt, txt_ids, img_ids, y)
            check(lib().mb_flux_denoise(self._h, _ptr(img), _ptr(img_ids), img.shape[0], _ptr(txt), _ptr(txt_ids),
                                        txt.shape[0], _ptr(y), ts, len(timesteps), float(guidance), _stream()))
            return img
        ip, cb, keep = denoise_extras(inpaint, on_step)
        self._keep = (txt, txt_ids, img_ids, y, keep)
        check(lib().mb_flux_denoise_ex(self._h, _ptr(img), _ptr(img_ids), img.shape[0], _ptr(txt), _ptr(txt_ids),
                                       txt.shape[0], _ptr(y), ts, len(timesteps), float(guidance), ip, cb, None,
                                       _stream()))
        return img
