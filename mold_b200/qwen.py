"""QwenImageTransformer — the Qwen-Image GGUF transformer behind the C ABI.

Mirrors `QuantizedQwenImageTransformer2DModel` (crates/mold-inference/src/qwen_image/
quantized_transformer.rs:991-1139): `forward(x, t, encoder_hidden_states, encoder_attention_mask)`
on packed latents, and `denoise(...)`, the step loop of qwen_image/pipeline.rs:2655-2716 with
its CFG + norm rescale (batch 2 = conditional then unconditional prompt). Weights are handed
over by GGUF tensor name, as `qlinear` / `dequant_rms_norm` read them (:79-121, :577-1040).
"""
import ctypes
from dataclasses import dataclass

import torch

from ._lib import QwenConfigC, check, lib
from .ops import QTensor, _ptr, _stream, denoise_extras, init


@dataclass
class QwenConfig:
    """QwenImageConfig (qwen_image/transformer.rs:204-230; Qwen-Image values by default)."""
    in_channels: int = 64
    out_channels: int = 16
    patch_size: int = 2
    joint_attention_dim: int = 3584
    hidden_size: int = 3072
    num_heads: int = 24
    num_layers: int = 60
    mlp_hidden: int = 12288
    axes_dim: tuple = (16, 56, 56)
    theta: int = 10000

    def to_c(self):
        c = QwenConfigC()
        c.in_channels, c.out_channels, c.patch_size = self.in_channels, self.out_channels, self.patch_size
        c.joint_attention_dim, c.hidden_size, c.num_heads = self.joint_attention_dim, self.hidden_size, self.num_heads
        c.num_layers, c.mlp_hidden = self.num_layers, self.mlp_hidden
        c.axes_dim[0], c.axes_dim[1], c.axes_dim[2] = self.axes_dim
        c.theta = self.theta
        return c


ATTN_LINEARS = ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out")
NORMS = ("norm_q", "norm_k", "norm_added_q", "norm_added_k")


def tensor_specs(cfg: QwenConfig):
    """(GGUF name, shape) of every tensor the model reads; matrices are [out, in]."""
    h, m, hd = cfg.hidden_size, cfg.mlp_hidden, cfg.hidden_size // cfg.num_heads
    out = []

    def lin(n, o, i):
        out.append((n + ".weight", (o, i)))
        out.append((n + ".bias", (o,)))
    lin("time_text_embed.timestep_embedder.linear_1", h, 256)
    lin("time_text_embed.timestep_embedder.linear_2", h, h)
    lin("img_in", h, cfg.in_channels)
    lin("txt_in", h, cfg.joint_attention_dim)
    out.append(("txt_norm.weight", (cfg.joint_attention_dim,)))
    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        for n in ATTN_LINEARS:
            lin(p + "attn." + n, h, h)
        for n in NORMS:
            out.append((p + "attn." + n + ".weight", (hd,)))
        for s in ("img", "txt"):
            lin(p + f"{s}_mlp.net.0.proj", m, h)
            lin(p + f"{s}_mlp.net.2", h, m)
            lin(p + f"{s}_mod.1", 6 * h, h)
    lin("norm_out.linear", 2 * h, h)
    lin("proj_out", cfg.patch_size * cfg.patch_size * cfg.out_channels, h)
    return out


def step_flops(cfg: QwenConfig, l_txt, l_img, batch=1):
    """Algorithmic FLOPs of one forward over `batch` sequences (2 per MAC): linears + attention."""
    h, m = cfg.hidden_size, cfg.mlp_hidden
    L = l_txt + l_img
    blk = 2 * L * h * (3 * h + h) + 2 * L * 2 * h * m + 4 * L * L * h
    stems = 2 * l_txt * cfg.joint_attention_dim * h + 2 * l_img * cfg.in_channels * h + 2 * l_img * h * cfg.in_channels
    return batch * (cfg.num_layers * blk + stems)


class QwenTransformer:
    def __init__(self, cfg: QwenConfig, max_txt=256, max_img=4096, max_batch=2, device=0):
        init(device)
        self.cfg, self.device = cfg, device
        self._cc = cfg.to_c()
        h = ctypes.c_void_p()
        check(lib().mb_qwen_create(ctypes.byref(self._cc), max_txt, max_img, max_batch, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().mb_qwen_destroy(h)
            except Exception:
                pass
            self._h = None

    def set_tensor(self, name, qt):
        """qt: QTensor (host bytes) or (CUDA uint8 tensor, ggml_type, shape)."""
        if isinstance(qt, QTensor):
            n_rows = qt.n_rows if len(qt.shape) > 1 else 1
            check(lib().mb_qwen_set_tensor(self._h, name.encode(), qt.ggml_type, n_rows, qt.n_cols,
                                           qt.raw.ctypes.data_as(ctypes.c_void_p), qt.raw.size, 0))
        else:
            raw, ggml_type, shape = qt
            n_rows = shape[0] if len(shape) > 1 else 1
            check(lib().mb_qwen_set_tensor(self._h, name.encode(), ggml_type, n_rows, shape[-1], _ptr(raw),
                                           raw.numel(), 1))

    def load(self, tensors):
        for name, qt in tensors.items():
            self.set_tensor(name, qt)
        return self

    def load_gguf(self, path):
        """Load a Qwen-Image GGUF file (qwen_image/pipeline.rs:258-275)."""
        n = ctypes.c_int(0)
        check(lib().mb_qwen_load_gguf(self._h, str(path).encode(), ctypes.byref(n)))
        return n.value

    def missing(self):
        buf = ctypes.create_string_buffer(1 << 16)
        check(lib().mb_qwen_missing(self._h, buf, len(buf)))
        return [s for s in buf.value.decode().split("\n") if s]

    @staticmethod
    def _mask(txt_mask, txt):
        if txt_mask is None:
            return None
        return txt_mask.to(device=txt.device, dtype=torch.uint8).contiguous()

    def forward(self, img, t, txt, txt_mask, h_tokens, w_tokens):
        """img [B, L_img, 64] packed latents, txt [B, L_txt, 3584], txt_mask [B, L_txt] (1 = keep),
        t = sigma * 1000 -> pred [B, L_img, 64] (f32, CUDA)."""
        img = img.contiguous().float()
        txt = txt.contiguous().float()
        if img.dim() == 2:
            img = img[None]
        if txt.dim() == 2:
            txt = txt[None]
        B = txt.shape[0]
        mask = self._mask(txt_mask, txt)
        pred = torch.empty_like(img)
        check(lib().mb_qwen_forward(self._h, _ptr(img), h_tokens, w_tokens, _ptr(txt), _ptr(mask), txt.shape[1], B,
                                    float(t), _ptr(pred), _stream()))
        return pred

    def denoise(self, img, txt, txt_mask, h_tokens, w_tokens, sigmas, guidance=1.0, inpaint=None, on_step=None):
        """In place on packed latents img [L_img, 64] f32: the Qwen step loop over `sigmas`
        (with batch-2 txt / txt_mask: CFG with norm rescale at `guidance`). Returns img.
        inpaint = (mask, original, noise) and on_step(step, total) as for FluxTransformer.denoise
        (qwen_image/pipeline.rs:2708-2724)."""
        assert img.dtype == torch.float32 and img.is_contiguous()
        txt = txt.contiguous().float()
        if txt.dim() == 2:
            txt = txt[None]
        mask = self._mask(txt_mask, txt)
        sg = (ctypes.c_double * len(sigmas))(*[float(s) for s in sigmas])
        if inpaint is None and on_step is None:
            self._keep = (txt, mask)
            check(lib().mb_qwen_denoise(self._h, _ptr(img), h_tokens, w_tokens, _ptr(txt), _ptr(mask), txt.shape[1],
                                        txt.shape[0], sg, len(sigmas), float(guidance), _stream()))
            return img
        ip, cb, keep = denoise_extras(inpaint, on_step)
        self._keep = (txt, mask, keep)
        check(lib().mb_qwen_denoise_ex(self._h, _ptr(img), h_tokens, w_tokens, _ptr(txt), _ptr(mask), txt.shape[1],
                                       txt.shape[0], sg, len(sigmas), float(guidance), ip, cb, None, _stream()))
        return img
