"""Torch-tensor front of the single-kernel C-ABI entry points.

Each function takes CUDA tensors, checks dtypes/contiguity, and passes raw
pointers plus the current torch stream to libmold_b200.so.
"""
import ctypes

import numpy as np
import torch

from ._lib import (STEP_CALLBACK, InpaintC, DT_BF16, DT_F32, EPI_GATE_RESIDUAL, EPI_GELU_TANH, EPI_NONE, GGML_BF16, GGML_F16, GGML_F32,
                   GGML_Q4_0, GGML_Q4_1, GGML_Q4_K, GGML_Q5_0, GGML_Q5_1, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, check, lib)

# (values, bytes) per GGUF block
_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144),
          GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20), GGML_Q5_0: (32, 22), GGML_Q5_1: (32, 24), GGML_Q5_K: (256, 176),
          GGML_Q6_K: (256, 210)}
_inited = set()


def init(device=0):
    """mb_init for `device` (idempotent); also makes it torch's current device."""
    torch.cuda.set_device(device)
    if device not in _inited:
        check(lib().mb_init(device))
        _inited.add(device)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _dt(t):
    if t.dtype == torch.float32:
        return DT_F32
    if t.dtype == torch.bfloat16:
        return DT_BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def row_bytes(ggml_type, n_cols):
    be, bb = _BLOCK[ggml_type]
    if n_cols % be:
        raise ValueError(f"n_cols {n_cols} not a multiple of block {be}")
    return n_cols // be * bb


class QTensor:
    """A GGUF tensor held as raw GGML bytes: rows = output features, blocks along cols
    (candle's QTensor)."""

    def __init__(self, ggml_type, shape, raw):
        self.ggml_type = int(ggml_type)
        self.shape = tuple(int(s) for s in shape)
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        n_rows = int(np.prod(self.shape[:-1])) if len(self.shape) > 1 else 1
        if raw.size != n_rows * row_bytes(self.ggml_type, self.shape[-1]):
            raise ValueError("raw byte count does not match shape/type")
        self.raw = raw

    @property
    def n_rows(self):
        return int(np.prod(self.shape[:-1])) if len(self.shape) > 1 else 1

    @property
    def n_cols(self):
        return self.shape[-1]


class QMatMul:
    """Device copy of a quantized weight; forward(x) = x W^T (candle QMatMul)."""

    def __init__(self, handle, n_rows, n_cols, ggml_type, device):
        self._h = handle
        self.n_rows, self.n_cols, self.ggml_type, self.device = n_rows, n_cols, ggml_type, device

    @classmethod
    def from_weights(cls, qt: QTensor, device=0):
        init(device)
        h = ctypes.c_void_p()
        check(lib().mb_weight_create(qt.ggml_type, qt.n_rows, qt.n_cols, qt.raw.ctypes.data_as(ctypes.c_void_p),
                                     qt.raw.size, 0, ctypes.byref(h)))
        return cls(h, qt.n_rows, qt.n_cols, qt.ggml_type, device)

    @classmethod
    def from_device_bytes(cls, raw, ggml_type, n_rows, n_cols, device=0):
        """A weight from GGUF bytes already in device memory (a uint8 CUDA tensor, GGUF layout);
        the library takes its own copy."""
        init(device)
        h = ctypes.c_void_p()
        check(lib().mb_weight_create(int(ggml_type), n_rows, n_cols, ctypes.c_void_p(raw.data_ptr()), raw.numel(), 1,
                                     ctypes.byref(h)))
        return cls(h, n_rows, n_cols, int(ggml_type), device)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and lib is not None:
            try:
                lib().mb_weight_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def forward(self, x, bias=None, epilogue=EPI_NONE, gelu_from=0, gate=None, residual=None, out=None,
                out_dtype=None):
        """x [..., K] (bf16 or f32, CUDA) -> [..., N]. Epilogues as mb_qlinear."""
        return qlinear(self, x, bias=bias, epilogue=epilogue, gelu_from=gelu_from, gate=gate, residual=residual,
                       out=out, out_dtype=out_dtype)

    __call__ = forward

    def download(self):
        """The weight's bytes in GGUF layout (host uint8 [n_rows * row bytes])."""
        out = np.empty(self.n_rows * row_bytes(self.ggml_type, self.n_cols), dtype=np.uint8)
        check(lib().mb_weight_download(self._h, out.ctypes.data_as(ctypes.c_void_p), out.size))
        return out

    def lora_merge(self, A, B, scale, row_offset=0):
        """In place: rows [row_offset, row_offset + B.shape[0]) += scale * (B @ A), re-quantized to
        the weight's own type (mb_weight_lora_merge). A [rank, n_cols], B [rows, rank] (CUDA)."""
        A, B = _lora_operands(A, B)
        check(lib().mb_weight_lora_merge(self._h, int(row_offset), B.shape[0], _ptr(A), _ptr(B), A.shape[0],
                                         float(scale), _stream()))


def _lora_operands(A, B):
    A = A.contiguous().float()
    B = B.contiguous().float()
    if A.dim() != 2 or B.dim() != 2 or B.shape[1] != A.shape[0]:
        raise ValueError(f"LoRA shapes A {tuple(A.shape)} and B {tuple(B.shape)} do not chain")
    if not (A.is_cuda and B.is_cuda):
        raise ValueError("LoRA A and B must be CUDA tensors")
    return A, B


def qlinear(w: QMatMul, x, bias=None, epilogue=EPI_NONE, gelu_from=0, gate=None, residual=None, out=None,
            out_dtype=None):
    K, N = w.n_cols, w.n_rows
    if x.shape[-1] != K:
        raise ValueError(f"x has K={x.shape[-1]}, weight expects {K}")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if epilogue == EPI_GATE_RESIDUAL:
        out_dtype = torch.float32
    if out is None:
        out_dtype = out_dtype or x.dtype
        out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    y2 = out.reshape(-1, out.shape[-1])
    res = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
    check(lib().mb_qlinear(w.handle, _ptr(x2), _dt(x2), M, x2.stride(0), _ptr(y2), _dt(y2), y2.stride(0),
                           _ptr(bias), epilogue, gelu_from, _ptr(gate), _ptr(res), res.stride(0) if res is not None else 0,
                           _stream()))
    return out.reshape(*x.shape[:-1], N) if out.dim() == 2 and x.dim() != 2 else out


def dequantize(w: QMatMul, dtype=torch.float32):
    out = torch.empty((w.n_rows, w.n_cols), dtype=dtype, device=f"cuda:{w.device}")
    check(lib().mb_dequant(w.handle, _ptr(out), _dt(out), _stream()))
    return out


def qgemv(w: QMatMul, x, apply_silu=False, bias=None):
    y = torch.empty(w.n_rows, dtype=torch.float32, device=x.device)
    check(lib().mb_qgemv(w.handle, _ptr(x.contiguous()), int(apply_silu), _ptr(bias), _ptr(y), _stream()))
    return y


def ln_modulate(x, shift, scale):
    M, C = x.shape
    y = torch.empty((M, C), dtype=torch.bfloat16, device=x.device)
    check(lib().mb_ln_modulate(_ptr(x), M, C, x.stride(0), _ptr(shift), _ptr(scale), _ptr(y), y.stride(0), _stream()))
    return y


def rope_table(ids, axes_dim=(16, 56, 56), theta=10000):
    L, n_axes = ids.shape
    pe = torch.empty((L, sum(axes_dim) // 2, 2, 2), dtype=torch.float32, device=ids.device)
    ax = (ctypes.c_int * len(axes_dim))(*axes_dim)
    check(lib().mb_rope_table(_ptr(ids.contiguous()), L, n_axes, ax, theta, _ptr(pe), _stream()))
    return pe


def qk_norm_rope(qkv, H, q_scale, k_scale, pe, row_offset=0, L_total=None, q=None, k=None, v=None, kv_pos=None):
    """kv_pos (int32 [L_total], optional): k / v of sequence row r go to row kv_pos[r]."""
    M = qkv.shape[0]
    L_total = L_total or M
    if q is None:
        q = torch.empty((H, L_total, 128), dtype=torch.bfloat16, device=qkv.device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
    if kv_pos is None:
        check(lib().mb_qk_norm_rope(_ptr(qkv), M, qkv.stride(0), H, _ptr(q_scale), _ptr(k_scale), _ptr(pe),
                                    row_offset, L_total, _ptr(q), _ptr(k), _ptr(v), _stream()))
    else:
        assert kv_pos.dtype == torch.int32 and kv_pos.numel() >= L_total
        check(lib().mb_qk_norm_rope_ex(_ptr(qkv), M, qkv.stride(0), H, _ptr(q_scale), _ptr(k_scale), _ptr(pe),
                                       row_offset, L_total, _ptr(q), _ptr(k), _ptr(v), _ptr(kv_pos), _stream()))
    return q, k, v


def key_order(txt_mask, l_img):
    """Key order for a masked joint sequence cat[txt, img]: kept text keys, image keys, masked
    text keys. Returns (kv_pos int32 [L], n_valid_keys) for qk_norm_rope / attention."""
    m = torch.as_tensor(txt_mask).to("cpu", torch.bool).reshape(-1)
    lt = m.numel()
    nv = int(m.sum())
    pos = torch.empty(lt + l_img, dtype=torch.int32)
    pos[:lt][m] = torch.arange(nv, dtype=torch.int32)
    pos[:lt][~m] = torch.arange(lt - nv, dtype=torch.int32) + nv + l_img
    pos[lt:] = torch.arange(l_img, dtype=torch.int32) + nv
    return pos, nv + l_img


def attention(q, k, v, n_valid_keys=None, out=None, split_row=None, out2=None):
    """q [H, Lq, 128], k/v [H, Lk, 128] bf16 -> out [Lq, H*128] bf16. With split_row, rows
    [split_row, Lq) go to out2 (same row stride) instead."""
    H, Lq, D = q.shape
    Lk = k.shape[1]
    if out is None:
        out = torch.empty((Lq if split_row is None else split_row, H * D), dtype=torch.bfloat16, device=q.device)
    if split_row is None:
        check(lib().mb_attention(_ptr(q), _ptr(k), _ptr(v), H, Lq, Lk, n_valid_keys or Lk, _ptr(out),
                                 out.stride(0), _stream()))
        return out
    if out2 is None:
        out2 = torch.empty((Lq - split_row, H * D), dtype=torch.bfloat16, device=q.device)
    assert out2.stride(0) == out.stride(0)
    check(lib().mb_attention_ex(_ptr(q), _ptr(k), _ptr(v), H, Lq, Lk, n_valid_keys or Lk, _ptr(out), out.stride(0),
                                split_row, _ptr(out2), _stream()))
    return out, out2


def rms_norm(x, w, eps=1e-6):
    """DynamicRmsNorm: x f32 [M, C] -> bf16 x / sqrt(mean(x^2) + eps) * w."""
    M, C = x.shape
    y = torch.empty((M, C), dtype=torch.bfloat16, device=x.device)
    check(lib().mb_rms_norm(_ptr(x), M, C, x.stride(0), _ptr(w), float(eps), _ptr(y), y.stride(0), _stream()))
    return y


def cfg_euler_step(img, cond, uncond, guidance, dt, channels=16, pp=4):
    """img += CFG(cond, uncond) * dt on packed latents [n_tok, channels * pp] (f32, in place)."""
    n_tok = img.shape[0]
    check(lib().mb_cfg_euler_step(_ptr(img), _ptr(cond), _ptr(uncond), n_tok, channels, pp, float(guidance),
                                  float(dt), _stream()))
    return img


def euler_step(img, pred, dt):
    check(lib().mb_euler_step(_ptr(img), _ptr(pred), img.numel(), float(dt), _stream()))
    return img


def device_status():
    s = ctypes.c_int(0)
    check(lib().mb_device_status(ctypes.byref(s)))
    return s.value


def gguf_inspect(path):
    """[(name, ggml_type, shape outermost-first)] of a GGUF file's tensors (no GPU needed)."""
    buf = ctypes.create_string_buffer(1 << 22)
    n = ctypes.c_int64(0)
    check(lib().mb_gguf_inspect(str(path).encode(), buf, len(buf), ctypes.byref(n)))
    out = []
    for line in buf.value.decode().split("\n"):
        if line:
            f = line.split("\t")
            out.append((f[0], int(f[1]), tuple(int(x) for x in f[2:])))
    return out


def denoise_extras(inpaint, on_step):
    """ctypes arguments of the *_denoise_ex calls: (pointer to an mb_inpaint or None, callback,
    objects to keep alive while the steps run). inpaint = (mask, original, noise), f32 CUDA
    tensors shaped like the packed latent (1 = repaint, 0 = preserve); on_step(step, total) is
    called from a CUDA host-function thread once each step has finished on the device (keep it
    short, and synchronise the stream before relying on every call having happened)."""
    keep = []
    ip = None
    if inpaint is not None:
        ts = [a.contiguous().float() for a in inpaint]
        keep += ts
        ip = InpaintC(*[ctypes.c_void_p(a.data_ptr()) for a in ts])
        keep.append(ip)
    cb = STEP_CALLBACK(lambda user, step, total: on_step(step, total)) if on_step is not None else STEP_CALLBACK()
    keep.append(cb)
    return (ctypes.byref(ip) if ip is not None else None), cb, keep
