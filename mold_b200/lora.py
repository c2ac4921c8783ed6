"""LoRA adapters merged into a GGUF FLUX transformer on the device.

Mirrors crates/mold-inference/src/flux/lora.rs:
  - `LoraAdapter.load` (lora.rs:62-97): `<layer>.lora_A.weight` / `<layer>.lora_B.weight` pairs
    and optional `<layer>.alpha` scalars from a safetensors file; rank = the largest A dim 0.
  - `map_lora_key` (lora.rs:117-231): diffusers key -> FLUX GGUF tensor, directly or as a row
    slice of a fused tensor (img/txt qkv, single-block linear1).
  - `fused_slice_range` (lora.rs:237-266).
  - `apply_lora` = the patch phase of `gguf_lora_var_builder` (lora.rs:661-868): per layer the
    effective scale is scale * alpha / rank(A) when alpha is present, else scale; the delta
    B @ A * scale is added to the (slice of the) dequantized tensor and the tensor is
    re-quantized to its own GGML type. Here that whole step is one kernel per patch
    (mb_flux_lora_merge) working on the weight already resident on the GPU.
"""
import json
import struct
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": None, "F64": np.float64}


def read_safetensors(path):
    """{name: f32 numpy array} of a safetensors file (F32 / F16 / BF16 / F64 tensors).

    Format: u64 little-endian header length, JSON header {name: {dtype, shape, data_offsets}},
    then the data block the offsets index."""
    with open(path, "rb") as f:
        buf = f.read()
    (n,) = struct.unpack("<Q", buf[:8])
    header = json.loads(buf[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _ST_DTYPES:
            raise ValueError(f"safetensors tensor {name}: dtype {dt} is not supported")
        b0, b1 = info["data_offsets"]
        raw = np.frombuffer(buf, dtype=np.uint8, count=b1 - b0, offset=base + b0)
        if dt == "BF16":
            a = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            a = raw.view(_ST_DTYPES[dt]).astype(np.float32)
        out[name] = a.reshape(info["shape"]) if info["shape"] else a.reshape(())
    return out


@dataclass
class LoraLayer:
    a: np.ndarray               # [rank, in]
    b: np.ndarray               # [out, rank]
    alpha: Optional[float] = None


@dataclass
class LoraAdapter:
    layers: dict
    rank: int

    @classmethod
    def load(cls, path):
        return cls.from_tensors(read_safetensors(path), str(path))

    @classmethod
    def from_tensors(cls, tensors, what="LoRA tensors"):
        a_t, b_t, alphas, rank = {}, {}, {}, 0
        for name, t in tensors.items():
            if name.endswith(".lora_A.weight"):
                layer = name[: -len(".lora_A.weight")]
                rank = max(rank, int(t.shape[0]))
                a_t[layer] = t
            elif name.endswith(".lora_B.weight"):
                b_t[name[: -len(".lora_B.weight")]] = t
            elif name.endswith(".alpha") and t.size == 1:
                alphas[name[: -len(".alpha")]] = float(np.asarray(t, dtype=np.float32).reshape(()))
        layers = {k: LoraLayer(a, b_t[k], alphas.get(k)) for k, a in a_t.items() if k in b_t}
        if not layers:
            raise ValueError(f"no LoRA A/B pairs found in {what}")
        return cls(layers, rank)


@dataclass(frozen=True)
class LoraTarget:
    candle_key: str
    component: Optional[int] = None       # None: direct (whole tensor)
    num_components: int = 0               # 0 with a component: single-block linear1 layout


_DOUBLE = {
    "attn.to_q": ("img_attn.qkv", 0, 3), "attn.to_k": ("img_attn.qkv", 1, 3), "attn.to_v": ("img_attn.qkv", 2, 3),
    "attn.add_q_proj": ("txt_attn.qkv", 0, 3), "attn.add_k_proj": ("txt_attn.qkv", 1, 3),
    "attn.add_v_proj": ("txt_attn.qkv", 2, 3),
    "attn.to_out.0": ("img_attn.proj", None, 0), "attn.to_add_out": ("txt_attn.proj", None, 0),
    "ff.net.0.proj": ("img_mlp.0", None, 0), "ff.net.2": ("img_mlp.2", None, 0),
    "ff_context.net.0.proj": ("txt_mlp.0", None, 0), "ff_context.net.2": ("txt_mlp.2", None, 0),
    "norm1.linear": ("img_mod.lin", None, 0), "norm1_context.linear": ("txt_mod.lin", None, 0),
}
_SINGLE = {
    "attn.to_q": ("linear1", 0, 0), "attn.to_k": ("linear1", 1, 0), "attn.to_v": ("linear1", 2, 0),
    "proj_mlp": ("linear1", 3, 0), "proj_out": ("linear2", None, 0), "norm.linear": ("modulation.lin", None, 0),
}


def map_lora_key(diffusers_key):
    """Diffusers LoRA layer name -> LoraTarget, or None for keys the FLUX model has no tensor for
    (lora.rs:117-231)."""
    key = diffusers_key[len("transformer."):] if diffusers_key.startswith("transformer.") else diffusers_key
    for prefix, table, block in (("transformer_blocks.", _DOUBLE, "double_blocks"),
                                 ("single_transformer_blocks.", _SINGLE, "single_blocks")):
        if key.startswith(prefix):
            rest = key[len(prefix):]
            if "." not in rest:
                return None
            idx, layer = rest.split(".", 1)
            if not idx.isdigit():
                return None
            hit = table.get(layer)
            if hit is None:
                return None
            name, comp, ncomp = hit
            return LoraTarget(f"{block}.{idx}.{name}.weight", comp, ncomp)
    return None


def fused_slice_range(base_rows, lora_out_dim, component, num_components):
    """(row offset, rows) of a fused-slice target (lora.rs:237-266): equal thirds for qkv; for
    single-block linear1 [Q, K, V, MLP] the q/k/v slices are lora_out_dim rows each and the MLP
    slice starts after 3 * (base_rows - lora_out_dim) / 3 rows."""
    if num_components:
        size = base_rows // num_components
        return component * size, size
    if component < 3:
        return component * lora_out_dim, lora_out_dim
    qkv = (base_rows - lora_out_dim) // 3
    return 3 * qkv, lora_out_dim


def plan_patches(adapter: LoraAdapter, scale, tensor_rows):
    """[(tensor name, row offset, A, B, effective scale)] for every layer that maps to a tensor of
    the model; `tensor_rows` = {GGUF name: rows}. Returns (patches, skipped keys)."""
    patches, skipped = [], []
    for key, layer in adapter.layers.items():
        target = map_lora_key(key)
        if target is None or target.candle_key not in tensor_rows:
            skipped.append(key)
            continue
        eff = scale * layer.alpha / layer.a.shape[0] if layer.alpha is not None else scale
        base = tensor_rows[target.candle_key]
        out_dim = int(layer.b.shape[0])
        if target.component is None:
            off, size = 0, base
        else:
            off, size = fused_slice_range(base, out_dim, target.component, target.num_components)
        if off + size > base:
            skipped.append(key)  # the reference warns and skips slices past the tensor's end
            continue
        if size != out_dim:  # the reference's tensor add fails on the shape mismatch
            raise ValueError(f"LoRA layer {key}: B has {out_dim} rows, target slice of {target.candle_key} {size}")
        patches.append((target.candle_key, off, layer.a, layer.b, eff))
    return patches, skipped


def apply_lora(model, adapter: LoraAdapter, scale=1.0):
    """Merge `adapter` into a loaded FluxTransformer (all GGUF types the model holds). Returns
    (applied patch count, skipped keys)."""
    from .flux import tensor_specs
    rows = {n: s[0] for n, s in tensor_specs(model.cfg) if len(s) == 2}
    patches, skipped = plan_patches(adapter, scale, rows)
    dev = torch.device(f"cuda:{model.device}")
    for name, off, a, b, eff in patches:
        model.lora_merge(name, torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev),
                         torch.from_numpy(np.ascontiguousarray(b, dtype=np.float32)).to(dev), eff, off)
    return len(patches), skipped
