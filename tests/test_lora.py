"""LoRA host logic (key mapping, slice ranges, adapter parsing, patch planning) and the oracle's
merge, pinned to gguf-py fixtures. Known answers follow crates/mold-inference/src/flux/lora.rs
tests (lora.rs:905-1072)."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from mold_b200.lora import LoraAdapter, LoraTarget, fused_slice_range, map_lora_key, plan_patches, read_safetensors

GOLD = os.path.join(os.path.dirname(__file__), "golden", "codec_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_map_double_block_img_attn_qkv():
    assert map_lora_key("transformer.transformer_blocks.5.attn.to_q") == LoraTarget(
        "double_blocks.5.img_attn.qkv.weight", 0, 3)
    assert map_lora_key("transformer.transformer_blocks.5.attn.to_k").component == 1
    assert map_lora_key("transformer.transformer_blocks.5.attn.to_v").component == 2


def test_map_double_block_txt_attn_qkv():
    assert map_lora_key("transformer.transformer_blocks.0.attn.add_q_proj") == LoraTarget(
        "double_blocks.0.txt_attn.qkv.weight", 0, 3)


@pytest.mark.parametrize("key,expected", [
    ("transformer.transformer_blocks.3.attn.to_out.0", "double_blocks.3.img_attn.proj.weight"),
    ("transformer.transformer_blocks.3.attn.to_add_out", "double_blocks.3.txt_attn.proj.weight"),
    ("transformer.transformer_blocks.3.ff.net.0.proj", "double_blocks.3.img_mlp.0.weight"),
    ("transformer.transformer_blocks.3.ff.net.2", "double_blocks.3.img_mlp.2.weight"),
    ("transformer.transformer_blocks.3.ff_context.net.0.proj", "double_blocks.3.txt_mlp.0.weight"),
    ("transformer.transformer_blocks.3.ff_context.net.2", "double_blocks.3.txt_mlp.2.weight"),
    ("transformer.transformer_blocks.3.norm1.linear", "double_blocks.3.img_mod.lin.weight"),
    ("transformer.transformer_blocks.3.norm1_context.linear", "double_blocks.3.txt_mod.lin.weight"),
])
def test_map_double_block_direct(key, expected):
    assert map_lora_key(key) == LoraTarget(expected)


def test_map_single_block():
    t = map_lora_key("transformer.single_transformer_blocks.7.attn.to_q")
    assert (t.candle_key, t.component) == ("single_blocks.7.linear1.weight", 0)
    assert map_lora_key("transformer.single_transformer_blocks.7.proj_mlp").component == 3
    assert map_lora_key("transformer.single_transformer_blocks.7.proj_out") == LoraTarget("single_blocks.7.linear2.weight")
    assert map_lora_key("transformer.single_transformer_blocks.7.norm.linear") == LoraTarget(
        "single_blocks.7.modulation.lin.weight")
    # the "transformer." prefix is optional
    assert map_lora_key("single_transformer_blocks.7.proj_out") == LoraTarget("single_blocks.7.linear2.weight")


def test_map_unknown_key_returns_none():
    assert map_lora_key("totally.unknown.key") is None
    assert map_lora_key("transformer.transformer_blocks.0.unknown_layer") is None
    assert map_lora_key("transformer.transformer_blocks.x.attn.to_q") is None


def test_fused_slice_range_equal_split():
    assert fused_slice_range(9216, 3072, 0, 3) == (0, 3072)
    assert fused_slice_range(9216, 3072, 1, 3) == (3072, 3072)
    assert fused_slice_range(9216, 3072, 2, 3) == (6144, 3072)


def test_fused_slice_range_single_block():
    assert fused_slice_range(21504, 3072, 0, 0) == (0, 3072)
    assert fused_slice_range(21504, 3072, 1, 0) == (3072, 3072)
    assert fused_slice_range(21504, 3072, 2, 0) == (6144, 3072)
    assert fused_slice_range(21504, 12288, 3, 0) == (9216, 12288)


def write_safetensors(path, tensors):
    """Minimal safetensors writer (F32 / BF16 given as ('BF16', uint16 array))."""
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        if isinstance(t, tuple):
            dt, arr = t
        else:
            dt, arr = "F32", np.ascontiguousarray(t, dtype=np.float32)
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def test_adapter_load_safetensors(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((4, 64)).astype(np.float32)
    b = rng.standard_normal((32, 4)).astype(np.float32)
    b_bf16 = (b.view(np.uint32) >> 16).astype(np.uint16)
    p = tmp_path / "l.safetensors"
    write_safetensors(p, {
        "transformer.transformer_blocks.0.attn.to_q.lora_A.weight": a,
        "transformer.transformer_blocks.0.attn.to_q.lora_B.weight": ("BF16", b_bf16),
        "transformer.transformer_blocks.0.attn.to_q.alpha": np.array(8.0, dtype=np.float32),
        "transformer.transformer_blocks.0.attn.to_k.lora_A.weight": a[:2],  # no B: dropped
    })
    t = read_safetensors(p)
    assert t["transformer.transformer_blocks.0.attn.to_q.lora_B.weight"].dtype == np.float32
    ad = LoraAdapter.load(p)
    assert ad.rank == 4 and list(ad.layers) == ["transformer.transformer_blocks.0.attn.to_q"]
    layer = ad.layers["transformer.transformer_blocks.0.attn.to_q"]
    assert layer.alpha == 8.0
    assert np.array_equal(layer.b, (b_bf16.astype(np.uint32) << 16).view(np.float32))


def test_adapter_without_pairs_fails(tmp_path):
    p = tmp_path / "e.safetensors"
    write_safetensors(p, {"x.lora_A.weight": np.zeros((2, 4), np.float32)})
    with pytest.raises(ValueError, match="no LoRA A/B pairs"):
        LoraAdapter.load(p)


def test_plan_patches_scales_and_slices():
    r, h, m = 4, 64, 256
    a = np.ones((r, h), np.float32)
    layers = {
        "transformer.transformer_blocks.0.attn.to_v": (a, np.ones((h, r), np.float32), 8.0),
        "transformer.single_transformer_blocks.1.proj_mlp": (a, np.ones((m, r), np.float32), None),
        "transformer.single_transformer_blocks.1.attn.to_k": (a, np.ones((h, r), np.float32), 2.0),
        "transformer.transformer_blocks.0.bogus": (a, np.ones((h, r), np.float32), None),
        "transformer.transformer_blocks.9.attn.to_q": (a, np.ones((h, r), np.float32), None),  # no such block
    }
    tensors = {}
    for k, (A, B, al) in layers.items():
        tensors[k + ".lora_A.weight"] = A
        tensors[k + ".lora_B.weight"] = B
        if al is not None:
            tensors[k + ".alpha"] = np.array(al, np.float32)
    ad = LoraAdapter.from_tensors(tensors)
    rows = {"double_blocks.0.img_attn.qkv.weight": 3 * h, "single_blocks.1.linear1.weight": 3 * h + m}
    patches, skipped = plan_patches(ad, 0.5, rows)
    got = {(n, off): eff for n, off, _, _, eff in patches}
    assert got == {("double_blocks.0.img_attn.qkv.weight", 2 * h): 0.5 * 8.0 / r,
                   ("single_blocks.1.linear1.weight", 3 * h): 0.5,
                   ("single_blocks.1.linear1.weight", h): 0.5 * 2.0 / r}
    assert sorted(skipped) == ["transformer.transformer_blocks.0.bogus", "transformer.transformer_blocks.9.attn.to_q"]


def test_plan_patches_shape_mismatch_raises():
    ad = LoraAdapter.from_tensors({"transformer_blocks.0.attn.to_q.lora_A.weight": np.ones((2, 8), np.float32),
                                   "transformer_blocks.0.attn.to_q.lora_B.weight": np.ones((5, 2), np.float32)})
    with pytest.raises(ValueError, match="B has 5 rows"):
        plan_patches(ad, 1.0, {"double_blocks.0.img_attn.qkv.weight": 24})


@pytest.mark.parametrize("name,t", [("q4_0", oracle.GGML_Q4_0), ("q4_1", oracle.GGML_Q4_1), ("q5_0", oracle.GGML_Q5_0),
                                    ("q5_1", oracle.GGML_Q5_1)])
def test_oracle_quantizer_matches_ggml_reference(gold, name, t):
    q = oracle.quantize(gold[name + "_qin"], t)
    assert np.array_equal(q.reshape(-1), gold[name + "_qblocks"].reshape(-1))


LORA_TYPES = [("q8_0", oracle.GGML_Q8_0), ("q4_0", oracle.GGML_Q4_0), ("q4_1", oracle.GGML_Q4_1),
              ("q5_0", oracle.GGML_Q5_0), ("q5_1", oracle.GGML_Q5_1), ("bf16", oracle.GGML_BF16)]


@pytest.mark.parametrize("name,t", LORA_TYPES)
def test_oracle_lora_merge_matches_gguf_requantize(gold, name, t):
    raw = gold["lora_" + name + "_raw"]
    row0 = int(gold["lora_row0"])
    out = oracle.lora_merge(raw.reshape(-1), t, (48, 256), row0, 16, gold["lora_A"], gold["lora_B"],
                            float(gold["lora_scale"]))
    assert np.array_equal(out, gold["lora_" + name + "_out"].reshape(-1))


@pytest.mark.parametrize("t", [oracle.GGML_Q4_K, oracle.GGML_Q5_K, oracle.GGML_Q6_K, oracle.GGML_F16, oracle.GGML_F32])
def test_oracle_lora_merge_other_types(t):
    w = oracle.randn(70, (32, 512), 0.05)
    raw = oracle.quantize(w, t).reshape(-1)
    A = oracle.randn(71, (4, 512), 0.1)
    B = oracle.randn(72, (8, 4), 0.1)
    out = oracle.lora_merge(raw, t, (32, 512), 12, 8, A, B, 0.5)
    rb = raw.size // 32
    assert np.array_equal(out[:12 * rb], raw[:12 * rb]) and np.array_equal(out[20 * rb:], raw[20 * rb:])
    want = oracle.dequantize(raw, t, (32, 512))[12:20] + 0.5 * (B.astype(np.float64) @ A)
    got = oracle.dequantize(out, t, (32, 512))[12:20]
    tol = 0.1 if t == oracle.GGML_Q4_K else 0.05  # the types' own round-trip error
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < tol
