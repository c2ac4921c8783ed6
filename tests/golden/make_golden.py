"""Generates the GGML codec golden vectors in this directory.

Run from the repository root, in a container where the `gguf` 0.19.0 package
is importable (it is the third-party codec the fixtures come from; it is not
needed to *read* the fixtures):

    python tests/golden/make_golden.py

Fixtures (codec_golden.npz):
  q8_in        f32 [64, 256]  seeded N(0, 0.02) (+ a zero row, a row of ±max)
  q8_blocks    gguf-py Q8_0.quantize_blocks of q8_in
  q8_deq       gguf-py Q8_0.dequantize_blocks of q8_blocks
  q4k_blocks   uint8 [96, 144]: 64 blocks of random bytes (finite f16 d/dmin,
               so every 6-bit scale/min packing pattern occurs) + 32 blocks from
               the oracle's own quantizer
  q4k_deq      gguf-py Q4_K.dequantize_blocks of q4k_blocks
  <t>_blocks / <t>_deq for t in q4_0, q4_1, q5_0, q5_1, q5_k, q6_k: 64 blocks of random bytes
               (finite, moderate f16 scale fields) + 16 blocks from the oracle's own quantizer,
               and gguf-py's dequantize_blocks of them
  <t>_qin / <t>_qblocks for t in q4_0, q4_1, q5_0, q5_1: f32 [16, 256] seeded input (one zero
               block) and gguf-py's quantize of it (ggml's reference quantizers)
  lora_<t>_raw / lora_<t>_out for t in q8_0, q4_0, q4_1, q5_0, q5_1, bf16, with lora_A f32 [1, 256],
               lora_B f32 [16, 1], lora_row0 = 8, lora_scale = 0.75: a [48, 256] weight quantized
               by gguf-py, and the same bytes with rows [8, 24) replaced by gguf-py's quantize of
               dequant(w) + fl(fl(B A) scale) (rank 1, so the delta has one rounding order)
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))

import gguf  # noqa: E402
from gguf import quants  # noqa: E402

import oracle  # noqa: E402


def main():
    rng = np.random.default_rng(1234)
    q8_in = oracle.randn(7, (64, 256), 0.02)
    q8_in[0] = 0.0
    q8_in[1, ::2] = 3.0
    q8_in[1, 1::2] = -3.0
    q8_blocks = quants.quantize(q8_in, gguf.GGMLQuantizationType.Q8_0)
    q8_deq = quants.dequantize(q8_blocks, gguf.GGMLQuantizationType.Q8_0).reshape(q8_in.shape)

    rand_blocks = rng.integers(0, 256, size=(64, 144), dtype=np.uint8)
    # finite, moderate f16 d / dmin
    d = rng.uniform(-0.01, 0.01, size=(64, 2)).astype(np.float16)
    rand_blocks[:, 0:4] = d.view(np.uint8).reshape(64, 4)
    own = oracle.quantize(oracle.randn(8, (32, 256), 0.02), oracle.GGML_Q4_K).reshape(32, 144)
    q4k_blocks = np.concatenate([rand_blocks, own], axis=0)
    q4k_deq = quants.dequantize(q4k_blocks.reshape(-1), gguf.GGMLQuantizationType.Q4_K).reshape(96, 256)

    extra = {}
    # (ggml id, gguf name, block bytes, block values, byte offsets of f16 scale fields)
    for tid, name, bb, be, f16_at in ((oracle.GGML_Q4_0, "Q4_0", 18, 32, (0,)), (oracle.GGML_Q4_1, "Q4_1", 20, 32, (0, 2)),
                                      (oracle.GGML_Q5_0, "Q5_0", 22, 32, (0,)), (oracle.GGML_Q5_1, "Q5_1", 24, 32, (0, 2)),
                                      (oracle.GGML_Q5_K, "Q5_K", 176, 256, (0, 2)), (oracle.GGML_Q6_K, "Q6_K", 210, 256, (208,))):
        rb = rng.integers(0, 256, size=(64, bb), dtype=np.uint8)
        for off in f16_at:
            rb[:, off:off + 2] = rng.uniform(-0.01, 0.01, size=(64, 1)).astype(np.float16).view(np.uint8).reshape(64, 2)
        own = oracle.quantize(oracle.randn(9 + tid, (16, be), 0.02), tid).reshape(16, bb)
        blocks = np.concatenate([rb, own], axis=0)
        deq = quants.dequantize(blocks.reshape(-1), getattr(gguf.GGMLQuantizationType, name)).reshape(80, be)
        extra[name.lower() + "_blocks"] = blocks
        extra[name.lower() + "_deq"] = deq.astype(np.float32)

    for tid, name in ((oracle.GGML_Q4_0, "Q4_0"), (oracle.GGML_Q4_1, "Q4_1"), (oracle.GGML_Q5_0, "Q5_0"),
                      (oracle.GGML_Q5_1, "Q5_1")):
        qin = oracle.randn(40 + tid, (16, 256), 0.05)
        qin[3, 32:64] = 0.0
        extra[name.lower() + "_qin"] = qin
        extra[name.lower() + "_qblocks"] = quants.quantize(qin, getattr(gguf.GGMLQuantizationType, name))

    lora_A = oracle.randn(60, (1, 256), 0.5)
    lora_B = oracle.randn(61, (16, 1), 0.5)
    row0, scale = 8, np.float32(0.75)
    delta = ((lora_B * lora_A).astype(np.float32) * scale).astype(np.float32)
    extra.update(lora_A=lora_A, lora_B=lora_B, lora_row0=np.int64(row0), lora_scale=scale)
    w = oracle.randn(62, (48, 256), 0.05)
    for name in ("Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "BF16"):
        gt = getattr(gguf.GGMLQuantizationType, name)
        raw = quants.quantize(w, gt)
        deq = quants.dequantize(raw, gt).reshape(w.shape).astype(np.float32)
        merged = (deq[row0:row0 + 16] + delta).astype(np.float32)
        out_raw = raw.copy()
        out_raw[row0:row0 + 16] = quants.quantize(merged, gt)
        extra["lora_" + name.lower() + "_raw"] = raw
        extra["lora_" + name.lower() + "_out"] = out_raw

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "codec_golden.npz")
    np.savez_compressed(out, q8_in=q8_in, q8_blocks=q8_blocks, q8_deq=q8_deq,
                        q4k_blocks=q4k_blocks, q4k_deq=q4k_deq, **extra)
    print("wrote", out)


if __name__ == "__main__":
    main()
