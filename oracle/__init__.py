"""CPU oracle for the mold quantized-DiT hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline. The product (``mold_b200``, the CUDA
library behind ``include/mold_b200.h``) never imports, links or calls it.

Pinning status:
  * GGML codecs (``codec.c``): bit-exact against the ``gguf`` 0.19.0 package
    (fixtures in ``tests/golden/``).
  * LoRA merge (``codec.c`` ``or_lora_merge``): for Q8_0 / Q4_0 / Q4_1 / Q5_0 / Q5_1 / BF16
    bit-exact against gguf-py's dequantize + requantize of the merged rows (fixtures); the
    K-type requantizers are this project's own (candle's k-quant quantizer is not vendored
    here), so K-type merges are pinned only through their dequantize.
  * Schedules (``flux_ref.get_schedule``, ``qwen_ref``): pinned against the
    reference's own known-answer tests (qwen_image/sampling.rs:136-140).
  * FLUX / Qwen block math: restated from the reference's in-repo copy of the
    block math (flux/offload.rs, flux2/transformer.rs:99-178); the reference
    cannot be built here (no Rust toolchain, candle not vendored), so the block
    math is **parity unpinned** beyond that restatement.
"""
from .codec import (  # noqa: F401
    GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q5_K,
    GGML_Q6_K,
    block_bytes, block_elems, dequantize, lora_merge, quantize, randn, round_bf16, lib_path,
)
