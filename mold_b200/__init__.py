"""mold_b200 — B200-native (sm_100a) quantized-DiT denoising hot path for mold.

Host-side mirror of the reference interfaces this library replaces:
  QTensor / QMatMul            candle-core-mold 0.9.10 (QMatMul::from_weights / forward)
  dequantize                   QTensor::dequantize (qwen_image/quantized_transformer.rs:60-67)
  FluxTransformer              crates/mold-inference/src/flux/transformer.rs (forward + denoise)
  QwenTransformer              qwen_image/quantized_transformer.rs:991-1139 + the pipeline's step loop
  sampling.get_schedule, ...   candle flux::sampling as called in flux/pipeline.rs:2044-2158

All arithmetic runs in libmold_b200.so behind the C ABI (include/mold_b200.h);
this package only moves pointers. PyTorch provides device memory and streams.
"""
from ._lib import (  # noqa: F401
    GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q5_K,
    GGML_Q6_K, DT_F32, DT_BF16,
    EPI_NONE, EPI_GELU_TANH, EPI_GATE_RESIDUAL, MoldError, lib, LIB_PATH, SIGNATURES,
)
from .ops import (  # noqa: F401
    QTensor, QMatMul, init, dequantize, qlinear, qgemv, ln_modulate, rope_table, qk_norm_rope, attention,
    euler_step, device_status, key_order, rms_norm, cfg_euler_step, gguf_inspect,
)
from .flux import FluxConfig, FluxTransformer  # noqa: F401
from .qwen import QwenConfig, QwenTransformer  # noqa: F401
from . import sampling  # noqa: F401
