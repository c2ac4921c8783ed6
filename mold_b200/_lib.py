"""ctypes binding of libmold_b200.so (the C ABI declared in include/mold_b200.h).

There is no fallback: if the shared library is missing or does not load, every
entry point raises. Build it with `python -m mold_b200.build`.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MOLD_B200_LIB") or os.path.join(_HERE, "libmold_b200.so")

MB_OK, MB_ERR_INVALID, MB_ERR_UNSUPPORTED, MB_ERR_CUDA, MB_ERR_TIMEOUT, MB_ERR_NOMEM, MB_ERR_NOT_READY = range(7)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16 = 0, 1, 8, 12, 30
GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_Q5_K, GGML_Q6_K = 2, 3, 6, 7, 13, 14
DT_F32, DT_BF16 = 0, 1
EPI_NONE, EPI_GELU_TANH, EPI_GATE_RESIDUAL = 0, 1, 2

_STATUS_NAMES = {0: "MB_OK", 1: "MB_ERR_INVALID", 2: "MB_ERR_UNSUPPORTED", 3: "MB_ERR_CUDA", 4: "MB_ERR_TIMEOUT",
                 5: "MB_ERR_NOMEM", 6: "MB_ERR_NOT_READY"}

# Every exported symbol with (restype, argtypes). Kept in the order of include/mold_b200.h.
P, I32, I64, F32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
# mb_step_callback: void (*)(void* user, int step, int total)
STEP_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int, ctypes.c_int)
SIGNATURES = {
    "mb_last_error": (ctypes.c_char_p, []),
    "mb_version": (I32, []),
    "mb_init": (I32, [I32]),
    "mb_device_status": (I32, [P]),
    "mb_weight_create": (I32, [I32, I64, I64, P, SZ, I32, P]),
    "mb_weight_destroy": (I32, [P]),
    "mb_weight_info": (I32, [P, P, P, P, P]),
    "mb_weight_download": (I32, [P, P, SZ]),
    "mb_dequant": (I32, [P, P, I32, P]),
    "mb_qlinear": (I32, [P, P, I32, I64, I64, P, I32, I64, P, I32, I64, P, P, I64, P]),
    "mb_qgemv": (I32, [P, P, I32, P, P, P]),
    "mb_qlinear_f32_static": (I32, [P, P, I64, I64, P, I32, I64, P, I32, I64, P, P, I64, P]),
    "mb_ln_modulate": (I32, [P, I64, I64, I64, P, P, P, I64, P]),
    "mb_rope_table": (I32, [P, I64, I32, P, I32, P, P]),
    "mb_qk_norm_rope": (I32, [P, I64, I64, I32, P, P, P, I64, I64, P, P, P, P]),
    "mb_attention": (I32, [P, P, P, I32, I64, I64, I64, P, I64, P]),
    "mb_qk_norm_rope_ex": (I32, [P, I64, I64, I32, P, P, P, I64, I64, P, P, P, P, P]),
    "mb_attention_ex": (I32, [P, P, P, I32, I64, I64, I64, P, I64, I64, P, P]),
    "mb_rms_norm": (I32, [P, I64, I64, I64, P, F32, P, I64, P]),
    "mb_cfg_euler_step": (I32, [P, P, P, I64, I32, I32, F32, F32, P]),
    "mb_euler_step": (I32, [P, P, I64, F32, P]),
    "mb_flux_create": (I32, [P, I64, I64, P]),
    "mb_flux_destroy": (I32, [P]),
    "mb_flux_set_tensor": (I32, [P, ctypes.c_char_p, I32, I64, I64, P, SZ, I32]),
    "mb_flux_missing": (I32, [P, P, SZ]),
    "mb_flux_forward": (I32, [P, P, P, I64, P, P, I64, F32, P, F32, P, P]),
    "mb_flux_denoise": (I32, [P, P, P, I64, P, P, I64, P, P, I32, F32, P]),
    "mb_flux_denoise_ex": (I32, [P, P, P, I64, P, P, I64, P, P, I32, F32, P, STEP_CALLBACK, P, P]),
    "mb_qwen_create": (I32, [P, I64, I64, I32, P]),
    "mb_qwen_destroy": (I32, [P]),
    "mb_qwen_set_tensor": (I32, [P, ctypes.c_char_p, I32, I64, I64, P, SZ, I32]),
    "mb_qwen_missing": (I32, [P, P, SZ]),
    "mb_qwen_forward": (I32, [P, P, I64, I64, P, P, I64, I32, F32, P, P]),
    "mb_qwen_denoise": (I32, [P, P, I64, I64, P, P, I64, I32, P, I32, F32, P]),
    "mb_qwen_denoise_ex": (I32, [P, P, I64, I64, P, P, I64, I32, P, I32, F32, P, STEP_CALLBACK, P, P]),
    "mb_gguf_inspect": (I32, [ctypes.c_char_p, P, SZ, P]),
    "mb_flux_load_gguf": (I32, [P, ctypes.c_char_p, ctypes.c_char_p, P]),
    "mb_qwen_load_gguf": (I32, [P, ctypes.c_char_p, P]),
    "mb_weight_lora_merge": (I32, [P, I64, I64, P, P, I32, F32, P]),
    "mb_flux_lora_merge": (I32, [P, ctypes.c_char_p, I64, I64, P, P, I32, F32, P]),
}


class MoldError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class FluxConfigC(ctypes.Structure):
    _fields_ = [("in_channels", I32), ("vec_in_dim", I32), ("context_in_dim", I32), ("hidden_size", I32),
                ("mlp_hidden", I32), ("num_heads", I32), ("depth", I32), ("depth_single", I32),
                ("axes_dim", I32 * 3), ("theta", I32), ("guidance_embed", I32)]


class InpaintC(ctypes.Structure):
    _fields_ = [("mask", P), ("original", P), ("noise", P)]


class QwenConfigC(ctypes.Structure):
    _fields_ = [("in_channels", I32), ("out_channels", I32), ("patch_size", I32), ("joint_attention_dim", I32),
                ("hidden_size", I32), ("num_heads", I32), ("num_layers", I32), ("mlp_hidden", I32),
                ("axes_dim", I32 * 3), ("theta", I32)]


_lib = None


def lib():
    """Load libmold_b200.so (raises if it is absent: there is no CPU or eager fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} not found: build it with `python -m mold_b200.build`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def check(status):
    if status != MB_OK:
        raise MoldError(status, lib().mb_last_error().decode(errors="replace"))
    return status
