//! Raw bindings of `include/mold_b200.h`, the C ABI of libmold_b200.so (one `extern "C"`
//! declaration per `MB_API` entry point, in header order). `tests/test_crate_ffi.py` checks
//! that the names and parameter counts here equal the header's.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

/// `mb_status`: 0 = MB_OK; see the `MB_*` constants.
pub type MbStatus = c_int;
pub const MB_OK: MbStatus = 0;
pub const MB_ERR_INVALID: MbStatus = 1;
pub const MB_ERR_UNSUPPORTED: MbStatus = 2;
pub const MB_ERR_CUDA: MbStatus = 3;
pub const MB_ERR_TIMEOUT: MbStatus = 4;
pub const MB_ERR_NOMEM: MbStatus = 5;
pub const MB_ERR_NOT_READY: MbStatus = 6;

/// GGUF type ids (`MB_GGML_*`).
pub const MB_GGML_F32: c_int = 0;
pub const MB_GGML_F16: c_int = 1;
pub const MB_GGML_Q4_0: c_int = 2;
pub const MB_GGML_Q4_1: c_int = 3;
pub const MB_GGML_Q5_0: c_int = 6;
pub const MB_GGML_Q5_1: c_int = 7;
pub const MB_GGML_Q8_0: c_int = 8;
pub const MB_GGML_Q4_K: c_int = 12;
pub const MB_GGML_Q5_K: c_int = 13;
pub const MB_GGML_Q6_K: c_int = 14;
pub const MB_GGML_BF16: c_int = 30;
pub const MB_DT_F32: c_int = 0;
pub const MB_DT_BF16: c_int = 1;
pub const MB_EPI_NONE: c_int = 0;
pub const MB_EPI_GELU_TANH: c_int = 1;
pub const MB_EPI_GATE_RESIDUAL: c_int = 2;

#[repr(C)]
pub struct MbWeight {
    _p: [u8; 0],
}
#[repr(C)]
pub struct MbFlux {
    _p: [u8; 0],
}
#[repr(C)]
pub struct MbQwen {
    _p: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct MbFluxConfig {
    pub in_channels: c_int,
    pub vec_in_dim: c_int,
    pub context_in_dim: c_int,
    pub hidden_size: c_int,
    pub mlp_hidden: c_int,
    pub num_heads: c_int,
    pub depth: c_int,
    pub depth_single: c_int,
    pub axes_dim: [c_int; 3],
    pub theta: c_int,
    pub guidance_embed: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct MbQwenConfig {
    pub in_channels: c_int,
    pub out_channels: c_int,
    pub patch_size: c_int,
    pub joint_attention_dim: c_int,
    pub hidden_size: c_int,
    pub num_heads: c_int,
    pub num_layers: c_int,
    pub mlp_hidden: c_int,
    pub axes_dim: [c_int; 3],
    pub theta: c_int,
}

/// `mb_inpaint`: packed [L_img, in_channels] f32 device operands (1 = repaint, 0 = preserve).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct MbInpaint {
    pub mask: *const f32,
    pub original: *const f32,
    pub noise: *const f32,
}

/// `mb_step_callback`: runs on a CUDA host-function thread after each finished step; it must
/// not call CUDA or mold_b200.
pub type MbStepCallback = Option<unsafe extern "C" fn(user: *mut c_void, step: c_int, total: c_int)>;

#[link(name = "mold_b200")]
extern "C" {
    pub fn mb_last_error() -> *const c_char;
    pub fn mb_version() -> c_int;
    pub fn mb_init(device: c_int) -> MbStatus;
    pub fn mb_device_status(status_out: *mut c_int) -> MbStatus;
    pub fn mb_weight_create(
        ggml_type: c_int, n_rows: i64, n_cols: i64, data: *const c_void, nbytes: usize,
        data_on_device: c_int, out: *mut *mut MbWeight,
    ) -> MbStatus;
    pub fn mb_weight_destroy(w: *mut MbWeight) -> MbStatus;
    pub fn mb_weight_info(
        w: *const MbWeight, ggml_type: *mut c_int, n_rows: *mut i64, n_cols: *mut i64,
        dev_ptr: *mut *const c_void,
    ) -> MbStatus;
    pub fn mb_weight_download(w: *const MbWeight, host: *mut c_void, nbytes: usize) -> MbStatus;
    pub fn mb_dequant(
        w: *const MbWeight, out: *mut c_void, out_dtype: c_int, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qlinear(
        w: *const MbWeight, x: *const c_void, x_dtype: c_int, m: i64, ldx: i64, y: *mut c_void,
        y_dtype: c_int, ldy: i64, bias: *const f32, epilogue: c_int, gelu_from: i64, gate: *const f32,
        residual: *const f32, ldr: i64, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qlinear_f32_static(
        w: *const MbWeight, x: *const f32, m: i64, ldx: i64, y: *mut c_void, y_dtype: c_int, ldy: i64,
        bias: *const f32, epilogue: c_int, gelu_from: i64, gate: *const f32, residual: *const f32, ldr: i64,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qgemv(
        w: *const MbWeight, x: *const f32, apply_silu: c_int, bias: *const f32, y: *mut f32,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_ln_modulate(
        x: *const f32, m: i64, c: i64, ldx: i64, shift: *const f32, scale: *const f32, y: *mut c_void,
        ldy: i64, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_rope_table(
        ids: *const f32, l: i64, n_axes: c_int, axes_dim: *const c_int, theta: c_int, pe: *mut f32,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qk_norm_rope(
        qkv: *const c_void, m: i64, ld_qkv: i64, h: c_int, q_scale: *const f32, k_scale: *const f32,
        pe: *const f32, row_offset: i64, l_total: i64, q: *mut c_void, k: *mut c_void, v: *mut c_void,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_attention(
        q: *const c_void, k: *const c_void, v: *const c_void, h: c_int, lq: i64, lk: i64, n_valid_keys: i64,
        out: *mut c_void, ldo: i64, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qk_norm_rope_ex(
        qkv: *const c_void, m: i64, ld_qkv: i64, h: c_int, q_scale: *const f32, k_scale: *const f32,
        pe: *const f32, row_offset: i64, l_total: i64, q: *mut c_void, k: *mut c_void, v: *mut c_void,
        kv_pos: *const c_int, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_attention_ex(
        q: *const c_void, k: *const c_void, v: *const c_void, h: c_int, lq: i64, lk: i64, n_valid_keys: i64,
        out: *mut c_void, ldo: i64, split_row: i64, out2: *mut c_void, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_rms_norm(
        x: *const f32, m: i64, c: i64, ldx: i64, w: *const f32, eps: f32, y: *mut c_void, ldy: i64,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_cfg_euler_step(
        img: *mut f32, cond: *const f32, uncond: *const f32, n_tok: i64, c: c_int, pp: c_int, guidance: f32,
        dt: f32, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_euler_step(img: *mut f32, pred: *const f32, n: i64, dt: f32, stream: *mut c_void) -> MbStatus;
    pub fn mb_flux_create(
        cfg: *const MbFluxConfig, max_txt: i64, max_img: i64, out: *mut *mut MbFlux,
    ) -> MbStatus;
    pub fn mb_flux_destroy(m: *mut MbFlux) -> MbStatus;
    pub fn mb_flux_set_tensor(
        m: *mut MbFlux, name: *const c_char, ggml_type: c_int, n_rows: i64, n_cols: i64, data: *const c_void,
        nbytes: usize, data_on_device: c_int,
    ) -> MbStatus;
    pub fn mb_flux_missing(m: *const MbFlux, buf: *mut c_char, buflen: usize) -> MbStatus;
    pub fn mb_flux_forward(
        m: *mut MbFlux, img: *const f32, img_ids: *const f32, l_img: i64, txt: *const f32,
        txt_ids: *const f32, l_txt: i64, t: f32, y: *const f32, guidance: f32, pred: *mut f32,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_flux_denoise(
        m: *mut MbFlux, img: *mut f32, img_ids: *const f32, l_img: i64, txt: *const f32, txt_ids: *const f32,
        l_txt: i64, y: *const f32, timesteps: *const f64, n_timesteps: c_int, guidance: f32,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_flux_denoise_ex(
        m: *mut MbFlux, img: *mut f32, img_ids: *const f32, l_img: i64, txt: *const f32, txt_ids: *const f32,
        l_txt: i64, y: *const f32, timesteps: *const f64, n_timesteps: c_int, guidance: f32,
        inpaint: *const MbInpaint, on_step: MbStepCallback, user: *mut c_void, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qwen_create(
        cfg: *const MbQwenConfig, max_txt: i64, max_img: i64, max_batch: c_int, out: *mut *mut MbQwen,
    ) -> MbStatus;
    pub fn mb_qwen_destroy(m: *mut MbQwen) -> MbStatus;
    pub fn mb_qwen_set_tensor(
        m: *mut MbQwen, name: *const c_char, ggml_type: c_int, n_rows: i64, n_cols: i64, data: *const c_void,
        nbytes: usize, data_on_device: c_int,
    ) -> MbStatus;
    pub fn mb_qwen_missing(m: *const MbQwen, buf: *mut c_char, buflen: usize) -> MbStatus;
    pub fn mb_qwen_forward(
        m: *mut MbQwen, img: *const f32, h_tokens: i64, w_tokens: i64, txt: *const f32, txt_mask: *const u8,
        l_txt: i64, batch: c_int, t: f32, pred: *mut f32, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qwen_denoise(
        m: *mut MbQwen, img: *mut f32, h_tokens: i64, w_tokens: i64, txt: *const f32, txt_mask: *const u8,
        l_txt: i64, batch: c_int, sigmas: *const f64, n_sigmas: c_int, guidance: f32, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_qwen_denoise_ex(
        m: *mut MbQwen, img: *mut f32, h_tokens: i64, w_tokens: i64, txt: *const f32, txt_mask: *const u8,
        l_txt: i64, batch: c_int, sigmas: *const f64, n_sigmas: c_int, guidance: f32,
        inpaint: *const MbInpaint, on_step: MbStepCallback, user: *mut c_void, stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_gguf_inspect(
        path: *const c_char, buf: *mut c_char, buflen: usize, n_tensors: *mut i64,
    ) -> MbStatus;
    pub fn mb_flux_load_gguf(
        m: *mut MbFlux, path: *const c_char, embeddings_path: *const c_char, n_loaded: *mut c_int,
    ) -> MbStatus;
    pub fn mb_qwen_load_gguf(m: *mut MbQwen, path: *const c_char, n_loaded: *mut c_int) -> MbStatus;
    pub fn mb_weight_lora_merge(
        w: *mut MbWeight, row_offset: i64, rows: i64, a: *const f32, b: *const f32, rank: c_int, scale: f32,
        stream: *mut c_void,
    ) -> MbStatus;
    pub fn mb_flux_lora_merge(
        m: *mut MbFlux, name: *const c_char, row_offset: i64, rows: i64, a: *const f32, b: *const f32,
        rank: c_int, scale: f32, stream: *mut c_void,
    ) -> MbStatus;
}
