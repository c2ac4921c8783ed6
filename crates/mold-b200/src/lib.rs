//! mold-b200: mold's quantized DiT denoising hot path on B200 (sm_100a), behind the same
//! layer and model seams mold-inference uses today.
//!
//! * [`B200QMatMul`] stands in for candle's `QMatMul` (`QMatMul::from_arc` + `Module::forward`,
//!   called through `quantized_nn::Linear` inside `flux::quantized_model`, flux/transformer.rs:64-72)
//!   and for `QwenLinear` (qwen_image/quantized_transformer.rs:54-94): the GGUF block bytes go to
//!   the device once, and every forward runs the fused dequant + tcgen05 GEMM (`mb_qlinear`).
//! * [`B200Flux`] is the `FluxTransformer::B200` arm (flux/transformer.rs:11-17): it loads the
//!   GGUF transformer (`mb_flux_load_gguf`, flux/pipeline.rs:254-330,976) and runs the whole
//!   `denoise` loop (flux/transformer.rs:30-98) with inpainting and per-step progress in one call.
//! * [`B200Qwen`] is the `QwenImageTransformer::Quantized` arm (qwen_image/pipeline.rs:177,258-275)
//!   and its step loop (qwen_image/pipeline.rs:2655-2724).
//!
//! Tensors cross the boundary as device pointers of candle CUDA tensors on the worker's device
//! (one GPU worker thread per device, crates/mold-server/src/gpu_worker.rs:18-39); every call is
//! asynchronous on the device's stream.

pub mod ffi;

use std::ffi::{CStr, CString};
use std::os::raw::{c_int, c_void};
use std::path::Path;

use candle_core::quantized::{GgmlDType, QTensor};
use candle_core::{DType, Device, Module, Result, Storage, Tensor};

/// Turn an `mb_status` into a candle error carrying `mb_last_error()`.
pub fn check(rc: ffi::MbStatus) -> Result<()> {
    if rc == ffi::MB_OK {
        return Ok(());
    }
    let msg = unsafe { CStr::from_ptr(ffi::mb_last_error()) }.to_string_lossy().into_owned();
    Err(candle_core::Error::Msg(format!("mold_b200 status {rc}: {msg}")))
}

/// GGUF type id of a candle GGML dtype (the ids of the GGUF file format).
pub fn ggml_type_id(dt: GgmlDType) -> Result<c_int> {
    Ok(match dt {
        GgmlDType::F32 => ffi::MB_GGML_F32,
        GgmlDType::F16 => ffi::MB_GGML_F16,
        GgmlDType::BF16 => ffi::MB_GGML_BF16,
        GgmlDType::Q4_0 => ffi::MB_GGML_Q4_0,
        GgmlDType::Q4_1 => ffi::MB_GGML_Q4_1,
        GgmlDType::Q5_0 => ffi::MB_GGML_Q5_0,
        GgmlDType::Q5_1 => ffi::MB_GGML_Q5_1,
        GgmlDType::Q8_0 => ffi::MB_GGML_Q8_0,
        GgmlDType::Q4K => ffi::MB_GGML_Q4_K,
        GgmlDType::Q5K => ffi::MB_GGML_Q5_K,
        GgmlDType::Q6K => ffi::MB_GGML_Q6_K,
        other => candle_core::bail!("mold_b200 has no kernel for ggml type {other:?}"),
    })
}

/// Select the worker's device once (candle's `Device::new_cuda(ordinal)`, device.rs:147-180).
pub fn init(ordinal: usize) -> Result<()> {
    check(unsafe { ffi::mb_init(ordinal as c_int) })
}

fn cuda_stream(dev: &Device) -> Result<*mut c_void> {
    match dev {
        Device::Cuda(d) => Ok(d.cuda_stream().cu_stream() as *mut c_void),
        _ => candle_core::bail!("mold_b200 needs a CUDA device"),
    }
}

/// Device pointer of a contiguous CUDA tensor (f32 or bf16).
fn device_ptr(t: &Tensor) -> Result<*const c_void> {
    use candle_core::cuda_backend::cudarc::driver::DevicePtr;
    let (storage, layout) = t.storage_and_layout();
    if !layout.is_contiguous() {
        candle_core::bail!("mold_b200 needs contiguous tensors");
    }
    let off = layout.start_offset();
    match &*storage {
        Storage::Cuda(cs) => match t.dtype() {
            DType::F32 => {
                let s = cs.as_cuda_slice::<f32>()?;
                Ok((*s.device_ptr() as usize + 4 * off) as *const c_void)
            }
            DType::BF16 => {
                let s = cs.as_cuda_slice::<half::bf16>()?;
                Ok((*s.device_ptr() as usize + 2 * off) as *const c_void)
            }
            dt => candle_core::bail!("mold_b200 takes f32 or bf16 activations, got {dt:?}"),
        },
        _ => candle_core::bail!("mold_b200 needs CUDA tensors"),
    }
}

/// A GGUF weight resident on the device in its raw GGML block layout.
pub struct B200Weight {
    raw: *mut ffi::MbWeight,
    pub n_rows: usize,
    pub n_cols: usize,
}

unsafe impl Send for B200Weight {}
unsafe impl Sync for B200Weight {}

impl B200Weight {
    /// Upload a `QTensor` [out, in] (`QMatMul::from_weights`): its block bytes are copied once.
    pub fn from_qtensor(qt: &QTensor) -> Result<Self> {
        let (n_rows, n_cols) = qt.shape().dims2()?;
        let bytes = qt.data()?;
        let mut raw = std::ptr::null_mut();
        check(unsafe {
            ffi::mb_weight_create(
                ggml_type_id(qt.dtype())?,
                n_rows as i64,
                n_cols as i64,
                bytes.as_ptr() as *const c_void,
                bytes.len(),
                0,
                &mut raw,
            )
        })?;
        Ok(Self { raw, n_rows, n_cols })
    }
}

impl Drop for B200Weight {
    fn drop(&mut self) {
        unsafe { ffi::mb_weight_destroy(self.raw) };
    }
}

/// The `QMatMul` / `QwenLinear` seam: y = x W^T (+ bias), x f32 or bf16 [.., K] on the GPU.
pub struct B200QMatMul {
    w: B200Weight,
    bias: Option<Tensor>, // f32 [N]
}

impl B200QMatMul {
    pub fn from_qtensor(qt: &QTensor, bias: Option<Tensor>) -> Result<Self> {
        let bias = bias.map(|b| b.to_dtype(DType::F32)?.contiguous()).transpose()?;
        Ok(Self { w: B200Weight::from_qtensor(qt)?, bias })
    }
}

impl Module for B200QMatMul {
    fn forward(&self, x: &Tensor) -> Result<Tensor> {
        let x = x.contiguous()?;
        let dims = x.dims().to_vec();
        let k = *dims.last().unwrap();
        if k != self.w.n_cols {
            candle_core::bail!("x has K = {k}, the weight expects {}", self.w.n_cols);
        }
        let m = x.elem_count() / k;
        let mut out_dims = dims.clone();
        *out_dims.last_mut().unwrap() = self.w.n_rows;
        // The output keeps x's dtype, as candle's QMatMul returns x's float type.
        let y = Tensor::zeros(out_dims, x.dtype(), x.device())?;
        let x_dt = if x.dtype() == DType::BF16 { ffi::MB_DT_BF16 } else { ffi::MB_DT_F32 };
        let bias = match &self.bias {
            Some(b) => device_ptr(b)? as *const f32,
            None => std::ptr::null(),
        };
        check(unsafe {
            ffi::mb_qlinear(
                self.w.raw,
                device_ptr(&x)?,
                x_dt,
                m as i64,
                k as i64,
                device_ptr(&y)? as *mut c_void,
                x_dt,
                self.w.n_rows as i64,
                bias,
                ffi::MB_EPI_NONE,
                0,
                std::ptr::null(),
                std::ptr::null(),
                0,
                cuda_stream(x.device())?,
            )
        })?;
        Ok(y)
    }
}

/// Flow-matching inpainting context in the packed [1, L_img, 64] layout (the reference's
/// `InpaintContext`, img_utils.rs:134-142, patchified like the state).
pub struct PackedInpaint<'a> {
    pub mask: &'a Tensor,
    pub original: &'a Tensor,
    pub noise: &'a Tensor,
}

/// Per-step progress: called with (step, total) once each step has finished on the device.
pub type StepFn<'a> = &'a mut dyn FnMut(usize, usize);

unsafe extern "C" fn step_trampoline(user: *mut c_void, step: c_int, total: c_int) {
    let f = &mut *(user as *mut StepFn);
    f(step as usize, total as usize);
}

/// The `FluxTransformer::B200` arm.
pub struct B200Flux {
    raw: *mut ffi::MbFlux,
    device: Device,
}

unsafe impl Send for B200Flux {}

impl B200Flux {
    /// FLUX.1-dev / schnell configuration (candle flux::model::Config::dev / schnell).
    pub fn config(guidance_embed: bool) -> ffi::MbFluxConfig {
        ffi::MbFluxConfig {
            in_channels: 64,
            vec_in_dim: 768,
            context_in_dim: 4096,
            hidden_size: 3072,
            mlp_hidden: 12288,
            num_heads: 24,
            depth: 19,
            depth_single: 38,
            axes_dim: [16, 56, 56],
            theta: 10000,
            guidance_embed: guidance_embed as c_int,
        }
    }

    /// Create the model for up to max_txt + max_img tokens and load the GGUF transformer
    /// (with the city96 embedding patch when `embeddings` names the FLUX file to take
    /// img_in / time_in / vector_in / guidance_in from).
    pub fn load_gguf(
        cfg: &ffi::MbFluxConfig,
        path: &Path,
        embeddings: Option<&Path>,
        max_txt: usize,
        max_img: usize,
        device: &Device,
    ) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::mb_flux_create(cfg, max_txt as i64, max_img as i64, &mut raw) })?;
        let me = Self { raw, device: device.clone() };
        let p = CString::new(path.to_string_lossy().as_bytes()).map_err(candle_core::Error::wrap)?;
        let e = embeddings
            .map(|e| CString::new(e.to_string_lossy().as_bytes()).map_err(candle_core::Error::wrap))
            .transpose()?;
        let mut n = 0;
        check(unsafe {
            ffi::mb_flux_load_gguf(me.raw, p.as_ptr(), e.as_ref().map_or(std::ptr::null(), |c| c.as_ptr()), &mut n)
        })?;
        Ok(me)
    }

    /// `FluxTransformer::denoise` (flux/transformer.rs:24-98) on the packed state: img
    /// [1, L_img, 64] f32, img_ids [1, L_img, 3], txt [1, L_txt, 4096], txt_ids, vec [1, 768].
    #[allow(clippy::too_many_arguments)]
    pub fn denoise(
        &self,
        img: &Tensor,
        img_ids: &Tensor,
        txt: &Tensor,
        txt_ids: &Tensor,
        vec_: &Tensor,
        timesteps: &[f64],
        guidance: f64,
        mut progress: Option<StepFn>,
        inpaint: Option<&PackedInpaint>,
    ) -> Result<Tensor> {
        let out = img.to_dtype(DType::F32)?.contiguous()?.copy()?;
        let (l_img, l_txt) = (img.dim(1)?, txt.dim(1)?);
        let ip = match inpaint {
            Some(c) => Some(ffi::MbInpaint {
                mask: device_ptr(c.mask)? as *const f32,
                original: device_ptr(c.original)? as *const f32,
                noise: device_ptr(c.noise)? as *const f32,
            }),
            None => None,
        };
        let (cb, user): (ffi::MbStepCallback, *mut c_void) = match progress.as_mut() {
            Some(f) => (Some(step_trampoline), f as *mut StepFn as *mut c_void),
            None => (None, std::ptr::null_mut()),
        };
        let stream = cuda_stream(&self.device)?;
        check(unsafe {
            ffi::mb_flux_denoise_ex(
                self.raw,
                device_ptr(&out)? as *mut f32,
                device_ptr(img_ids)? as *const f32,
                l_img as i64,
                device_ptr(txt)? as *const f32,
                device_ptr(txt_ids)? as *const f32,
                l_txt as i64,
                device_ptr(vec_)? as *const f32,
                timesteps.as_ptr(),
                timesteps.len() as c_int,
                guidance as f32,
                ip.as_ref().map_or(std::ptr::null(), |p| p as *const ffi::MbInpaint),
                cb,
                user,
                stream,
            )
        })?;
        // The callbacks borrow `progress`: wait for the last step before returning.
        self.device.synchronize()?;
        Ok(out)
    }
}

impl Drop for B200Flux {
    fn drop(&mut self) {
        unsafe { ffi::mb_flux_destroy(self.raw) };
    }
}

/// The `QwenImageTransformer::Quantized` arm.
pub struct B200Qwen {
    raw: *mut ffi::MbQwen,
    device: Device,
}

unsafe impl Send for B200Qwen {}

impl B200Qwen {
    /// Qwen-Image configuration (qwen_image/quantized_transformer.rs:1004-1040 defaults).
    pub fn config() -> ffi::MbQwenConfig {
        ffi::MbQwenConfig {
            in_channels: 64,
            out_channels: 16,
            patch_size: 2,
            joint_attention_dim: 3584,
            hidden_size: 3072,
            num_heads: 24,
            num_layers: 60,
            mlp_hidden: 12288,
            axes_dim: [16, 56, 56],
            theta: 10000,
        }
    }

    pub fn load_gguf(
        cfg: &ffi::MbQwenConfig,
        path: &Path,
        max_txt: usize,
        max_img: usize,
        max_batch: usize,
        device: &Device,
    ) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::mb_qwen_create(cfg, max_txt as i64, max_img as i64, max_batch as c_int, &mut raw) })?;
        let me = Self { raw, device: device.clone() };
        let p = CString::new(path.to_string_lossy().as_bytes()).map_err(candle_core::Error::wrap)?;
        let mut n = 0;
        check(unsafe { ffi::mb_qwen_load_gguf(me.raw, p.as_ptr(), &mut n) })?;
        Ok(me)
    }

    /// The step loop of qwen_image/pipeline.rs:2655-2724 on packed latents [L_img, 64]:
    /// `txt` [B, L_txt, 3584] and `mask` u8 [B, L_txt] hold the conditional prompt, then (B = 2)
    /// the unconditional one; `sigmas` are `QwenImageScheduler::new`'s (with the final 0).
    #[allow(clippy::too_many_arguments)]
    pub fn denoise(
        &self,
        latents: &Tensor,
        h_tokens: usize,
        w_tokens: usize,
        txt: &Tensor,
        mask: &Tensor,
        sigmas: &[f64],
        guidance: f64,
        mut progress: Option<StepFn>,
        inpaint: Option<&PackedInpaint>,
    ) -> Result<Tensor> {
        use candle_core::cuda_backend::cudarc::driver::DevicePtr;
        let out = latents.to_dtype(DType::F32)?.contiguous()?.copy()?;
        let mask = mask.to_dtype(DType::U8)?.contiguous()?;
        let mask_ptr = {
            let (st, layout) = mask.storage_and_layout();
            match &*st {
                Storage::Cuda(cs) => *cs.as_cuda_slice::<u8>()?.device_ptr() as usize + layout.start_offset(),
                _ => candle_core::bail!("mold_b200 needs CUDA tensors"),
            }
        };
        let (b, l_txt) = (txt.dim(0)?, txt.dim(1)?);
        let ip = match inpaint {
            Some(c) => Some(ffi::MbInpaint {
                mask: device_ptr(c.mask)? as *const f32,
                original: device_ptr(c.original)? as *const f32,
                noise: device_ptr(c.noise)? as *const f32,
            }),
            None => None,
        };
        let (cb, user): (ffi::MbStepCallback, *mut c_void) = match progress.as_mut() {
            Some(f) => (Some(step_trampoline), f as *mut StepFn as *mut c_void),
            None => (None, std::ptr::null_mut()),
        };
        check(unsafe {
            ffi::mb_qwen_denoise_ex(
                self.raw,
                device_ptr(&out)? as *mut f32,
                h_tokens as i64,
                w_tokens as i64,
                device_ptr(txt)? as *const f32,
                mask_ptr as *const u8,
                l_txt as i64,
                b as c_int,
                sigmas.as_ptr(),
                sigmas.len() as c_int,
                guidance as f32,
                ip.as_ref().map_or(std::ptr::null(), |p| p as *const ffi::MbInpaint),
                cb,
                user,
                cuda_stream(&self.device)?,
            )
        })?;
        self.device.synchronize()?;
        Ok(out)
    }
}

impl Drop for B200Qwen {
    fn drop(&mut self) {
        unsafe { ffi::mb_qwen_destroy(self.raw) };
    }
}
