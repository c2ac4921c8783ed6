/*
 * mold_b200.h — C ABI of the B200 (sm_100a) quantized-DiT denoising hot path.
 *
 * This is the drop-in boundary for mold's GGUF-quantized FLUX / Qwen-Image
 * transformer. Every entry point below names the reference interface it stands
 * in for (paths are inside utensils/mold; third-party candle items carry the
 * crate version pinned in the reference's Cargo.lock).
 *
 * Conventions
 *  - All functions return an mb_status (0 = MB_OK). On failure a message for the
 *    calling thread is available from mb_last_error(). No C++ exception crosses
 *    this boundary. (Reference: candle_core::Result / anyhow::Result with bail!
 *    on shape errors, e.g. qwen_image/quantized_transformer.rs:223-225.)
 *  - Activations are caller-owned device buffers (plain pointers + sizes); the
 *    library never frees them. Weights are copied into library-owned device
 *    memory by mb_weight_create and freed by mb_weight_destroy.
 *  - Every compute call takes an explicit cudaStream_t (passed as void*; NULL =
 *    the legacy default stream) and is asynchronous with respect to the host.
 *  - One thread per device, as in mold's per-GPU worker threads
 *    (crates/mold-server/src/gpu_worker.rs:18-39); calls for different devices
 *    may run concurrently from different threads.
 *  - GGML type ids are GGUF's: F32=0, F16=1, Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8,
 *    Q4_K=12, Q5_K=13, Q6_K=14, BF16=30. Q6_K rows are re-laid on upload (each 210-byte
 *    super-block padded to 224 bytes) so every 256-value chunk starts 16-byte aligned.
 *  - Element types of activations: MB_DT_F32 or MB_DT_BF16.
 */
#ifndef MOLD_B200_H
#define MOLD_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MB_API __attribute__((visibility("default")))
#else
#define MB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MB_OK = 0,
  MB_ERR_INVALID = 1,     /* bad argument, shape or alignment */
  MB_ERR_UNSUPPORTED = 2, /* ggml type / feature not supported */
  MB_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  MB_ERR_TIMEOUT = 4,     /* a kernel gave up on a bounded wait (see mb_device_status) */
  MB_ERR_NOMEM = 5,       /* device allocation failed */
  MB_ERR_NOT_READY = 6    /* model missing tensors / not initialised */
} mb_status;

enum {
  MB_GGML_F32 = 0,
  MB_GGML_F16 = 1,
  MB_GGML_Q4_0 = 2,
  MB_GGML_Q4_1 = 3,
  MB_GGML_Q5_0 = 6,
  MB_GGML_Q5_1 = 7,
  MB_GGML_Q8_0 = 8,
  MB_GGML_Q4_K = 12,
  MB_GGML_Q5_K = 13,
  MB_GGML_Q6_K = 14,
  MB_GGML_BF16 = 30
};
enum { MB_DT_F32 = 0, MB_DT_BF16 = 1 };

/* Epilogues fused into the quantized linear. */
enum {
  MB_EPI_NONE = 0,          /* y = x W^T + b                                         */
  MB_EPI_GELU_TANH = 1,     /* y = gelu_tanh(x W^T + b) for columns >= gelu_from      */
  MB_EPI_GATE_RESIDUAL = 2  /* y = residual + gate[n] * (x W^T + b)  (f32 out; y may alias residual) */
};

typedef struct mb_weight mb_weight;
typedef struct mb_flux mb_flux;

/* ------------------------------------------------------------------ runtime */

/* Message for the last failing call on this thread ("" if none). */
MB_API const char* mb_last_error(void);

/* ABI version (major*10000 + minor*100 + patch). */
MB_API int mb_version(void);

/* Select and initialise a device for the calling thread (driver entry points,
 * SM count). Replaces candle's `Device::new_cuda(ordinal)` as called from
 * crates/mold-inference/src/device.rs:147-180. */
MB_API mb_status mb_init(int device);

/* Read and clear the device status word that kernels raise when a bounded wait
 * expires (0 = no event). */
MB_API mb_status mb_device_status(int* status_out);

/* ------------------------------------------------------------------ weights */

/* Upload one GGUF tensor [n_rows, n_cols] (rows = output features, ggml blocks
 * run along n_cols) in its raw GGML block layout. `data` is host memory unless
 * data_on_device != 0. Replaces `QMatMul::from_weights(Arc<QTensor>)`
 * (candle-core-mold 0.9.10; pattern at crates/mold-inference/src/encoders/qwen3_gguf.rs:273-305)
 * and the per-tensor part of `quantized_var_builder::VarBuilder::from_gguf`
 * (flux/pipeline.rs:976). */
MB_API mb_status mb_weight_create(int ggml_type, int64_t n_rows, int64_t n_cols, const void* data, size_t nbytes,
                           int data_on_device, mb_weight** out);
MB_API mb_status mb_weight_destroy(mb_weight* w);
/* Raw device pointer of the weight bytes and their GGML type. */
MB_API mb_status mb_weight_info(const mb_weight* w, int* ggml_type, int64_t* n_rows, int64_t* n_cols, const void** dev_ptr);
/* Copy the weight's bytes back to host memory in GGUF layout (n_rows x GGUF row bytes; Q6_K's
 * device padding removed). Synchronous. */
MB_API mb_status mb_weight_download(const mb_weight* w, void* host, size_t nbytes);

/* ------------------------------------------------------------------ kernels */

/* K1. Dequantize a whole weight to f32 or bf16 [n_rows, n_cols] (bit-exact GGML
 * decode; bf16 = round-to-nearest-even of that f32). Replaces
 * `QTensor::dequantize` (qwen_image/quantized_transformer.rs:60-67). */
MB_API mb_status mb_dequant(const mb_weight* w, void* out, int out_dtype, void* stream);

/* K2. Quantized linear y[M,N] = epilogue(x[M,K] W^T + bias). x is bf16 (row
 * stride ldx elements) or f32 (converted to bf16 on the way in). y is bf16 or
 * f32 with row stride ldy. bias: f32 [N] or NULL. For MB_EPI_GATE_RESIDUAL y
 * must be f32, gate is f32 [N] and residual f32 [M, ldr] (may equal y).
 * Replaces `QMatMul::forward` (candle, called through quantized_nn::Linear inside
 * flux::quantized_model; flux/transformer.rs:64-72) and `QwenLinear::forward`
 * (qwen_image/quantized_transformer.rs:54-77).
 * Scratch: with an f32 x the bf16 copy goes to a per-device scratch buffer that the
 * library owns and shares with mb_qgemv. It grows on demand; growing it frees the old
 * buffer after a cudaDeviceSynchronize (so that call is not asynchronous) and allocates
 * a larger one. Calls on one device from several host threads or streams whose work
 * overlaps race on this buffer; serialise them, or pass bf16 x (no scratch). */
MB_API mb_status mb_qlinear(const mb_weight* w, const void* x, int x_dtype, int64_t M, int64_t ldx, void* y, int y_dtype,
                     int64_t ldy, const float* bias, int epilogue, int64_t gelu_from, const float* gate,
                     const float* residual, int64_t ldr, void* stream);

/* Same as mb_qlinear with an f32 x, but allocates nothing. No counterpart in the
 * reference: it is for callers that cannot let the library call cudaMalloc (callers
 * whose device memory comes from their own pool or arena, hosts that forbid
 * allocation after start-up). The bf16 copy of
 * x is staged in a fixed 8 MiB array in the library's device image (M * K must be
 * <= 4,194,304; larger inputs are rejected with MB_ERR_INVALID); every GPU that
 * loads the library holds that array until exit. mb_init must have been called on
 * the device first (else MB_ERR_NOT_READY). The first call on a device looks up the
 * array's device address, so make it before any stream capture. All calls on a
 * device share the array: calls whose execution overlaps on the GPU race. */
MB_API mb_status mb_qlinear_f32_static(const mb_weight* w, const float* x, int64_t M, int64_t ldx, void* y,
                                       int y_dtype, int64_t ldy, const float* bias, int epilogue,
                                       int64_t gelu_from, const float* gate, const float* residual, int64_t ldr,
                                       void* stream);

/* K3. Quantized GEMV for the modulation vectors: y[N] = W silu?(x)[K] + bias.
 * Replaces Modulation1/2::forward's silu(vec)->Linear (flux/offload.rs:117-156).
 * Stages silu(x) in the per-device scratch buffer that mb_qlinear's f32 path uses
 * (grown on demand with a device synchronisation; overlapping calls on one device
 * race on it, as for mb_qlinear). */
MB_API mb_status mb_qgemv(const mb_weight* w, const float* x, int apply_silu, const float* bias, float* y, void* stream);

/* K5. LayerNorm (no affine, eps 1e-6) + AdaLN modulate: y = LN(x) * (1 + scale) + shift.
 * x f32 [M, C] (row stride ldx), y bf16 [M, C] (row stride ldy); shift, scale f32 [C].
 * Replaces LayerNorm + broadcast_mul/add (flux/offload.rs:286-295,379-382,424-427). */
MB_API mb_status mb_ln_modulate(const float* x, int64_t M, int64_t C, int64_t ldx, const float* shift, const float* scale,
                         void* y, int64_t ldy, void* stream);

/* RoPE table pe f32 [L, D/2, 2, 2] from position ids f32 [L, n_axes] (EmbedNd:
 * flux2/transformer.rs:99-118,170-184; FLUX.1 axes (16,56,56), theta 10000). */
MB_API mb_status mb_rope_table(const float* ids, int64_t L, int n_axes, const int* axes_dim, int theta, float* pe,
                        void* stream);

/* K6. Split a fused qkv row block, RMSNorm q and k (learned scale [D], eps 1e-6),
 * apply RoPE (pe rows row_offset.. row_offset+M) and write q, k, v in attention
 * layout bf16 [H, L_total, D] at rows row_offset..row_offset+M.
 * qkv: bf16 [M, 3*H*D] with row stride ld_qkv. D must be 128.
 * Replaces SelfAttention::qkv + apply_rope (flux/offload.rs:56-72,191-201). */
MB_API mb_status mb_qk_norm_rope(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                          const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q, void* k,
                          void* v, void* stream);

/* K4. Attention softmax(q k^T / sqrt(D)) v, non-causal, D = 128.
 * q: bf16 [H, Lq, D]; k, v: bf16 [H, Lk, D]; out: bf16 [Lq, ldo] with head h in
 * columns h*D..h*D+D (the (B,H,L,D)->(B,L,H*D) transpose of the reference is
 * fused). n_valid_keys < Lk masks keys >= n_valid_keys (key padding, Qwen).
 * Replaces scaled_dot_product_attention (flux/offload.rs:40-54) and Qwen's
 * masked attention (qwen_image/quantized_transformer.rs:799-816). */
MB_API mb_status mb_attention(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                       int64_t n_valid_keys, void* out, int64_t ldo, void* stream);

/* K6 with a key order: as mb_qk_norm_rope, but the k and v of sequence row r are
 * written to row kv_pos[r] (device int32 [L_total], NULL = r) while q stays at row r.
 * Attention is invariant to the order of its keys, so a caller that places the keys a
 * mask keeps first can pass n_valid_keys to mb_attention_ex instead of a mask.
 * Replaces the key-mask half of Qwen's JointAttention (qwen_image/quantized_transformer.rs:
 * 716-770: QK-RMSNorm, apply_rotary_emb, cat[txt, img] and the [txt_mask, ones] key mask). */
MB_API mb_status mb_qk_norm_rope_ex(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                                    const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total,
                                    void* q, void* k, void* v, const int* kv_pos, void* stream);

/* K4 with a split output: rows [0, split_row) of the result go to out (row stride ldo),
 * rows [split_row, Lq) to out2 from its row 0, so the text and image halves of the joint
 * sequence land in separate buffers (qwen_image/quantized_transformer.rs:772-780,
 * narrow(1, 0, txt) / narrow(1, txt, img)). split_row < 0: everything to out. */
MB_API mb_status mb_attention_ex(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                                 int64_t n_valid_keys, void* out, int64_t ldo, int64_t split_row, void* out2,
                                 void* stream);

/* RMSNorm rows with a learned weight: y bf16 [M, C] = x / sqrt(mean(x^2) + eps) * w;
 * x f32 [M, C] (row stride ldx), w f32 [C], C % 128 == 0, C <= 8192.
 * Replaces DynamicRmsNorm::forward (qwen_image/quantized_transformer.rs:102-108; txt_norm). */
MB_API mb_status mb_rms_norm(const float* x, int64_t M, int64_t C, int64_t ldx, const float* w, float eps, void* y,
                             int64_t ldy, void* stream);

/* Classifier-free guidance with norm rescale fused with the Euler step, on packed latents
 * img, cond, uncond f32 [n_tok, C * pp] (feature c * pp + j for pixel j of the patch):
 * comb = u + g (c - u); pred = comb * ||c|| / max(||comb||, 1e-8) (norms over the C
 * channels of one pixel); img += pred * dt.
 * Replaces qwen_image/pipeline.rs:2693-2698 + QwenImageScheduler::step (sampling.rs:117-129). */
MB_API mb_status mb_cfg_euler_step(float* img, const float* cond, const float* uncond, int64_t n_tok, int C, int pp,
                                   float guidance, float dt, void* stream);

/* K9. Euler step of the flow-matching loop: img += pred * (t_prev - t_curr), f32 [n].
 * Replaces flux/transformer.rs:84 and qwen_image/sampling.rs:117-129. */
MB_API mb_status mb_euler_step(float* img, const float* pred, int64_t n, float dt, void* stream);

/* ------------------------------------------------------------------ FLUX model */

/* FLUX.1 configuration (candle flux::model::Config as used by mold). */
typedef struct {
  int in_channels;        /* 64 */
  int vec_in_dim;         /* 768 */
  int context_in_dim;     /* 4096 */
  int hidden_size;        /* 3072 */
  int mlp_hidden;         /* 12288 */
  int num_heads;          /* 24 (head_dim must be 128) */
  int depth;              /* 19 double-stream blocks */
  int depth_single;       /* 38 single-stream blocks */
  int axes_dim[3];        /* 16, 56, 56 */
  int theta;              /* 10000 */
  int guidance_embed;     /* 1 for dev */
} mb_flux_config;

/* Create a FLUX transformer on the current device for sequences up to
 * max_txt + max_img tokens. Replaces the `FluxTransformer::Quantized` arm
 * (flux/transformer.rs:17-23) built at flux/pipeline.rs:976-977. */
MB_API mb_status mb_flux_create(const mb_flux_config* cfg, int64_t max_txt, int64_t max_img, mb_flux** out);
MB_API mb_status mb_flux_destroy(mb_flux* m);

/* Hand one GGUF tensor to the model by its GGUF name (e.g.
 * "double_blocks.0.img_attn.qkv.weight"); 1-D tensors (biases, norm scales)
 * have n_rows = 1. Names as read by flux/pipeline.rs:255-276. */
MB_API mb_status mb_flux_set_tensor(mb_flux* m, const char* name, int ggml_type, int64_t n_rows, int64_t n_cols,
                             const void* data, size_t nbytes, int data_on_device);

/* Names of tensors the model still lacks (newline separated) — 0 bytes when complete. */
MB_API mb_status mb_flux_missing(const mb_flux* m, char* buf, size_t buflen);

/* One transformer forward (batch 1). Device pointers:
 *   img f32 [L_img, in_channels], img_ids f32 [L_img, 3], txt f32 [L_txt, context_in_dim],
 *   txt_ids f32 [L_txt, 3], y f32 [vec_in_dim]; pred f32 [L_img, in_channels].
 * Replaces `flux::quantized_model::Flux::forward` (WithForward; called at
 * flux/transformer.rs:64-72; math of flux/offload.rs:525-580). */
MB_API mb_status mb_flux_forward(mb_flux* m, const float* img, const float* img_ids, int64_t L_img, const float* txt,
                          const float* txt_ids, int64_t L_txt, float t, const float* y, float guidance, float* pred,
                          void* stream);

/* The whole denoising loop in place on img (f32 [L_img, in_channels], device):
 * for each (t_curr, t_prev) in timesteps: img += forward(img, t_curr) * (t_prev - t_curr).
 * One CUDA graph per step shape is captured on first use and replayed.
 * Replaces `FluxTransformer::denoise` (flux/transformer.rs:30-98; no inpaint context). */
MB_API mb_status mb_flux_denoise(mb_flux* m, float* img, const float* img_ids, int64_t L_img, const float* txt,
                          const float* txt_ids, int64_t L_txt, const float* y, const double* timesteps,
                          int n_timesteps, float guidance, void* stream);

/* Called on a CUDA host-function thread once denoising step `step` (1-based) of `total` has
 * finished on the device. It must not call CUDA or mold_b200 functions. Replaces the
 * per-step `ProgressEvent::DenoiseStep { step, total, elapsed }` of flux/transformer.rs:89-93
 * and qwen_image/pipeline.rs:2720-2724 (the host can time steps by the calls' wall clock). */
typedef void (*mb_step_callback)(void* user, int step, int total);

/* Flow-matching inpainting inputs, all device f32 in the packed latent layout
 * [L_img, in_channels] (patchified like img; the mask is the latent-resolution mask broadcast
 * over the latent channels before packing): 1 = repaint, 0 = preserve. */
typedef struct {
  const float* mask;
  const float* original;  /* clean (VAE-encoded) latents of the source image */
  const float* noise;     /* the noise the initial latent was drawn with */
} mb_inpaint;

/* mb_flux_denoise with inpainting and per-step progress (either may be NULL). After each
 * step's Euler update, with t = the step's t_prev:
 *   img = img * mask + (original * (1 - t) + noise * t) * (1 - mask)
 * inside the same replayed step graph (flux/transformer.rs:79-87, img2img.rs:36-42,79-98).
 * on_step(user, step, total) runs after each step has finished on the device; the call
 * itself stays asynchronous. The reference blends [1, 16, H, W] context tensors with the
 * packed state; here every operand is packed, so the caller patchifies them once. */
MB_API mb_status mb_flux_denoise_ex(mb_flux* m, float* img, const float* img_ids, int64_t L_img, const float* txt,
                                    const float* txt_ids, int64_t L_txt, const float* y, const double* timesteps,
                                    int n_timesteps, float guidance, const mb_inpaint* inpaint,
                                    mb_step_callback on_step, void* user, void* stream);

/* ------------------------------------------------------------------ Qwen-Image model */

typedef struct mb_qwen mb_qwen;

typedef struct {
  int in_channels;          /* 64 = 16 latent channels x patch 2 x 2 */
  int out_channels;         /* 16 */
  int patch_size;           /* 2 */
  int joint_attention_dim;  /* 3584 (text encoder width) */
  int hidden_size;          /* 3072 = num_heads * 128 */
  int num_heads;            /* 24 */
  int num_layers;           /* 60 */
  int mlp_hidden;           /* 12288 */
  int axes_dim[3];          /* 16, 56, 56 */
  int theta;                /* 10000 */
} mb_qwen_config;

/* Create a Qwen-Image transformer on the current device for up to max_batch sequences
 * (2 = conditional + unconditional CFG batch) of max_txt + max_img tokens. Replaces
 * `QuantizedQwenImageTransformer2DModel::new` (qwen_image/quantized_transformer.rs:1004-1040),
 * the `QwenImageTransformer::Quantized` arm (qwen_image/pipeline.rs:177,258-275). */
MB_API mb_status mb_qwen_create(const mb_qwen_config* cfg, int64_t max_txt, int64_t max_img, int max_batch,
                                mb_qwen** out);
MB_API mb_status mb_qwen_destroy(mb_qwen* m);

/* Hand one GGUF tensor to the model by name (e.g. "transformer_blocks.0.attn.to_q.weight";
 * names as built at qwen_image/quantized_transformer.rs:577-1040). 1-D tensors (biases, norm
 * weights) have n_rows = 1. Biases are optional, as in `qlinear` (:79-94). */
MB_API mb_status mb_qwen_set_tensor(mb_qwen* m, const char* name, int ggml_type, int64_t n_rows, int64_t n_cols,
                                    const void* data, size_t nbytes, int data_on_device);

/* Names of required tensors the model still lacks (newline separated) — 0 bytes when complete. */
MB_API mb_status mb_qwen_missing(const mb_qwen* m, char* buf, size_t buflen);

/* One transformer forward over `batch` sequences. Device pointers:
 *   img f32 [batch, L_img, in_channels] packed latents (L_img = h_tokens * w_tokens, raster order),
 *   txt f32 [batch, L_txt, joint_attention_dim] encoder states,
 *   txt_mask u8 [batch, L_txt] (1 = attend; NULL = all ones), pred f32 [batch, L_img, in_channels].
 * t is the timestep value (sigma * 1000). The mask is read back to the host once per call.
 * Replaces `QuantizedQwenImageTransformer2DModel::forward` (quantized_transformer.rs:1048-1139)
 * on packed latents (the patchify / unpatchify reshapes stay with the caller). */
MB_API mb_status mb_qwen_forward(mb_qwen* m, const float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                                 const uint8_t* txt_mask, int64_t L_txt, int batch, float t, float* pred,
                                 void* stream);

/* The denoising loop in place on img (f32 [L_img, in_channels], device): for each step i,
 * t = sigmas[i] * 1000, pred = forward(img); with batch == 2 (txt / txt_mask hold the
 * conditional then the unconditional prompt) pred = CFG with norm rescale (guidance);
 * img += pred * (sigmas[i+1] - sigmas[i]). sigmas: host f64 [n_sigmas]. One CUDA graph per
 * shape is captured on first use and replayed. Replaces the Qwen step loop
 * (qwen_image/pipeline.rs:2655-2716 without inpainting; scheduler sampling.rs:54-129). */
MB_API mb_status mb_qwen_denoise(mb_qwen* m, float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                                 const uint8_t* txt_mask, int64_t L_txt, int batch, const double* sigmas, int n_sigmas,
                                 float guidance, void* stream);

/* mb_qwen_denoise with inpainting and per-step progress (either may be NULL): after each
 * step's (CFG) Euler update, img = img * mask + (original * (1 - s) + noise * s) * (1 - mask)
 * with s = sigmas[i + 1] (qwen_image/pipeline.rs:2708-2715, img2img::apply_flow_match_inpaint),
 * on packed [L_img, in_channels] operands; on_step as for mb_flux_denoise_ex. */
MB_API mb_status mb_qwen_denoise_ex(mb_qwen* m, float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                                    const uint8_t* txt_mask, int64_t L_txt, int batch, const double* sigmas,
                                    int n_sigmas, float guidance, const mb_inpaint* inpaint,
                                    mb_step_callback on_step, void* user, void* stream);

/* ------------------------------------------------------------------ GGUF files */

/* List the tensors of a GGUF (v2/v3) file without touching a GPU: one line per tensor,
 * "name<TAB>ggml type<TAB>dim ... (outermost first)", newline separated, into buf (truncated
 * at buflen - 1). Replaces candle's gguf_file::Content::read as used at flux/pipeline.rs:285-296. */
MB_API mb_status mb_gguf_inspect(const char* path, char* buf, size_t buflen, int64_t* n_tensors);

/* Load every tensor of a FLUX GGUF file into m (names as in the file; tensors the model does
 * not read are skipped). With embeddings_path, the embedding tensors the file lacks (img_in,
 * time_in, vector_in, guidance_in — city96 fine-tune files) are taken from that FLUX GGUF
 * (flux/pipeline.rs:254-330). The file is memory-mapped; each tensor is copied to the device
 * once. Replaces VarBuilder::from_gguf (flux/pipeline.rs:976) for the transformer. */
MB_API mb_status mb_flux_load_gguf(mb_flux* m, const char* path, const char* embeddings_path, int* n_loaded);

/* Load every tensor of a Qwen-Image GGUF file into m (qwen_image/pipeline.rs:258-275). */
MB_API mb_status mb_qwen_load_gguf(mb_qwen* m, const char* path, int* n_loaded);

/* ------------------------------------------------------------------ LoRA merge */

/* Merge a LoRA delta into rows [row_offset, row_offset + rows) of a weight, in place and in the
 * weight's own GGML type (flux/lora.rs:661-868, `gguf_lora_var_builder`: dequantize, add
 * scale * (B A) to the row slice, re-quantize to the original type). A is device f32
 * [rank, n_cols] (lora_A), B is device f32 [rows, rank] (lora_B); scale is the effective scale
 * (user scale * alpha / rank when the adapter has an alpha). Per value
 *   w' = quantize(w + fl(fl(sum_k B[r,k] A[k,c]) * scale)), the sum by fmaf in ascending k.
 * Q8_0, Q4_0, Q4_1, Q5_0, Q5_1 and BF16 / F16 re-quantize with ggml's reference quantizers
 * (idempotent on their own output, so rows outside the slice need no pass); Q4_K, Q5_K and
 * Q6_K with one-pass quantizers of this library. Asynchronous on `stream`. */
MB_API mb_status mb_weight_lora_merge(mb_weight* w, int64_t row_offset, int64_t rows, const float* A, const float* B,
                                      int rank, float scale, void* stream);

/* mb_weight_lora_merge on the FLUX model's tensor `name` (GGUF name, e.g.
 * "double_blocks.0.img_attn.qkv.weight"). Allowed before or after the first forward: the model
 * reads the merged bytes from then on (no forward may be running on another stream). */
MB_API mb_status mb_flux_lora_merge(mb_flux* m, const char* name, int64_t row_offset, int64_t rows, const float* A,
                                    const float* B, int rank, float scale, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MOLD_B200_H */
