// Host-side internals shared by the .cu files of libmold_b200 (not part of the C ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/mold_b200.h"

struct mb_weight {
  int type;        // GGML type id
  int64_t n_rows;  // output features
  int64_t n_cols;  // input features (blocks run along this axis)
  int64_t row_bytes;  // bytes per row on the device (Q6_K: 224 per 256 values, others as in GGUF)
  void* dev;       // device copy of the raw GGML bytes
  int device;
};

namespace mb {

// ---- error plumbing (thread-local last error) ----
mb_status set_error(mb_status s, const std::string& msg);
mb_status cuda_error(cudaError_t e, const char* what);
#define MB_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e__ = (call);                           \
    if (e__ != cudaSuccess) return ::mb::cuda_error(e__, #call); \
  } while (0)
#define MB_CHECK(cond, status, msg)                     \
  do {                                                  \
    if (!(cond)) return ::mb::set_error(status, msg);   \
  } while (0)

int num_sms();
int* device_status_ptr();
bool device_status_ready();  // true once mb_init allocated the status word on the current device  // per-device status word (allocated on first use)
int64_t row_bytes_of(int ggml_type, int64_t n_cols);         // GGUF bytes per row; -1 if unsupported / not divisible
int64_t device_row_bytes_of(int ggml_type, int64_t n_cols);  // bytes per row as stored on the device
bool ggml_type_supported(int ggml_type);
// Weight types the tensor-core GEMM reads (quantized ones need n_cols % 256 == 0; BF16: % 64).
inline bool gemm_type_supported(int t) {
  return t == MB_GGML_BF16 || t == MB_GGML_Q8_0 || t == MB_GGML_Q4_K || t == MB_GGML_Q4_0 || t == MB_GGML_Q4_1 ||
         t == MB_GGML_Q5_0 || t == MB_GGML_Q5_1 || t == MB_GGML_Q5_K || t == MB_GGML_Q6_K;
}

// ---- TMA descriptors ----
bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz);
bool make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                  uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                  uint32_t b2, CUtensorMapSwizzle swz);

// ---- per-device scratch (grown on demand; used by the f32-input path of mb_qlinear) ----
void* device_scratch(size_t bytes);

// ---- launchers (return cudaError_t of the launch) ----
struct GemmEpilogue {
  int kind;          // MB_EPI_*
  int out_bf16;      // 1: bf16 output, 0: f32
  int64_t gelu_from;
  void* y;
  int64_t ldy;
  const float* bias;
  const float* gate;
  const float* res;
  int64_t ldr;
};
cudaError_t launch_qgemm(const mb_weight* w, const void* x_bf16, int64_t M, int64_t ldx, const GemmEpilogue& epi,
                         cudaStream_t st);
// Up to two independent GEMMs (same weight type) in one persistent launch (e.g. the text and
// image streams of a double block), so the small one fills SMs the large one leaves idle.
struct GemmProblem {
  const mb_weight* w;
  const void* x;
  int64_t M, ldx;
  GemmEpilogue epi;
};
cudaError_t launch_qgemm_group(int n, const GemmProblem* g, cudaStream_t st);
cudaError_t launch_dequant(int type, const void* raw, int64_t n_rows, int64_t n_cols, int64_t row_bytes, void* out,
                           int out_bf16, cudaStream_t st);
cudaError_t launch_relayout_q6k(const void* in, void* out, int64_t n_superblocks, cudaStream_t st);
cudaError_t launch_cast_f32_bf16(const float* x, int64_t M, int64_t K, int64_t ldx, void* y, int64_t ldy,
                                 cudaStream_t st);

struct GemvJob {
  const void* w;       // raw GGML rows
  int type;
  int n_rows, n_cols;
  int64_t row_bytes;
  const float* bias;   // [n_rows] or null
  float* y;            // [n_rows]
  int x_slot;          // which staged input vector (0..3)
  int row_begin;       // first global row of this job (prefix sum)
};
struct GemvInput {
  const float* parts[3];  // x = silu?(sum of non-null parts)
  int n_parts;
  int apply_silu;
  int len;
};
constexpr int kGemvRowsPerBlock = 32;  // rows of one job handled by one GEMV block
// Runs a batch of GEMV jobs: one launch stages the inputs (len % 32 == 0, <= 4096) into
// `stage` (gemv_stage_floats() floats, owned by the caller), one launch runs every job.
// jobs_dev / block_job_dev live in device memory.
// `kinds`: bit gemv_kind(type) set for every weight type among the jobs (one kernel per kind
// runs; blocks of a job of the other kind exit at once).
// `smem_row_bytes`: the largest row_bytes among the batch's Q4_K / Q8_0 jobs (their blocks copy
// their rows to shared memory in one bulk copy; 0 if there are none).
cudaError_t launch_gemv_batch(const GemvJob* jobs_dev, int kinds, const int* block_job_dev, int n_blocks,
                              const GemvInput* inputs, int n_inputs, float* stage, int64_t smem_row_bytes,
                              cudaStream_t st);
// Row bytes a Q4_K / Q8_0 GEMV block stages in shared memory for this weight type (0 = none).
int64_t gemv_smem_row_bytes(int ggml_type, int64_t row_bytes);
// 0: Q4_K, Q8_0 and plain types (their own row kernels); 1: the other block types (decode_unit)
int gemv_kind(int ggml_type);
size_t gemv_stage_floats();

cudaError_t launch_ln_modulate(const float* x, int64_t M, int64_t C, int64_t ldx, const float* shift,
                               const float* scale, void* y, int64_t ldy, cudaStream_t st);
// Row segments of one elementwise launch (the text / image streams, batch items).
constexpr int kMaxSegs = 4;
struct LnSeg {
  int64_t row0, rows;        // rows of x and y
  const float *shift, *scale;
};
struct LnSegs {
  LnSeg s[kMaxSegs];
  int n;
};
cudaError_t launch_ln_modulate_segs(const float* x, int64_t C, int64_t ldx, const LnSegs& segs, void* y, int64_t ldy,
                                    cudaStream_t st);
struct QkSeg {
  int64_t row0, rows;   // rows of the qkv buffer
  int64_t pos0;         // sequence position (RoPE row, q row) of the segment's first row
  int64_t off;          // element offset of this sequence's [H, L_total, 128] q / k / v
  const int* kv_pos;    // key order of this sequence (NULL = identity)
  const float *qs, *ks; // RMSNorm scales [128]
};
struct QkSegs {
  QkSeg s[kMaxSegs];
  int n;
};
cudaError_t launch_qk_norm_rope_segs(const void* qkv, int64_t ld_qkv, int H, const float* pe, int64_t L_total,
                                     const QkSegs& segs, void* q, void* k, void* v, cudaStream_t st);
cudaError_t launch_rope_table(const float* ids, int64_t L, int n_axes, const int* axes_dim, int theta, float* pe,
                              cudaStream_t st);
cudaError_t launch_qk_norm_rope(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                                const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q,
                                void* k, void* v, cudaStream_t st, const int* kv_pos = nullptr);
// Output rows [0, split_row) go to out, rows [split_row, Lq) to out2 (from its row 0);
// split_row < 0 writes every row to out.
cudaError_t launch_attention(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                             int64_t n_valid, void* out, int64_t ldo, cudaStream_t st, int64_t split_row = -1,
                             void* out2 = nullptr);
// RMSNorm over rows (f32 statistics, learned weight): y bf16 = x / sqrt(mean(x^2) + eps) * w.
cudaError_t launch_rms_norm(const float* x, int64_t M, int64_t C, int64_t ldx, const float* w, float eps, void* y,
                            int64_t ldy, cudaStream_t st);
// Classifier-free guidance with norm rescale, then Euler, on packed latents [n_tok, C * p * p].
cudaError_t launch_cfg_euler(float* img, const float* cond, const float* uncond, int64_t n_tok, int C, int pp,
                             float guidance, float dt, const float* dt_dev, cudaStream_t st);
cudaError_t launch_euler(float* img, const float* pred, int64_t n, float dt, cudaStream_t st);
cudaError_t launch_euler_dev(float* img, const float* pred, int64_t n, const float* dt_dev, cudaStream_t st);
cudaError_t launch_timestep_embedding(const float* t_dev, float scale, float* out, int dim, cudaStream_t st);

}  // namespace mb
