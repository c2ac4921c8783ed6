// C-ABI entry points: runtime, weights, single kernels. (FLUX model entry points: flux.cu.)
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace mb {

static int* g_status[64];

int* device_status_ptr() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!g_status[dev]) {
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(ptr, 0, sizeof(int));
    g_status[dev] = (int*)ptr;
  }
  return g_status[dev];
}

bool device_status_ready() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev >= 0 && dev < 64 && g_status[dev] != nullptr;
}

static thread_local std::string t_last_error;

mb_status set_error(mb_status s, const std::string& msg) {
  t_last_error = msg;
  return s;
}
mb_status cuda_error(cudaError_t e, const char* what) {
  return set_error(MB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

static int g_num_sms[64];

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!g_num_sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 148;
  }
  return g_num_sms[dev];
}

bool ggml_type_supported(int t) {
  return t == MB_GGML_F32 || t == MB_GGML_F16 || t == MB_GGML_BF16 || t == MB_GGML_Q8_0 || t == MB_GGML_Q4_K ||
         t == MB_GGML_Q4_0 || t == MB_GGML_Q4_1 || t == MB_GGML_Q5_0 || t == MB_GGML_Q5_1 || t == MB_GGML_Q5_K ||
         t == MB_GGML_Q6_K;
}

int64_t row_bytes_of(int t, int64_t n_cols) {
  switch (t) {
    case MB_GGML_F32: return n_cols * 4;
    case MB_GGML_F16:
    case MB_GGML_BF16: return n_cols * 2;
    case MB_GGML_Q8_0: return n_cols % 32 ? -1 : n_cols / 32 * 34;
    case MB_GGML_Q4_K: return n_cols % 256 ? -1 : n_cols / 256 * 144;
    case MB_GGML_Q4_0: return n_cols % 32 ? -1 : n_cols / 32 * 18;
    case MB_GGML_Q4_1: return n_cols % 32 ? -1 : n_cols / 32 * 20;
    case MB_GGML_Q5_0: return n_cols % 32 ? -1 : n_cols / 32 * 22;
    case MB_GGML_Q5_1: return n_cols % 32 ? -1 : n_cols / 32 * 24;
    case MB_GGML_Q5_K: return n_cols % 256 ? -1 : n_cols / 256 * 176;
    case MB_GGML_Q6_K: return n_cols % 256 ? -1 : n_cols / 256 * 210;
    default: return -1;
  }
}

int64_t device_row_bytes_of(int t, int64_t n_cols) {
  if (t == MB_GGML_Q6_K) return n_cols % 256 ? -1 : n_cols / 256 * 224;
  return row_bytes_of(t, n_cols);
}

// ---------------------------------------------------------------- TMA encode
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_encodeTiled_t)p;
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return false;
  (void)elem_bytes;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                  uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                  uint32_t b2, CUtensorMapSwizzle swz) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return false;
  (void)elem_bytes;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- scratch
static std::mutex g_scratch_mu;
static void* g_scratch[64];
static size_t g_scratch_size[64];

void* device_scratch(size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_size[dev] < bytes) {
    if (g_scratch[dev]) {
      cudaDeviceSynchronize();
      cudaFree(g_scratch[dev]);
    }
    g_scratch[dev] = nullptr;
    g_scratch_size[dev] = 0;
    if (cudaMalloc(&g_scratch[dev], bytes) != cudaSuccess) return nullptr;
    g_scratch_size[dev] = bytes;
  }
  return g_scratch[dev];
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace mb

using namespace mb;

extern "C" {

const char* mb_last_error(void) { return t_last_error.c_str(); }

int mb_version(void) { return 100; }

mb_status mb_init(int device) {
  MB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  MB_CUDA(cudaGetDeviceProperties(&prop, device));
  MB_CHECK(prop.major == 10 && prop.minor == 0, MB_ERR_UNSUPPORTED,
           "mold_b200 kernels are built for sm_100a (B200); device " + std::to_string(device) + " is sm_" +
               std::to_string(prop.major) + std::to_string(prop.minor));
  MB_CHECK(encode_fn() != nullptr, MB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
  num_sms();
  MB_CHECK(device_status_ptr() != nullptr, MB_ERR_NOMEM, "device status word allocation failed");
  return MB_OK;
}

mb_status mb_device_status(int* status_out) {
  MB_CHECK(status_out, MB_ERR_INVALID, "status_out is NULL");
  int* st = device_status_ptr();
  MB_CHECK(st, MB_ERR_NOMEM, "device status word unavailable");
  MB_CUDA(cudaMemcpy(status_out, st, sizeof(int), cudaMemcpyDeviceToHost));
  MB_CUDA(cudaMemset(st, 0, sizeof(int)));
  return MB_OK;
}

mb_status mb_weight_create(int ggml_type, int64_t n_rows, int64_t n_cols, const void* data, size_t nbytes,
                           int data_on_device, mb_weight** out) {
  MB_CHECK(out, MB_ERR_INVALID, "out is NULL");
  *out = nullptr;
  MB_CHECK(ggml_type_supported(ggml_type), MB_ERR_UNSUPPORTED, "unsupported ggml type " + std::to_string(ggml_type));
  MB_CHECK(n_rows > 0 && n_cols > 0, MB_ERR_INVALID, "weight shape must be positive");
  int64_t rb = row_bytes_of(ggml_type, n_cols);
  MB_CHECK(rb > 0, MB_ERR_INVALID,
           "n_cols " + std::to_string(n_cols) + " is not a multiple of the block size of ggml type " +
               std::to_string(ggml_type));
  MB_CHECK((int64_t)nbytes == rb * n_rows, MB_ERR_INVALID,
           "nbytes " + std::to_string(nbytes) + " != " + std::to_string(rb * n_rows) + " expected for the shape");
  MB_CHECK(data, MB_ERR_INVALID, "data is NULL");
  mb_weight* w = new mb_weight();
  w->type = ggml_type;
  w->n_rows = n_rows;
  w->n_cols = n_cols;
  w->row_bytes = device_row_bytes_of(ggml_type, n_cols);
  cudaGetDevice(&w->device);
  const size_t dev_bytes = (size_t)w->row_bytes * (size_t)n_rows;
  if (cudaMalloc(&w->dev, dev_bytes) != cudaSuccess) {
    delete w;
    return set_error(MB_ERR_NOMEM, "cudaMalloc of " + std::to_string(dev_bytes) + " bytes for a weight failed");
  }
  cudaError_t e = cudaSuccess;
  if (ggml_type == MB_GGML_Q6_K) {
    // re-lay 210-byte super-blocks into 224-byte ones (16-byte aligned chunks)
    void* tmp = nullptr;
    e = cudaMalloc(&tmp, nbytes);
    if (e == cudaSuccess)
      e = cudaMemcpy(tmp, data, nbytes, data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_relayout_q6k(tmp, w->dev, (int64_t)(nbytes / 210), 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (tmp) cudaFree(tmp);
  } else {
    e = cudaMemcpy(w->dev, data, nbytes, data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    delete w;
    return cuda_error(e, "weight upload");
  }
  *out = w;
  return MB_OK;
}

mb_status mb_weight_destroy(mb_weight* w) {
  if (!w) return MB_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != w->device) cudaSetDevice(w->device);
  cudaFree(w->dev);
  if (cur != w->device) cudaSetDevice(cur);
  delete w;
  return MB_OK;
}

mb_status mb_weight_info(const mb_weight* w, int* ggml_type, int64_t* n_rows, int64_t* n_cols, const void** dev_ptr) {
  MB_CHECK(w, MB_ERR_INVALID, "weight is NULL");
  if (ggml_type) *ggml_type = w->type;
  if (n_rows) *n_rows = w->n_rows;
  if (n_cols) *n_cols = w->n_cols;
  if (dev_ptr) *dev_ptr = w->dev;
  return MB_OK;
}

mb_status mb_weight_download(const mb_weight* w, void* host, size_t nbytes) {
  MB_CHECK(w && host, MB_ERR_INVALID, "weight or host buffer is NULL");
  const int64_t rb = row_bytes_of(w->type, w->n_cols);
  MB_CHECK(nbytes == (size_t)(rb * w->n_rows), MB_ERR_INVALID,
           "host buffer holds " + std::to_string(nbytes) + " bytes, the weight " + std::to_string(rb * w->n_rows));
  if (w->row_bytes == rb) {
    MB_CUDA(cudaMemcpy(host, w->dev, nbytes, cudaMemcpyDeviceToHost));
    return MB_OK;
  }
  // Q6_K: 224-byte device super-blocks back to GGUF's 210
  std::vector<uint8_t> dev((size_t)(w->row_bytes * w->n_rows));
  MB_CUDA(cudaMemcpy(dev.data(), w->dev, dev.size(), cudaMemcpyDeviceToHost));
  const int64_t nsb = w->n_rows * (w->n_cols / 256);
  for (int64_t i = 0; i < nsb; i++) memcpy((uint8_t*)host + i * 210, dev.data() + i * 224, 210);
  return MB_OK;
}

mb_status mb_dequant(const mb_weight* w, void* out, int out_dtype, void* stream) {
  MB_CHECK(w && out, MB_ERR_INVALID, "weight or out is NULL");
  MB_CHECK(out_dtype == MB_DT_F32 || out_dtype == MB_DT_BF16, MB_ERR_INVALID, "out_dtype must be F32 or BF16");
  MB_CUDA(launch_dequant(w->type, w->dev, w->n_rows, w->n_cols, w->row_bytes, out, out_dtype == MB_DT_BF16,
                         (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_qlinear(const mb_weight* w, const void* x, int x_dtype, int64_t M, int64_t ldx, void* y, int y_dtype,
                     int64_t ldy, const float* bias, int epilogue, int64_t gelu_from, const float* gate,
                     const float* residual, int64_t ldr, void* stream) {
  MB_CHECK(w && x && y, MB_ERR_INVALID, "weight, x or y is NULL");
  MB_CHECK(M >= 0, MB_ERR_INVALID, "M must be >= 0");
  MB_CHECK(gemm_type_supported(w->type), MB_ERR_UNSUPPORTED,
           "mb_qlinear supports BF16 and the quantized types Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K (got ggml type " + std::to_string(w->type) + ")");
  const int64_t K = w->n_cols, N = w->n_rows;
  MB_CHECK(K % 64 == 0, MB_ERR_INVALID, "K must be a multiple of 64");
  MB_CHECK(w->type == MB_GGML_BF16 || K % 256 == 0, MB_ERR_INVALID, "quantized K must be a multiple of 256");
  MB_CHECK(M < (1LL << 31) && N < (1LL << 31), MB_ERR_INVALID, "M and N must fit in 31 bits");
  MB_CHECK(ldx >= K && ldy >= N, MB_ERR_INVALID, "ldx must be >= K and ldy >= N");
  MB_CHECK(x_dtype == MB_DT_BF16 || x_dtype == MB_DT_F32, MB_ERR_INVALID, "x_dtype must be BF16 or F32");
  MB_CHECK(y_dtype == MB_DT_BF16 || y_dtype == MB_DT_F32, MB_ERR_INVALID, "y_dtype must be BF16 or F32");
  MB_CHECK(epilogue >= MB_EPI_NONE && epilogue <= MB_EPI_GATE_RESIDUAL, MB_ERR_INVALID, "unknown epilogue");
  if (epilogue == MB_EPI_GATE_RESIDUAL) {
    MB_CHECK(y_dtype == MB_DT_F32 && gate && residual && ldr >= N, MB_ERR_INVALID,
             "gate-residual epilogue needs f32 y, gate, residual and ldr >= N");
  }
  cudaStream_t st = (cudaStream_t)stream;
  const void* xb = x;
  int64_t ldxb = ldx;
  if (x_dtype == MB_DT_F32) {
    MB_CHECK(ldx % 4 == 0 && aligned16(x), MB_ERR_INVALID, "f32 x must be 16-byte aligned with ldx % 4 == 0");
    void* s = device_scratch((size_t)M * K * 2);
    MB_CHECK(s || M == 0, MB_ERR_NOMEM, "scratch allocation for the f32->bf16 input failed");
    MB_CUDA(launch_cast_f32_bf16((const float*)x, M, K, ldx, s, K, st));
    xb = s;
    ldxb = K;
  }
  MB_CHECK(aligned16(xb) && (ldxb * 2) % 16 == 0, MB_ERR_INVALID, "bf16 x must be 16-byte aligned with ldx % 8 == 0");
  GemmEpilogue e;
  e.kind = epilogue;
  e.out_bf16 = y_dtype == MB_DT_BF16;
  e.gelu_from = epilogue == MB_EPI_GELU_TANH ? gelu_from : (int64_t)1 << 40;
  e.y = y;
  e.ldy = ldy;
  e.bias = bias;
  e.gate = gate;
  e.res = residual;
  e.ldr = ldr;
  MB_CUDA(launch_qgemm(w, xb, M, ldxb, e, st));
  return MB_OK;
}

mb_status mb_ln_modulate(const float* x, int64_t M, int64_t C, int64_t ldx, const float* shift, const float* scale,
                         void* y, int64_t ldy, void* stream) {
  MB_CHECK(x && shift && scale && y, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(C % 128 == 0 && C <= 8192 && ldx >= C && ldy >= C && ldx % 4 == 0 && ldy % 8 == 0, MB_ERR_INVALID,
           "ln_modulate needs C % 128 == 0, C <= 8192, ldx % 4 == 0, ldy % 8 == 0");
  MB_CUDA(launch_ln_modulate(x, M, C, ldx, shift, scale, y, ldy, (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_rope_table(const float* ids, int64_t L, int n_axes, const int* axes_dim, int theta, float* pe,
                        void* stream) {
  MB_CHECK(ids && axes_dim && pe && n_axes > 0 && n_axes <= 4, MB_ERR_INVALID, "bad rope_table arguments");
  int tot = 0;
  for (int i = 0; i < n_axes; i++) {
    MB_CHECK(axes_dim[i] % 2 == 0, MB_ERR_INVALID, "axes_dim entries must be even");
    tot += axes_dim[i];
  }
  MB_CHECK(tot == 128, MB_ERR_INVALID, "sum(axes_dim) must equal head_dim 128");
  MB_CUDA(launch_rope_table(ids, L, n_axes, axes_dim, theta, pe, (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_qk_norm_rope(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                          const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q, void* k,
                          void* v, void* stream) {
  MB_CHECK(qkv && q_scale && k_scale && pe && q && k && v, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(H > 0 && ld_qkv >= 3LL * H * 128 && ld_qkv % 8 == 0 && row_offset >= 0 && row_offset + M <= L_total,
           MB_ERR_INVALID, "bad qk_norm_rope shape");
  MB_CUDA(launch_qk_norm_rope(qkv, M, ld_qkv, H, q_scale, k_scale, pe, row_offset, L_total, q, k, v,
                              (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_attention(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                       int64_t n_valid_keys, void* out, int64_t ldo, void* stream) {
  MB_CHECK(q && k && v && out, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(H > 0 && Lq > 0 && Lk > 0 && ldo >= (int64_t)H * 128 && ldo % 8 == 0, MB_ERR_INVALID,
           "bad attention shape");
  MB_CHECK(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out), MB_ERR_INVALID,
           "attention buffers must be 16-byte aligned");
  if (n_valid_keys <= 0 || n_valid_keys > Lk) n_valid_keys = Lk;
  MB_CUDA(launch_attention(q, k, v, H, Lq, Lk, n_valid_keys, out, ldo, (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_qk_norm_rope_ex(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                             const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q,
                             void* k, void* v, const int* kv_pos, void* stream) {
  MB_CHECK(qkv && q_scale && k_scale && pe && q && k && v, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(H > 0 && ld_qkv >= 3LL * H * 128 && ld_qkv % 8 == 0 && row_offset >= 0 && row_offset + M <= L_total,
           MB_ERR_INVALID, "bad qk_norm_rope shape");
  MB_CUDA(launch_qk_norm_rope(qkv, M, ld_qkv, H, q_scale, k_scale, pe, row_offset, L_total, q, k, v,
                              (cudaStream_t)stream, kv_pos));
  return MB_OK;
}

mb_status mb_attention_ex(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                          int64_t n_valid_keys, void* out, int64_t ldo, int64_t split_row, void* out2, void* stream) {
  MB_CHECK(q && k && v && out, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(H > 0 && Lq > 0 && Lk > 0 && ldo >= (int64_t)H * 128 && ldo % 8 == 0, MB_ERR_INVALID,
           "bad attention shape");
  MB_CHECK(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) && (!out2 || aligned16(out2)),
           MB_ERR_INVALID, "attention buffers must be 16-byte aligned");
  MB_CHECK(split_row < 0 || split_row >= Lq || out2, MB_ERR_INVALID, "split_row inside [0, Lq) needs out2");
  if (n_valid_keys <= 0 || n_valid_keys > Lk) n_valid_keys = Lk;
  MB_CUDA(launch_attention(q, k, v, H, Lq, Lk, n_valid_keys, out, ldo, (cudaStream_t)stream, split_row, out2));
  return MB_OK;
}

mb_status mb_rms_norm(const float* x, int64_t M, int64_t C, int64_t ldx, const float* w, float eps, void* y,
                      int64_t ldy, void* stream) {
  MB_CHECK(x && w && y, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(M >= 0 && C > 0 && C % 128 == 0 && C <= 8192 && ldx >= C && ldx % 4 == 0 && ldy >= C && ldy % 4 == 0,
           MB_ERR_INVALID, "rms_norm needs C % 128 == 0, C <= 8192, ldx, ldy >= C and multiples of 4");
  MB_CHECK(aligned16(x) && aligned16(w) && ((uintptr_t)y & 7) == 0, MB_ERR_INVALID, "misaligned rms_norm buffers");
  MB_CUDA(launch_rms_norm(x, M, C, ldx, w, eps, y, ldy, (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_cfg_euler_step(float* img, const float* cond, const float* uncond, int64_t n_tok, int C, int pp,
                            float guidance, float dt, void* stream) {
  MB_CHECK(img && cond && uncond && n_tok >= 0 && C > 0 && pp > 0, MB_ERR_INVALID, "bad cfg_euler arguments");
  MB_CUDA(launch_cfg_euler(img, cond, uncond, n_tok, C, pp, guidance, dt, nullptr, (cudaStream_t)stream));
  return MB_OK;
}

mb_status mb_euler_step(float* img, const float* pred, int64_t n, float dt, void* stream) {
  MB_CHECK(img && pred && n >= 0, MB_ERR_INVALID, "bad euler arguments");
  MB_CUDA(launch_euler(img, pred, n, dt, (cudaStream_t)stream));
  return MB_OK;
}

}  // extern "C"
