// Shared model-object helpers (see model_util.h).
#include <cstdlib>

#include "common.cuh"
#include "model_util.h"

namespace mb {
namespace {

__global__ void k_set_scalars(float* dst, float a, float b) {
  dst[0] = a;
  dst[1] = b;
}

__global__ void k_step_prologue(const double* sched, int* counter, float* scal) {
  const int i = *counter;
  scal[0] = (float)sched[i];
  scal[2] = (float)(sched[i + 1] - sched[i]);
  *counter = i + 1;
}

}  // namespace

bool profile_requested() {
  const char* pe = getenv("MOLD_B200_PROFILE");
  return pe && pe[0] == '1';
}

cudaError_t launch_set_scalars(float* scal, float a, float b, cudaStream_t st) {
  k_set_scalars<<<1, 1, 0, st>>>(scal, a, b);
  return cudaGetLastError();
}

cudaError_t launch_step_prologue(const double* sched, int* counter, float* scal, cudaStream_t st) {
  k_step_prologue<<<1, 1, 0, st>>>(sched, counter, scal);
  return cudaGetLastError();
}

mb_status upload_vec1(int ggml_type, int64_t len, const void* data, size_t nbytes, int on_device, Vec1* out) {
  MB_CHECK(ggml_type == MB_GGML_F32 || ggml_type == MB_GGML_F16 || ggml_type == MB_GGML_BF16, MB_ERR_UNSUPPORTED,
           "1-D tensors must be F32, F16 or BF16");
  const int64_t rb = len * (ggml_type == MB_GGML_F32 ? 4 : 2);
  MB_CHECK((int64_t)nbytes == rb, MB_ERR_INVALID, "nbytes does not match the 1-D tensor length");
  Vec1 v;
  v.n = len;
  MB_TRY(dalloc(&v.dev, (size_t)len));
  void* tmp = nullptr;
  if (cudaMalloc(&tmp, nbytes) != cudaSuccess) {
    cudaFree(v.dev);
    return set_error(MB_ERR_NOMEM, "staging alloc failed");
  }
  cudaError_t e = cudaMemcpy(tmp, data, nbytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = launch_dequant(ggml_type, tmp, 1, len, rb, v.dev, 0, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(tmp);
  if (e != cudaSuccess) {
    cudaFree(v.dev);
    return cuda_error(e, "vector upload");
  }
  *out = v;
  return MB_OK;
}

mb_status upload_matrix(int ggml_type, int64_t n_rows, int64_t n_cols, const void* data, size_t nbytes,
                        int on_device, bool gemm, mb_weight** out) {
  mb_weight* w = nullptr;
  MB_TRY(mb_weight_create(ggml_type, n_rows, n_cols, data, nbytes, on_device, &w));
  const bool gemm_ready =
      w->type == MB_GGML_BF16 ? n_cols % 64 == 0 : (gemm_type_supported(w->type) && n_cols % 256 == 0);
  if (gemm && !gemm_ready) {
    // e.g. img_in [3072, 64]: rows shorter than the GEMM's quantized K step.
    mb_weight* wb = new mb_weight(*w);
    wb->type = MB_GGML_BF16;
    wb->row_bytes = n_cols * 2;
    if (cudaMalloc(&wb->dev, (size_t)n_rows * n_cols * 2) != cudaSuccess) {
      delete wb;
      mb_weight_destroy(w);
      return set_error(MB_ERR_NOMEM, "bf16 copy alloc failed");
    }
    cudaError_t e = launch_dequant(w->type, w->dev, n_rows, n_cols, w->row_bytes, wb->dev, 1, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    mb_weight_destroy(w);
    if (e != cudaSuccess) {
      mb_weight_destroy(wb);
      return cuda_error(e, "bf16 conversion");
    }
    w = wb;
  }
  *out = w;
  return MB_OK;
}

}  // namespace mb
