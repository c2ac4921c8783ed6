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

// scal: [0] t (or sigma), [2] dt = t_next - t, [3] t_next, [4] 1 - t_next (the inpaint blend's
// weights, each formed in f64 and rounded once, as the reference's f64 scalar multiplies are).
__global__ void k_step_prologue(const double* sched, int* counter, float* scal) {
  const int i = *counter;
  scal[0] = (float)sched[i];
  scal[2] = (float)(sched[i + 1] - sched[i]);
  scal[3] = (float)sched[i + 1];
  scal[4] = (float)(1.0 - sched[i + 1]);
  *counter = i + 1;
}

// Per-step host callbacks: one context per enqueued step; the last one frees the array.
struct StepCallCtx {
  mb_step_callback fn;
  void* user;
  int step, total;
  StepCallCtx* array;
};
void CUDART_CB step_trampoline(void* p) {
  StepCallCtx* c = (StepCallCtx*)p;
  c->fn(c->user, c->step, c->total);
  if (c->step == c->total) delete[] c->array;
}

}  // namespace

cudaError_t enqueue_steps(cudaGraphExec_t graph, int n_steps, mb_step_callback fn, void* user, cudaStream_t st) {
  if (!fn) {
    for (int i = 0; i < n_steps; i++) {
      cudaError_t e = cudaGraphLaunch(graph, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  StepCallCtx* ctx = new StepCallCtx[n_steps];
  for (int i = 0; i < n_steps; i++) ctx[i] = StepCallCtx{fn, user, i + 1, n_steps, ctx};
  for (int i = 0; i < n_steps; i++) {
    cudaError_t e = cudaGraphLaunch(graph, st);
    if (e == cudaSuccess) e = cudaLaunchHostFunc(st, step_trampoline, &ctx[i]);
    // On failure the callbacks already enqueued may still run and read ctx: it is leaked.
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

bool profile_requested() {
  const char* pe = getenv("MOLD_B200_PROFILE");
  return pe && pe[0] == '1';
}

namespace {
// Inpainting blend after the step's Euler update (flux/transformer.rs:79-87,
// img2img.rs:36-42,79-98): img = img * mask + ((orig * (1 - t_next)) + (noise * t_next)) * (1 - mask),
// each product and sum rounded separately as the reference's tensor ops are.
__global__ void k_inpaint_blend(float* __restrict__ img, int64_t n, const float* __restrict__ scal,
                                const float* __restrict__ mask, const float* __restrict__ orig,
                                const float* __restrict__ noise) {
  const float t = scal[3], omt = scal[4];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float m = mask[i];
    const float keep = __fadd_rn(__fmul_rn(orig[i], omt), __fmul_rn(noise[i], t));
    img[i] = __fadd_rn(__fmul_rn(img[i], m), __fmul_rn(keep, __fsub_rn(1.f, m)));
  }
}
}  // namespace

cudaError_t launch_inpaint_blend(float* img, int64_t n, const float* scal, const float* mask, const float* orig,
                                 const float* noise, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_inpaint_blend<<<(int)blocks, 256, 0, st>>>(img, n, scal, mask, orig, noise);
  return cudaGetLastError();
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
