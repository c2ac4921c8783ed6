// Host helpers shared by the model objects (mb_flux, mb_qwen): device allocation with
// status codes, the per-op profiler, the step-prologue kernels of the denoising graphs,
// and conversion of 1-D tensors and of weights the GEMM cannot read in their GGUF type.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <map>
#include <string>
#include <vector>

#include "internal.h"

namespace mb {

struct Vec1 {  // a 1-D f32 tensor on the device (bias, norm weight)
  float* dev = nullptr;
  int64_t n = 0;
};

struct Seg {  // a row range of the residual stream
  int64_t row0, rows;
};

template <typename T>
mb_status dalloc(T** p, size_t n) {
  if (cudaMalloc((void**)p, n * sizeof(T)) != cudaSuccess)
    return set_error(MB_ERR_NOMEM, "cudaMalloc of " + std::to_string(n * sizeof(T)) + " bytes failed");
  return MB_OK;
}

inline mb_status check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return cuda_error(e, what);
  return MB_OK;
}

// Opt-in per-op timing of an eager forward (MOLD_B200_PROFILE=1): CUDA events around every
// launch, summed per op category and printed to stderr. Off by default; never inside a graph.
struct OpProfiler {
  std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> ev;
  void begin(cudaStream_t st) {
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
    ev.push_back({"", {a, b}});
  }
  void end(cudaStream_t st, const std::string& cat) {
    ev.back().first = cat;
    cudaEventRecord(ev.back().second.second, st);
  }
  void report() {
    cudaDeviceSynchronize();
    std::map<std::string, std::pair<int, double>> agg;
    double tot = 0;
    for (auto& e : ev) {
      float ms = 0;
      cudaEventElapsedTime(&ms, e.second.first, e.second.second);
      agg[e.first].first++;
      agg[e.first].second += ms;
      tot += ms;
      cudaEventDestroy(e.second.first);
      cudaEventDestroy(e.second.second);
    }
    fprintf(stderr, "[mold_b200 profile] %zu launches, %.3f ms of kernel time\n", ev.size(), tot);
    for (auto& a : agg)
      fprintf(stderr, "[mold_b200 profile] %-28s %5d launches %9.3f ms %5.1f%%\n", a.first.c_str(), a.second.first,
              a.second.second, 100.0 * a.second.second / tot);
    ev.clear();
  }
};
inline OpProfiler* g_prof = nullptr;

bool profile_requested();  // MOLD_B200_PROFILE=1

// scal[0] = a, scal[1] = b.
cudaError_t launch_set_scalars(float* scal, float a, float b, cudaStream_t st);
// scal[0] = sched[i], scal[2] = sched[i+1] - sched[i] (f64 difference), scal[3] = sched[i+1],
// scal[4] = 1 - sched[i+1], then ++*counter. Runs at the start of each replayed step so one
// captured graph serves every step. scal must hold 8 floats.
cudaError_t launch_step_prologue(const double* sched, int* counter, float* scal, cudaStream_t st);
// img[i] = img[i] * mask[i] + (orig[i] * scal[4] + noise[i] * scal[3]) * (1 - mask[i]), f32 [n].
cudaError_t launch_inpaint_blend(float* img, int64_t n, const float* scal, const float* mask, const float* orig,
                                 const float* noise, cudaStream_t st);
// Launches `graph` n_steps times on st; with fn, a host function after each launch calls
// fn(user, step, n_steps) once that step has finished on the device (cudaLaunchHostFunc).
cudaError_t enqueue_steps(cudaGraphExec_t graph, int n_steps, mb_step_callback fn, void* user, cudaStream_t st);

// Uploads a 1-D F32/F16/BF16 tensor as f32.
mb_status upload_vec1(int ggml_type, int64_t len, const void* data, size_t nbytes, int on_device, Vec1* out);
// Creates the weight; when `gemm` and the GEMM cannot read its type at this row length
// (quantized rows not a multiple of 256, F32/F16 storage), keeps a BF16 copy instead.
mb_status upload_matrix(int ggml_type, int64_t n_rows, int64_t n_cols, const void* data, size_t nbytes,
                        int on_device, bool gemm, mb_weight** out);

}  // namespace mb

#define MB_TRY(expr)              \
  do {                            \
    mb_status s__ = (expr);       \
    if (s__ != MB_OK) return s__; \
  } while (0)
#define TIMED(cat, expr)                    \
  do {                                      \
    if (::mb::g_prof) ::mb::g_prof->begin(st); \
    mb_status s__ = (expr);                 \
    if (s__ != MB_OK) return s__;           \
    if (::mb::g_prof) ::mb::g_prof->end(st, cat); \
  } while (0)
