// K3: batched quantized GEMV (M = 1) for the conditioning path: the stems'
// MLPs (time_in / guidance_in / vector_in, flux/offload.rs:583-609) and every
// block's AdaLN modulation silu(vec) -> Linear (flux/offload.rs:117-156).
// All of a step's modulations depend only on vec, so they run as ONE launch over
// a job table (one job per weight). Weight-bandwidth bound: each weight byte is
// read once; one warp per output row, lanes stride over 64-value units.
#include "common.cuh"
#include "internal.h"

namespace mb {
namespace gemv {

constexpr int kWarps = 8;  // rows per block
constexpr int kMaxLen = 4096;

struct Inputs {
  GemvInput in[4];
};

MB_DEV float h16(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }

__global__ void __launch_bounds__(kWarps * 32)
    k_gemv(const GemvJob* __restrict__ jobs, const int2* __restrict__ blocks, GemvJob inline_job, Inputs ins) {
  __shared__ float xs[kMaxLen];
  __shared__ float xsum[kMaxLen / 32];
  const int2 bj = jobs ? blocks[blockIdx.x] : make_int2(0, blockIdx.x * kWarps);
  const GemvJob job = jobs ? jobs[bj.x] : inline_job;
  const GemvInput in = ins.in[job.x_slot];
  const int K = job.n_cols;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v = 0.f;
    for (int t = 0; t < in.n_parts; t++) v += in.parts[t][i];
    xs[i] = in.apply_silu ? silu(v) : v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < K / 32; i += blockDim.x) {
    float s = 0.f;
    for (int t = 0; t < 32; t++) s += xs[i * 32 + t];
    xsum[i] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = bj.y + warp;
  if (row >= job.n_rows) return;
  const uint8_t* wr = (const uint8_t*)job.w + (int64_t)row * job.row_bytes;
  float acc = 0.f;
  if (job.type == MB_GGML_Q4_K) {
    const int units = K / 64;
    for (int u = lane; u < units; u += 32) {
      const int kb = u >> 2, g = u & 3;
      const uint8_t* b = wr + kb * 144;
      const uint4 h = *(const uint4*)b;
      const uint4 qa = *(const uint4*)(b + 16 + 32 * g), qb = *(const uint4*)(b + 32 + 32 * g);
      const float d = h16(h.x), dmin = h16(h.x >> 16);
      const uint8_t* s = b + 4;
      int sc0, m0, sc1, m1;
      const int j0 = 2 * g, j1 = 2 * g + 1;
      if (j0 < 4) { sc0 = s[j0] & 63; m0 = s[j0 + 4] & 63; }
      else { sc0 = (s[j0 + 4] & 0xF) | ((s[j0 - 4] >> 6) << 4); m0 = (s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4); }
      if (j1 < 4) { sc1 = s[j1] & 63; m1 = s[j1 + 4] & 63; }
      else { sc1 = (s[j1 + 4] & 0xF) | ((s[j1 - 4] >> 6) << 4); m1 = (s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4); }
      const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const float* x = xs + kb * 256 + g * 64;
      float dlo = 0.f, dhi = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++) {
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const uint32_t byte = (w[i] >> (8 * t)) & 0xFFu;
          dlo += (float)(byte & 0xF) * x[4 * i + t];
          dhi += (float)(byte >> 4) * x[32 + 4 * i + t];
        }
      }
      const float* xsm = xsum + (kb * 256 + g * 64) / 32;
      acc += d * (float)sc0 * dlo - dmin * (float)m0 * xsm[0] + d * (float)sc1 * dhi - dmin * (float)m1 * xsm[1];
    }
  } else if (job.type == MB_GGML_Q8_0) {
    const int nb = K / 32;
    for (int bidx = lane; bidx < nb; bidx += 32) {
      const uint16_t* b = (const uint16_t*)(wr + bidx * 34);
      const float d = h16(b[0]);
      const float* x = xs + bidx * 32;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const uint32_t two = b[1 + i];
        s += (float)(int8_t)(two & 0xFF) * x[2 * i] + (float)(int8_t)(two >> 8) * x[2 * i + 1];
      }
      acc += d * s;
    }
  } else if (job.type == MB_GGML_F32) {
    const float* wf = (const float*)wr;
    for (int i = lane; i < K; i += 32) acc += wf[i] * xs[i];
  } else if (job.type == MB_GGML_F16) {
    const __half* wf = (const __half*)wr;
    for (int i = lane; i < K; i += 32) acc += __half2float(wf[i]) * xs[i];
  } else {
    const uint16_t* wf = (const uint16_t*)wr;
    for (int i = lane; i < K; i += 32) acc += __uint_as_float((uint32_t)wf[i] << 16) * xs[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) job.y[row] = acc + (job.bias ? job.bias[row] : 0.f);
}

}  // namespace gemv

cudaError_t launch_gemv_batch(const GemvJob* jobs_dev, int n_jobs, const int* block_job_dev, int n_blocks,
                              const GemvInput* inputs, int n_inputs, int max_len, cudaStream_t st) {
  (void)n_jobs;
  if (max_len > gemv::kMaxLen || n_inputs > 4) return cudaErrorInvalidValue;
  gemv::Inputs ins = {};
  for (int i = 0; i < n_inputs; i++) ins.in[i] = inputs[i];
  GemvJob dummy = {};
  gemv::k_gemv<<<n_blocks, gemv::kWarps * 32, 0, st>>>(jobs_dev, (const int2*)block_job_dev, dummy, ins);
  return cudaGetLastError();
}

// Single-weight GEMV without a device job table (mb_qgemv).
cudaError_t launch_gemv_single(const mb_weight* w, const float* x, int apply_silu, const float* bias, float* y,
                               cudaStream_t st) {
  if (w->n_cols > gemv::kMaxLen) return cudaErrorInvalidValue;
  GemvJob j = {};
  j.w = w->dev;
  j.type = w->type;
  j.n_rows = (int)w->n_rows;
  j.n_cols = (int)w->n_cols;
  j.row_bytes = w->row_bytes;
  j.bias = bias;
  j.y = y;
  j.x_slot = 0;
  gemv::Inputs ins = {};
  ins.in[0].parts[0] = x;
  ins.in[0].n_parts = 1;
  ins.in[0].apply_silu = apply_silu;
  ins.in[0].len = (int)w->n_cols;
  const int blocks = (int)((w->n_rows + gemv::kWarps - 1) / gemv::kWarps);
  gemv::k_gemv<<<blocks, gemv::kWarps * 32, 0, st>>>(nullptr, nullptr, j, ins);
  return cudaGetLastError();
}

}  // namespace mb

extern "C" mb_status mb_qgemv(const mb_weight* w, const float* x, int apply_silu, const float* bias, float* y,
                              void* stream) {
  using namespace mb;
  MB_CHECK(w && x && y, MB_ERR_INVALID, "weight, x or y is NULL");
  MB_CHECK(w->n_cols <= 4096, MB_ERR_INVALID, "mb_qgemv supports K <= 4096");
  MB_CUDA(launch_gemv_single(w, x, apply_silu, bias, y, (cudaStream_t)stream));
  return MB_OK;
}
