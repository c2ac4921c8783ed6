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

constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 4;
constexpr int kMaxLen = 4096;

struct Inputs {
  GemvInput in[4];
};

MB_DEV float h16(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }

MB_DEV uint32_t sb(uint32_t sy, uint32_t sz, uint32_t sw, int k) {
  const uint32_t w = k < 4 ? sy : (k < 8 ? sz : sw);
  return (w >> ((k & 3) * 8)) & 0xFFu;
}
MB_DEV void q4k_sm(int j, uint32_t sy, uint32_t sz, uint32_t sw, int& sc, int& m) {
  if (j < 4) {
    sc = sb(sy, sz, sw, j) & 63;
    m = sb(sy, sz, sw, j + 4) & 63;
  } else {
    sc = (sb(sy, sz, sw, j + 4) & 0xF) | ((sb(sy, sz, sw, j - 4) >> 6) << 4);
    m = (sb(sy, sz, sw, j + 4) >> 4) | ((sb(sy, sz, sw, j) >> 6) << 4);
  }
}

// One block = 8 warps x 4 rows of one job. The input vector (silu of the sum of its
// parts) and its 32-value partial sums are staged once per block in shared memory;
// each warp streams its 4 weight rows and reuses every staged x value for all 4.
__global__ void __launch_bounds__(kWarps * 32)
    k_gemv(const GemvJob* __restrict__ jobs, const int2* __restrict__ blocks, GemvJob inline_job, Inputs ins) {
  __shared__ __align__(16) float xs[kMaxLen];
  __shared__ float xsum[kMaxLen / 32];
  const int2 bj = jobs ? blocks[blockIdx.x] : make_int2(0, blockIdx.x * kGemvRowsPerBlock);
  const GemvJob job = jobs ? jobs[bj.x] : inline_job;
  const GemvInput in = ins.in[job.x_slot];
  const int K = job.n_cols;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < in.n_parts; t++) {
      const float4 u = *(const float4*)(in.parts[t] + i);
      v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
    }
    if (in.apply_silu) {
      v.x = silu(v.x); v.y = silu(v.y); v.z = silu(v.z); v.w = silu(v.w);
    }
    *(float4*)(xs + i) = v;
  }
  __syncthreads();
  for (int c = warp; c < K / 32; c += kWarps) {
    float v = xs[c * 32 + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) xsum[c] = v;
  }
  __syncthreads();

  const int r0 = bj.y + warp * kRowsPerWarp;
  if (r0 >= job.n_rows) return;
  const int nr = min(kRowsPerWarp, job.n_rows - r0);
  const uint8_t* wbase = (const uint8_t*)job.w + (int64_t)r0 * job.row_bytes;
  float acc[kRowsPerWarp] = {0.f, 0.f, 0.f, 0.f};
  if (job.type == MB_GGML_Q4_K) {
    for (int u = lane; u < K / 64; u += 32) {
      const int kb = u >> 2, g = u & 3;
      const float* xl = xs + kb * 256 + g * 64;
      float x[64];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const float4 t = *(const float4*)(xl + 4 * i);
        x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
      }
      const float s_lo = xsum[(kb * 256 + g * 64) / 32], s_hi = xsum[(kb * 256 + g * 64) / 32 + 1];
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarp; rr++) {
        if (rr < nr) {
          const uint8_t* b = wbase + (int64_t)rr * job.row_bytes + kb * 144;
          const uint4 h = __ldg((const uint4*)b);
          const uint4 qa = __ldg((const uint4*)(b + 16 + 32 * g)), qb = __ldg((const uint4*)(b + 32 + 32 * g));
          const float d = h16(h.x), dmin = h16(h.x >> 16);
          int sc0, m0, sc1, m1;
          q4k_sm(2 * g, h.y, h.z, h.w, sc0, m0);
          q4k_sm(2 * g + 1, h.y, h.z, h.w, sc1, m1);
          const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
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
          acc[rr] += d * (float)sc0 * dlo - dmin * (float)m0 * s_lo + d * (float)sc1 * dhi - dmin * (float)m1 * s_hi;
        }
      }
    }
  } else if (job.type == MB_GGML_Q8_0) {
    for (int bi = lane; bi < K / 32; bi += 32) {
      const float* xl = xs + bi * 32;
      float x[32];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float4 t = *(const float4*)(xl + 4 * i);
        x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
      }
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarp; rr++) {
        if (rr < nr) {
          const uint8_t* b = wbase + (int64_t)rr * job.row_bytes + bi * 34;
          const uint32_t* a4 = (const uint32_t*)((uintptr_t)b & ~(uintptr_t)3);
          const bool sh = ((uintptr_t)b & 3) != 0;  // block starts 2 bytes into a word
          uint32_t wv[10];
#pragma unroll
          for (int i = 0; i < 10; i++) wv[i] = __ldg(a4 + i);
          const float d = sh ? h16(wv[0] >> 16) : h16(wv[0]);
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const uint32_t q = sh ? wv[i + 1] : __byte_perm(wv[i], wv[i + 1], 0x5432);
#pragma unroll
            for (int t = 0; t < 4; t++) sum += (float)(int8_t)((q >> (8 * t)) & 0xFF) * x[4 * i + t];
          }
          acc[rr] += d * sum;
        }
      }
    }
  } else {
    for (int i = lane; i < K; i += 32) {
      const float xv = xs[i];
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarp; rr++) {
        if (rr < nr) {
          const uint8_t* row = wbase + (int64_t)rr * job.row_bytes;
          float wv;
          if (job.type == MB_GGML_F32) wv = ((const float*)row)[i];
          else if (job.type == MB_GGML_F16) wv = __half2float(((const __half*)row)[i]);
          else wv = __uint_as_float((uint32_t)((const uint16_t*)row)[i] << 16);
          acc[rr] += wv * xv;
        }
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < kRowsPerWarp; rr++) {
    float v = acc[rr];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && rr < nr) job.y[r0 + rr] = v + (job.bias ? job.bias[r0 + rr] : 0.f);
  }
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
  const int blocks = (int)((w->n_rows + kGemvRowsPerBlock - 1) / kGemvRowsPerBlock);
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
