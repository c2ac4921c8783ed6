// K5 LayerNorm+AdaLN modulate, RoPE table, K6 QK-RMSNorm+RoPE+layout, K9 Euler, timestep embedding.
// All HBM-bound: 128-bit vector loads/stores, one warp per row (or per row x head).
#include <math.h>

#include <vector>

#include "common.cuh"
#include "internal.h"

namespace mb {

static int grid_cap(int64_t blocks) {
  int64_t cap = (int64_t)num_sms() * 32;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

MB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ K5
// y = LN(x) * (1 + scale) + shift, LN without affine, eps 1e-6 (flux/offload.rs:286-295,
// qwen_image/quantized_transformer.rs:136-151). One warp per row, the row in registers
// (C <= 128 * VEC); the rows of up to kMaxSegs segments (e.g. the text and image streams,
// each with its own modulation vectors) run in one launch.
template <int VEC>
__global__ void k_ln_modulate(const float* __restrict__ x, int C, int64_t ldx, LnSegs segs,
                              __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = C / 128;  // float4 per lane actually used (<= VEC)
  int64_t total = 0;
  for (int i = 0; i < segs.n; i++) total += segs.s[i].rows;
  for (int64_t u = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); u < total; u += warps) {
    int si = 0;
    int64_t r = u;
    while (si + 1 < segs.n && r >= segs.s[si].rows) r -= segs.s[si++].rows;
    const LnSeg sg = segs.s[si];
    const int64_t row = sg.row0 + r;
    const float* xr = x + row * ldx;
    float4 v[VEC];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      if (i < nvec) {
        v[i] = *(const float4*)(xr + (i * 32 + lane) * 4);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    const float mean = warp_sum(s) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      if (i < nvec) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
      }
    }
    const float var = warp_sum(q) / (float)C;
    const float rstd = 1.f / sqrtf(var + 1e-6f);
    __nv_bfloat16* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      if (i < nvec) {
        const int c = (i * 32 + lane) * 4;
        const float4 sc = __ldg((const float4*)(sg.scale + c)), sh = __ldg((const float4*)(sg.shift + c));
        const float o0 = (v[i].x - mean) * rstd * (1.f + sc.x) + sh.x;
        const float o1 = (v[i].y - mean) * rstd * (1.f + sc.y) + sh.y;
        const float o2 = (v[i].z - mean) * rstd * (1.f + sc.z) + sh.z;
        const float o3 = (v[i].w - mean) * rstd * (1.f + sc.w) + sh.w;
        uint2 w;
        w.x = pack_bf16x2(o0, o1);
        w.y = pack_bf16x2(o2, o3);
        *(uint2*)(yr + c) = w;
      }
    }
  }
}

// Block-per-row form: C / (4 NV) threads per row, NV float4 each (little state per thread, so
// many rows are in flight per SM); the row's sums go through shared memory.
MB_DEV float block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();  // red is reused by the next reduction
  return t;
}

// Mean and sum of squared deviations of two equal-count groups merged (Chan et al.):
// mean = (ma + mb) / 2, M2 = M2a + M2b + (mb - ma)^2 n / 2 for groups of n values each.
MB_DEV void chan_merge(float& m, float& q, float mo, float qo, float n) {
  const float d = mo - m;
  q = q + qo + d * d * (0.5f * n);
  m = 0.5f * (m + mo);
}
// Block-wide mean and M2 from per-thread ones over n values each (blockDim a power-of-two number
// of warps): one pass over the data and one shared-memory exchange, with the two-pass form's
// numerical stability.
MB_DEV void block_mean_m2(float& m, float& q, float n, float2* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o), qo = __shfl_xor_sync(0xffffffffu, q, o);
    chan_merge(m, q, mo, qo, n);
    n *= 2.f;
  }
  if (lane == 0) red[warp] = make_float2(m, q);
  __syncthreads();
  float2 a = red[lane < nw ? lane : 0];
  for (int o = 1; o < nw; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, a.x, o), qo = __shfl_xor_sync(0xffffffffu, a.y, o);
    chan_merge(a.x, a.y, mo, qo, n);
    n *= 2.f;
  }
  m = __shfl_sync(0xffffffffu, a.x, 0);
  q = __shfl_sync(0xffffffffu, a.y, 0);
}

template <int NV>
__global__ void __launch_bounds__(1024) k_ln_modulate_blk(const float* __restrict__ x, int C, int64_t ldx, LnSegs segs,
                                                          __nv_bfloat16* __restrict__ y, int64_t ldy) {
  __shared__ float2 red2[32];
  __shared__ float red[32];
  int si = 0;
  int64_t r = blockIdx.x;
  while (si + 1 < segs.n && r >= segs.s[si].rows) r -= segs.s[si++].rows;
  const LnSeg sg = segs.s[si];
  const int64_t row = sg.row0 + r;
  const float* xr = x + row * ldx;
  const int t = threadIdx.x, nt = blockDim.x;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) v[i] = *(const float4*)(xr + (i * nt + t) * 4);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  float mean, rstd;
  if (((blockDim.x >> 5) & ((blockDim.x >> 5) - 1)) == 0) {
    // one pass: per-thread mean and M2, merged across the block in one exchange
    mean = s * (1.f / (4 * NV));
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
    block_mean_m2(mean, q, (float)(4 * NV), red2);
#pragma unroll
    for (int i = 0; i < NV; i++) {
      v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
    }
    rstd = 1.f / sqrtf(q / (float)C + 1e-6f);
  } else {
    // a number of warps that is not a power of two: two passes through block_sum
    mean = block_sum(s, red) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
      q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    }
    rstd = 1.f / sqrtf(block_sum(q, red) / (float)C + 1e-6f);
  }
  __nv_bfloat16* yr = y + row * ldy;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c = (i * nt + t) * 4;
    const float4 sc = __ldg((const float4*)(sg.scale + c)), sh = __ldg((const float4*)(sg.shift + c));
    uint2 w;
    w.x = pack_bf16x2(v[i].x * rstd * (1.f + sc.x) + sh.x, v[i].y * rstd * (1.f + sc.y) + sh.y);
    w.y = pack_bf16x2(v[i].z * rstd * (1.f + sc.z) + sh.z, v[i].w * rstd * (1.f + sc.w) + sh.w);
    *(uint2*)(yr + c) = w;
  }
}

cudaError_t launch_ln_modulate_segs(const float* x, int64_t C, int64_t ldx, const LnSegs& segs, void* y, int64_t ldy,
                                    cudaStream_t st) {
  int64_t M = 0;
  for (int i = 0; i < segs.n; i++) M += segs.s[i].rows;
  if (M <= 0) return cudaSuccess;
  if (segs.n < 1 || segs.n > kMaxSegs || C % 128 != 0 || C > 8192) return cudaErrorInvalidValue;
  __nv_bfloat16* yb = (__nv_bfloat16*)y;
  // block per row (measured on 4608 x 3072 from cold L2: 2.6 TB/s warp per row, 3.8 TB/s with
  // 128 threads x 6 float4)
#ifndef MB_LN_NV
#define MB_LN_NV 6  // float4 per thread (4608 x 3072 from cold L2: 6 -> 22.5 us, 2 -> 24.5, 8 -> 26.6, 12 -> 30.7)
#endif
  if (M < (int64_t)1 << 31 && C % (128 * MB_LN_NV) == 0 && C / (4 * MB_LN_NV) <= 1024) {
    k_ln_modulate_blk<MB_LN_NV><<<(unsigned)M, (unsigned)(C / (4 * MB_LN_NV)), 0, st>>>(x, (int)C, ldx, segs, yb, ldy);
    return cudaGetLastError();
  }
  if (M < (int64_t)1 << 31 && C % 256 == 0 && C / 8 <= 1024) {
    k_ln_modulate_blk<2><<<(unsigned)M, (unsigned)(C / 8), 0, st>>>(x, (int)C, ldx, segs, yb, ldy);
    return cudaGetLastError();
  }
  const int threads = 256;
  const int g = grid_cap((M + 7) / 8);
  if (C <= 3072)
    k_ln_modulate<24><<<g, threads, 0, st>>>(x, (int)C, ldx, segs, yb, ldy);
  else
    k_ln_modulate<64><<<g, threads, 0, st>>>(x, (int)C, ldx, segs, yb, ldy);
  return cudaGetLastError();
}

cudaError_t launch_ln_modulate(const float* x, int64_t M, int64_t C, int64_t ldx, const float* shift,
                               const float* scale, void* y, int64_t ldy, cudaStream_t st) {
  LnSegs s = {};
  s.n = 1;
  s.s[0] = {0, M, shift, scale};
  return launch_ln_modulate_segs(x, C, ldx, s, y, ldy, st);
}

// ------------------------------------------------------------------ RoPE table
// pe[l][i] = {cos f, -sin f, sin f, cos f}, f = pos_axis(l) * inv_freq_i
// inv_freq_i = 1 / (float)(theta^(2j/dim_a)) for pair j of axis a (flux2/transformer.rs:99-118).
struct RopeTab {
  float inv[64];
  int axis[64];
};

__global__ void k_rope_table(const float* __restrict__ ids, int64_t L, int n_axes, RopeTab tab, float* __restrict__ pe) {
  const int64_t total = L * 64;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = u >> 6;
    const int i = (int)(u & 63);
    const float pos = ids[l * n_axes + tab.axis[i]];
    const float f = __fmul_rn(pos, tab.inv[i]);
    float s, c;
    sincosf(f, &s, &c);
    *(float4*)(pe + u * 4) = make_float4(c, -s, s, c);
  }
}

cudaError_t launch_rope_table(const float* ids, int64_t L, int n_axes, const int* axes_dim, int theta, float* pe,
                              cudaStream_t st) {
  RopeTab tab;
  int k = 0;
  for (int a = 0; a < n_axes; a++) {
    for (int i = 0; i < axes_dim[a]; i += 2) {
      const float p = (float)pow((double)theta, (double)i / (double)axes_dim[a]);
      tab.inv[k] = 1.0f / p;
      tab.axis[k] = a;
      k++;
    }
  }
  k_rope_table<<<grid_cap((L * 64 + 255) / 256), 256, 0, st>>>(ids, L, n_axes, tab, pe);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ K6
// qkv row block [rows, 3*H*128] bf16 -> RMSNorm(q), RMSNorm(k) (eps 1e-6, learned scale),
// RoPE on interleaved pairs, v copied; outputs [H, L_total, 128] bf16 (flux/offload.rs:56-72,
// 191-201; qwen_image/quantized_transformer.rs:716-753). One warp per (sequence row, group of
// G heads): lane l holds features 4l..4l+3 (two rope pairs) of each head, so the row's RoPE
// entries are loaded once per G heads, and all G heads' loads are issued first. G = 4 (cold-L2
// FLUX shape: 8 heads 47.1 us, 4 heads 41.0, 2 heads 43.0).
// Rows of up to kMaxSegs segments (streams, batch items) run in one launch.
template <int G>
__global__ void k_qk_norm_rope(const __nv_bfloat16* __restrict__ qkv, int64_t ld, int H,
                               const float* __restrict__ pe, int64_t L_total, QkSegs segs,
                               __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                               __nv_bfloat16* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t total = 0;
  for (int i = 0; i < segs.n; i++) total += segs.s[i].rows;
  const int groups = (H + G - 1) / G;
  total *= groups;
  for (int64_t u = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); u < total; u += warps) {
    int si = 0;
    int64_t r = u / groups;
    const int h0 = (int)(u % groups) * G;
    while (si + 1 < segs.n && r >= segs.s[si].rows) r -= segs.s[si++].rows;
    const QkSeg sg = segs.s[si];
    const int64_t prow = sg.pos0 + r;  // sequence position: RoPE row and q row
    const int64_t kvrow = sg.kv_pos ? sg.kv_pos[prow] : prow;
    const __nv_bfloat16* src = qkv + (sg.row0 + r) * ld + lane * 4;
    const float4* per = (const float4*)(pe + prow * 256);
    const float4 p0 = __ldg(per + lane * 2), p1 = __ldg(per + lane * 2 + 1);
    const float4 qsc = __ldg((const float4*)(sg.qs + lane * 4));
    const float4 ksc = __ldg((const float4*)(sg.ks + lane * 4));
    __nv_bfloat16* qb = q + sg.off;
    __nv_bfloat16* kb = k + sg.off;
    __nv_bfloat16* vb = v + sg.off;
    {
      const int nh = min(G, H - h0);
      uint2 rq[G], rk[G], rv[G];
#pragma unroll
      for (int j = 0; j < G; j++) {
        if (j < nh) {
          const __nv_bfloat16* sp = src + (h0 + j) * 128;
          rq[j] = *(const uint2*)(sp);
          rk[j] = *(const uint2*)(sp + (int64_t)H * 128);
          rv[j] = *(const uint2*)(sp + (int64_t)2 * H * 128);
        }
      }
#pragma unroll
      for (int j = 0; j < G; j++) {
        if (j < nh) {
          const int h = h0 + j;
          const int64_t dq = ((int64_t)h * L_total + prow) * 128 + lane * 4;
          const int64_t dkv = ((int64_t)h * L_total + kvrow) * 128 + lane * 4;
#pragma unroll
          for (int which = 0; which < 2; which++) {
            const uint2 rr = which ? rk[j] : rq[j];
            const float4 sc = which ? ksc : qsc;
            float x0 = bf16_lo(rr.x), x1 = bf16_hi(rr.x), x2 = bf16_lo(rr.y), x3 = bf16_hi(rr.y);
            const float ms = warp_sum((x0 * x0 + x1 * x1) + (x2 * x2 + x3 * x3)) * (1.f / 128.f);
            const float rinv = 1.f / sqrtf(ms + 1e-6f);
            x0 = x0 * rinv * sc.x;
            x1 = x1 * rinv * sc.y;
            x2 = x2 * rinv * sc.z;
            x3 = x3 * rinv * sc.w;
            const float y0 = p0.x * x0 + p0.y * x1, y1 = p0.z * x0 + p0.w * x1;
            const float y2 = p1.x * x2 + p1.y * x3, y3 = p1.z * x2 + p1.w * x3;
            uint2 o;
            o.x = pack_bf16x2(y0, y1);
            o.y = pack_bf16x2(y2, y3);
            if (which)
              *(uint2*)(kb + dkv) = o;
            else
              *(uint2*)(qb + dq) = o;
          }
          *(uint2*)(vb + dkv) = rv[j];
        }
      }
    }
  }
}

cudaError_t launch_qk_norm_rope_segs(const void* qkv, int64_t ld_qkv, int H, const float* pe, int64_t L_total,
                                     const QkSegs& segs, void* q, void* k, void* v, cudaStream_t st) {
  int64_t M = 0;
  for (int i = 0; i < segs.n; i++) M += segs.s[i].rows;
  if (M <= 0) return cudaSuccess;
  if (segs.n < 1 || segs.n > kMaxSegs) return cudaErrorInvalidValue;
#ifndef MB_QK_G
#define MB_QK_G 4
#endif
  constexpr int G = MB_QK_G;
#ifndef MB_QK_BLK
#define MB_QK_BLK 128  // threads per block (cold-L2 FLUX shape: 128 -> 36.9 us, 256 -> 40.9, 64 -> 38.9)
#endif
  k_qk_norm_rope<G><<<grid_cap((M * ((H + G - 1) / G) + MB_QK_BLK / 32 - 1) / (MB_QK_BLK / 32)), MB_QK_BLK, 0, st>>>(
      (const __nv_bfloat16*)qkv, ld_qkv, H, pe, L_total, segs, (__nv_bfloat16*)q, (__nv_bfloat16*)k, (__nv_bfloat16*)v);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                                const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q,
                                void* k, void* v, cudaStream_t st, const int* kv_pos) {
  QkSegs s = {};
  s.n = 1;
  s.s[0].row0 = 0;
  s.s[0].rows = M;
  s.s[0].pos0 = row_offset;
  s.s[0].off = 0;
  s.s[0].kv_pos = kv_pos;
  s.s[0].qs = q_scale;
  s.s[0].ks = k_scale;
  return launch_qk_norm_rope_segs(qkv, ld_qkv, H, pe, L_total, s, q, k, v, st);
}

// ------------------------------------------------------------------ K9
__global__ void k_euler(float* __restrict__ img, const float* __restrict__ pred, int64_t n, float dt,
                        const float* __restrict__ dt_dev) {
  const float d = dt_dev ? *dt_dev : dt;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    img[i] = img[i] + pred[i] * d;
}

cudaError_t launch_euler(float* img, const float* pred, int64_t n, float dt, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_euler<<<grid_cap((n + 255) / 256), 256, 0, st>>>(img, pred, n, dt, nullptr);
  return cudaGetLastError();
}
cudaError_t launch_euler_dev(float* img, const float* pred, int64_t n, const float* dt_dev, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_euler<<<grid_cap((n + 255) / 256), 256, 0, st>>>(img, pred, n, 0.f, dt_dev);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ RMSNorm rows
// y = x / sqrt(mean(x^2) + eps) * w (qwen_image/quantized_transformer.rs:96-108, txt_norm);
// one warp per row, row in registers (C <= 128 * VEC, C % 128 == 0).
template <int VEC>
__global__ void k_rms_norm(const float* __restrict__ x, int64_t M, int C, int64_t ldx, const float* __restrict__ w,
                           float eps, __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = C / 128;
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
    const float* xr = x + row * ldx;
    float4 v[VEC];
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      if (i < nvec) {
        v[i] = *(const float4*)(xr + (i * 32 + lane) * 4);
        q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
      }
    }
    const float r = 1.f / sqrtf(warp_sum(q) / (float)C + eps);
    __nv_bfloat16* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      if (i < nvec) {
        const int c = (i * 32 + lane) * 4;
        const float4 g = *(const float4*)(w + c);
        uint2 u;
        u.x = pack_bf16x2(v[i].x * r * g.x, v[i].y * r * g.y);
        u.y = pack_bf16x2(v[i].z * r * g.z, v[i].w * r * g.w);
        *(uint2*)(yr + c) = u;
      }
    }
  }
}

cudaError_t launch_rms_norm(const float* x, int64_t M, int64_t C, int64_t ldx, const float* w, float eps, void* y,
                            int64_t ldy, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (C % 128 != 0 || C > 8192) return cudaErrorInvalidValue;
  const int g = grid_cap((M + 7) / 8);
  __nv_bfloat16* yb = (__nv_bfloat16*)y;
  if (C <= 4096)
    k_rms_norm<32><<<g, 256, 0, st>>>(x, M, (int)C, ldx, w, eps, yb, ldy);
  else
    k_rms_norm<64><<<g, 256, 0, st>>>(x, M, (int)C, ldx, w, eps, yb, ldy);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ CFG + Euler
// Packed latents [n_tok, C * pp] (feature = c * pp + j, j the pixel inside the patch).
// Per pixel: comb = u + g (c - u); pred = comb * ||c|| / max(||comb||, 1e-8) over the C
// channels (qwen_image/pipeline.rs:2693-2698); img += pred * dt (qwen_image/sampling.rs:117-129).
__global__ void k_cfg_euler(float* __restrict__ img, const float* __restrict__ cond, const float* __restrict__ unc,
                            int64_t n_pix, int C, int pp, float g, float dt, const float* __restrict__ dt_dev) {
  const float d = dt_dev ? *dt_dev : dt;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n_pix; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = u / pp;
    const int j = (int)(u % pp);
    const int64_t base = tok * (int64_t)C * pp + j;
    float cn = 0.f, bn = 0.f;
    for (int c = 0; c < C; c++) {
      const float cv = cond[base + (int64_t)c * pp], uv = unc[base + (int64_t)c * pp];
      const float b = uv + g * (cv - uv);
      cn += cv * cv;
      bn += b * b;
    }
    const float f = sqrtf(cn) / fmaxf(sqrtf(bn), 1e-8f);
    for (int c = 0; c < C; c++) {
      const int64_t i = base + (int64_t)c * pp;
      const float cv = cond[i], uv = unc[i];
      img[i] = img[i] + (uv + g * (cv - uv)) * f * d;
    }
  }
}

cudaError_t launch_cfg_euler(float* img, const float* cond, const float* uncond, int64_t n_tok, int C, int pp,
                             float guidance, float dt, const float* dt_dev, cudaStream_t st) {
  const int64_t n = n_tok * pp;
  if (n <= 0) return cudaSuccess;
  k_cfg_euler<<<grid_cap((n + 255) / 256), 256, 0, st>>>(img, cond, uncond, n, C, pp, guidance, dt, dt_dev);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ timestep embedding
// out[i] = cos(t*1000*f_i) (i < dim/2), sin(...) after; f_i = exp(-ln(10000) i / (dim/2))
// (flux/offload.rs:21-38). t is read from device memory so the step graph can replay it.
__global__ void k_temb(const float* __restrict__ t_dev, float scale, float* __restrict__ out, int dim) {
  const int half = dim / 2;
  const float t = *t_dev * scale;
  const float c = -logf(10000.f) / (float)half;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = expf((float)i * c);
    const float a = t * f;
    out[i] = cosf(a);
    out[i + half] = sinf(a);
  }
}

cudaError_t launch_timestep_embedding(const float* t_dev, float scale, float* out, int dim, cudaStream_t st) {
  k_temb<<<1, 128, 0, st>>>(t_dev, scale, out, dim);
  return cudaGetLastError();
}

}  // namespace mb
