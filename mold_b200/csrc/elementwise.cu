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
// y = LN(x) * (1 + scale) + shift, LN without affine, eps 1e-6 (flux/offload.rs:286-295).
// One warp per row; the row stays in registers (C <= 32*4*VEC).
template <int VEC>
__global__ void k_ln_modulate(const float* __restrict__ x, int64_t M, int C, int64_t ldx,
                              const float* __restrict__ shift, const float* __restrict__ scale,
                              __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = C / 128;  // float4 per lane actually used (<= VEC)
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
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
        const float4 sc = *(const float4*)(scale + c), sh = *(const float4*)(shift + c);
        const float o0 = (v[i].x - mean) * rstd * (1.f + sc.x) + sh.x;
        const float o1 = (v[i].y - mean) * rstd * (1.f + sc.y) + sh.y;
        const float o2 = (v[i].z - mean) * rstd * (1.f + sc.z) + sh.z;
        const float o3 = (v[i].w - mean) * rstd * (1.f + sc.w) + sh.w;
        uint2 u;
        u.x = pack_bf16x2(o0, o1);
        u.y = pack_bf16x2(o2, o3);
        *(uint2*)(yr + c) = u;
      }
    }
  }
}

cudaError_t launch_ln_modulate(const float* x, int64_t M, int64_t C, int64_t ldx, const float* shift,
                               const float* scale, void* y, int64_t ldy, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  const int threads = 256;
  const int g = grid_cap((M + 7) / 8);
  __nv_bfloat16* yb = (__nv_bfloat16*)y;
  if (C <= 3072)
    k_ln_modulate<24><<<g, threads, 0, st>>>(x, M, (int)C, ldx, shift, scale, yb, ldy);
  else
    k_ln_modulate<64><<<g, threads, 0, st>>>(x, M, (int)C, ldx, shift, scale, yb, ldy);
  return cudaGetLastError();
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
// qkv row block [M, 3*H*128] bf16 -> RMSNorm(q), RMSNorm(k) (eps 1e-6, learned scale),
// RoPE on interleaved pairs, v copied; outputs [H, L_total, 128] bf16 at rows row_offset+.
// One warp per (row, head); lane holds 4 consecutive features (two rope pairs).
__global__ void k_qk_norm_rope(const __nv_bfloat16* __restrict__ qkv, int64_t M, int64_t ld, int H,
                               const float* __restrict__ qs, const float* __restrict__ ks,
                               const float* __restrict__ pe, int64_t row_off, int64_t L_total,
                               __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                               __nv_bfloat16* __restrict__ v, const int* __restrict__ kv_pos) {
  const int lane = threadIdx.x & 31;
  const int64_t total = M * H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const float4 qsc = *(const float4*)(qs + lane * 4);
  const float4 ksc = *(const float4*)(ks + lane * 4);
  for (int64_t u = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); u < total; u += warps) {
    const int64_t row = u / H;
    const int h = (int)(u % H);
    const __nv_bfloat16* src = qkv + row * ld + h * 128 + lane * 4;
    const uint2 rq = *(const uint2*)(src);
    const uint2 rk = *(const uint2*)(src + (int64_t)H * 128);
    const uint2 rv = *(const uint2*)(src + (int64_t)2 * H * 128);
    const int64_t prow = row_off + row;
    const float4* per = (const float4*)(pe + prow * 256);
    const float4 p0 = per[lane * 2], p1 = per[lane * 2 + 1];
    const int64_t dst = ((int64_t)h * L_total + prow) * 128 + lane * 4;
    const int64_t dkv = kv_pos ? ((int64_t)h * L_total + kv_pos[prow]) * 128 + lane * 4 : dst;
#pragma unroll
    for (int which = 0; which < 2; which++) {
      const uint2 r = which ? rk : rq;
      const float4 sc = which ? ksc : qsc;
      float x0 = bf16_lo(r.x), x1 = bf16_hi(r.x), x2 = bf16_lo(r.y), x3 = bf16_hi(r.y);
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
        *(uint2*)(k + dkv) = o;
      else
        *(uint2*)(q + dst) = o;
    }
    *(uint2*)(v + dkv) = rv;
  }
}

cudaError_t launch_qk_norm_rope(const void* qkv, int64_t M, int64_t ld_qkv, int H, const float* q_scale,
                                const float* k_scale, const float* pe, int64_t row_offset, int64_t L_total, void* q,
                                void* k, void* v, cudaStream_t st, const int* kv_pos) {
  if (M <= 0) return cudaSuccess;
  k_qk_norm_rope<<<grid_cap((M * H + 7) / 8), 256, 0, st>>>(
      (const __nv_bfloat16*)qkv, M, ld_qkv, H, q_scale, k_scale, pe, row_offset, L_total, (__nv_bfloat16*)q,
      (__nv_bfloat16*)k, (__nv_bfloat16*)v, kv_pos);
  return cudaGetLastError();
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
