// K1: standalone GGML dequantization (QTensor::dequantize, qwen_image/quantized_transformer.rs:60-67)
// and the f32 -> bf16 activation cast used by mb_qlinear's f32-input path.
//
// HBM-bound. One thread decodes one 64-value Q4_K group (16-byte header + 32
// bytes of nibbles), one 32-value Q8_0 block, or one 32-value unit of the other
// chunked types (ggml_decode.cuh); stores are 16-byte vectors.
// Decode order follows the GGML formula with one rounding per operation
// (multiply, then subtract), so the f32 output is bit-identical to the CPU
// decode; the bf16 output is its round-to-nearest-even.
#include "common.cuh"
#include "ggml_decode.cuh"
#include "internal.h"

namespace mb {

// Any chunked type (decode_unit): one thread per 32-value unit. Unit u of a row is unit u % 8 of
// 256-value chunk u / 8 (for the 32-value block types that is simply block u, so rows only need
// a multiple of 32 values).
template <int T, bool BF16>
__global__ void k_dequant_units(const uint8_t* __restrict__ raw, int64_t n_rows, int64_t n_units, int64_t row_bytes,
                                void* __restrict__ out) {
  const int64_t total = n_rows * n_units;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = v / n_units, u = v % n_units;
    float y[32];
    decode_unit<T>(raw + row * row_bytes + (u >> 3) * kDeviceChunk(T), (int)(u & 7), y);
    const int64_t obase = v * 32;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      if (BF16) {
        uint4 w;
        w.x = pack_bf16x2(y[8 * c + 0], y[8 * c + 1]);
        w.y = pack_bf16x2(y[8 * c + 2], y[8 * c + 3]);
        w.z = pack_bf16x2(y[8 * c + 4], y[8 * c + 5]);
        w.w = pack_bf16x2(y[8 * c + 6], y[8 * c + 7]);
        *(uint4*)((__nv_bfloat16*)out + obase + 8 * c) = w;
      } else {
        float4* o = (float4*)((float*)out + obase + 8 * c);
        o[0] = make_float4(y[8 * c + 0], y[8 * c + 1], y[8 * c + 2], y[8 * c + 3]);
        o[1] = make_float4(y[8 * c + 4], y[8 * c + 5], y[8 * c + 6], y[8 * c + 7]);
      }
    }
  }
}

// Q6_K super-blocks 210 B (GGUF) -> 224 B (device layout, zero padding), one thread per 16 bytes.
__global__ void k_relayout_q6k(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t n_sb) {
  const int64_t total = n_sb * 14;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sb = v / 14;
    const int part = (int)(v % 14);
    uint8_t b[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const int o = part * 16 + i;
      b[i] = o < 210 ? in[sb * 210 + o] : 0;
    }
    uint4 w;
    memcpy(&w, b, 16);
    *(uint4*)(out + sb * 224 + part * 16) = w;
  }
}

MB_DEV float h2f_bits(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }

template <bool BF16>
MB_DEV void store8(void* out, int64_t idx, const float (&v)[8]) {
  if (BF16) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *(uint4*)((__nv_bfloat16*)out + idx) = u;
  } else {
    float4* o = (float4*)((float*)out + idx);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <bool BF16>
__global__ void k_dequant_q4k(const uint8_t* __restrict__ raw, int64_t n_rows, int64_t nsb, int64_t row_bytes,
                              void* __restrict__ out) {
  const int64_t total = n_rows * nsb * 4;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(u & 3);
    const int64_t sbi = u >> 2;
    const int64_t row = sbi / nsb, kb = sbi % nsb;
    const uint8_t* b = raw + row * row_bytes + kb * 144;
    const uint4 h = *(const uint4*)b;
    const uint4 qa = *(const uint4*)(b + 16 + 32 * g), qb = *(const uint4*)(b + 32 + 32 * g);
    const float d = h2f_bits(h.x), dmin = h2f_bits(h.x >> 16);
    const uint8_t* s = b + 4;
    int sc0, m0, sc1, m1;
    const int j0 = 2 * g, j1 = 2 * g + 1;
    if (j0 < 4) { sc0 = s[j0] & 63; m0 = s[j0 + 4] & 63; }
    else { sc0 = (s[j0 + 4] & 0xF) | ((s[j0 - 4] >> 6) << 4); m0 = (s[j0 + 4] >> 4) | ((s[j0] >> 6) << 4); }
    if (j1 < 4) { sc1 = s[j1] & 63; m1 = s[j1 + 4] & 63; }
    else { sc1 = (s[j1 + 4] & 0xF) | ((s[j1 - 4] >> 6) << 4); m1 = (s[j1 + 4] >> 4) | ((s[j1] >> 6) << 4); }
    const float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
    const float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int64_t obase = row * nsb * 256 + kb * 256 + g * 64;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      float lo[8], hi[8];
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const uint32_t byte = (w[2 * c + (t >> 2)] >> (8 * (t & 3))) & 0xFFu;
        lo[t] = __fsub_rn(__fmul_rn(d1, (float)(byte & 0xF)), mm1);
        hi[t] = __fsub_rn(__fmul_rn(d2, (float)(byte >> 4)), mm2);
      }
      store8<BF16>(out, obase + 8 * c, lo);
      store8<BF16>(out, obase + 32 + 8 * c, hi);
    }
  }
}

template <bool BF16>
__global__ void k_dequant_q8_0(const uint8_t* __restrict__ raw, int64_t n_rows, int64_t nb, int64_t row_bytes,
                               void* __restrict__ out) {
  const int64_t total = n_rows * nb;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = u / nb, kb = u % nb;
    const uint8_t* b = raw + row * row_bytes + kb * 34;
    const float d = h2f_bits((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    const int8_t* q = (const int8_t*)(b + 2);
    const int64_t obase = row * nb * 32 + kb * 32;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      float v[8];
#pragma unroll
      for (int t = 0; t < 8; t++) v[t] = __fmul_rn((float)q[8 * c + t], d);
      store8<BF16>(out, obase + 8 * c, v);
    }
  }
}

// F32 / F16 / BF16 weights: plain element conversion.
template <int T, bool BF16>
__global__ void k_convert(const void* __restrict__ in, int64_t n, void* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v;
    if (T == MB_GGML_F32) v = ((const float*)in)[i];
    else if (T == MB_GGML_F16) v = __half2float(((const __half*)in)[i]);
    else v = __uint_as_float((uint32_t)((const uint16_t*)in)[i] << 16);
    if (BF16) ((__nv_bfloat16*)out)[i] = __float2bfloat16_rn(v);
    else ((float*)out)[i] = v;
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 16;
  return (int)(g < cap ? (g > 0 ? g : 1) : cap);
}

cudaError_t launch_dequant(int type, const void* raw, int64_t n_rows, int64_t n_cols, int64_t row_bytes, void* out,
                           int out_bf16, cudaStream_t st) {
  const int T = 256;
  const uint8_t* r = (const uint8_t*)raw;
  const int64_t n = n_rows * n_cols;
  switch (type) {
    case MB_GGML_Q4_K: {
      const int64_t nsb = n_cols / 256;
      const int g = grid_for(n_rows * nsb * 4, T);
      if (out_bf16) k_dequant_q4k<true><<<g, T, 0, st>>>(r, n_rows, nsb, row_bytes, out);
      else k_dequant_q4k<false><<<g, T, 0, st>>>(r, n_rows, nsb, row_bytes, out);
      break;
    }
    case MB_GGML_Q8_0: {
      const int64_t nb = n_cols / 32;
      const int g = grid_for(n_rows * nb, T);
      if (out_bf16) k_dequant_q8_0<true><<<g, T, 0, st>>>(r, n_rows, nb, row_bytes, out);
      else k_dequant_q8_0<false><<<g, T, 0, st>>>(r, n_rows, nb, row_bytes, out);
      break;
    }
#define MB_UNITS_CASE(TT)                                                                          \
    case TT: {                                                                                     \
      const int64_t nu = n_cols / 32;                                                              \
      const int g = grid_for(n_rows * nu, T);                                                      \
      if (out_bf16) k_dequant_units<TT, true><<<g, T, 0, st>>>(r, n_rows, nu, row_bytes, out);     \
      else k_dequant_units<TT, false><<<g, T, 0, st>>>(r, n_rows, nu, row_bytes, out);             \
      break;                                                                                       \
    }
    MB_UNITS_CASE(MB_GGML_Q4_0)
    MB_UNITS_CASE(MB_GGML_Q4_1)
    MB_UNITS_CASE(MB_GGML_Q5_0)
    MB_UNITS_CASE(MB_GGML_Q5_1)
    MB_UNITS_CASE(MB_GGML_Q5_K)
    MB_UNITS_CASE(MB_GGML_Q6_K)
#undef MB_UNITS_CASE
    case MB_GGML_F32:
      if (out_bf16) k_convert<MB_GGML_F32, true><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      else k_convert<MB_GGML_F32, false><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      break;
    case MB_GGML_F16:
      if (out_bf16) k_convert<MB_GGML_F16, true><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      else k_convert<MB_GGML_F16, false><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      break;
    case MB_GGML_BF16:
      if (out_bf16) k_convert<MB_GGML_BF16, true><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      else k_convert<MB_GGML_BF16, false><<<grid_for(n, T), T, 0, st>>>(raw, n, out);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_relayout_q6k(const void* in, void* out, int64_t n_superblocks, cudaStream_t st) {
  if (n_superblocks <= 0) return cudaSuccess;
  k_relayout_q6k<<<grid_for(n_superblocks * 14, 256), 256, 0, st>>>((const uint8_t*)in, (uint8_t*)out, n_superblocks);
  return cudaGetLastError();
}

// x f32 [M, K] (row stride ldx) -> y bf16 [M, K] (row stride ldy); K % 4 == 0.
__global__ void k_cast_f32_bf16(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
                                __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int64_t kq = K / 4, total = M * kq;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / kq, k = (i % kq) * 4;
    const float4 v = *(const float4*)(x + m * ldx + k);
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *(uint2*)(y + m * ldy + k) = o;
  }
}

cudaError_t launch_cast_f32_bf16(const float* x, int64_t M, int64_t K, int64_t ldx, void* y, int64_t ldy,
                                 cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  k_cast_f32_bf16<<<grid_for(M * K / 4, 256), 256, 0, st>>>(x, M, K, ldx, (__nv_bfloat16*)y, ldy);
  return cudaGetLastError();
}

}  // namespace mb
