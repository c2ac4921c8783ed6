// Device decode of GGML quantized rows, shared by the dequant, GEMV and GEMM kernels.
//
// A row is processed in chunks of 256 values. In device memory every supported type's chunk is
// a multiple of 16 bytes, so chunk c of a row starts 16-byte aligned (TMA boxes need that):
//   Q4_0  8 blocks x 18 B = 144      Q4_1  8 x 20 = 160     Q5_0  8 x 22 = 176
//   Q5_1  8 x 24 = 192               Q8_0  8 x 34 = 272     Q4_K  144   Q5_K  176
//   Q6_K  210 B + 14 B padding = 224 (super-blocks are re-laid at upload; see kDeviceChunk)
// decode_unit<T>(chunk, u, y) writes values [32u, 32u + 32) of the chunk as f32, each exactly
// GGML's value: every scale x quant product here is exact in f32 (at most 24 significant
// bits), so each value is a single rounding of the exact result.
//
// Block formats (the published GGML layouts):
//   Q4_0  f16 d, u8 qs[16]                 x_j = d (q_j - 8)
//   Q4_1  f16 d, f16 m, u8 qs[16]          x_j = d q_j + m
//   Q5_0  f16 d, u32 qh, u8 qs[16]         x_j = d (q5_j - 16)
//   Q5_1  f16 d, f16 m, u32 qh, u8 qs[16]  x_j = d q5_j + m
//         (j < 16: low nibble of qs[j], fifth bit = qh bit j; j >= 16: high nibble of
//          qs[j - 16], fifth bit = qh bit j)
//   Q8_0  f16 d, i8 qs[32]                 x_j = d q_j
//   Q4_K  f16 d, f16 dmin, u8 scales[12] (6-bit scale / min per 32 values), u8 qs[128]
//   Q5_K  as Q4_K plus u8 qh[32] before qs: fifth bit of value 64g + 32h + l = qh[l] bit 2g + h
//   Q6_K  u8 ql[128], u8 qh[64], i8 scales[16], f16 d; value 128n + 32g + l (g = 0..3) =
//         (d sc[8n + 2g + l/16]) (q6 - 32) with q6 = nibble (g >> 1) of ql[64n + 32(g & 1) + l]
//         | two bits (2g) of qh[32n + l] << 4
#pragma once
#include "../../include/mold_b200.h"
#include "common.cuh"

namespace mb {

// Bytes of one 256-value chunk in device memory (0: type not chunked / unsupported).
__host__ __device__ constexpr int kDeviceChunk(int t) {
  return t == MB_GGML_Q4_0   ? 144
         : t == MB_GGML_Q4_1 ? 160
         : t == MB_GGML_Q5_0 ? 176
         : t == MB_GGML_Q5_1 ? 192
         : t == MB_GGML_Q8_0 ? 272
         : t == MB_GGML_Q4_K ? 144
         : t == MB_GGML_Q5_K ? 176
         : t == MB_GGML_Q6_K ? 224
                             : 0;
}

namespace dec {

MB_DEV float f16(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }

// NW 32-bit words starting at byte address p (p even): aligned word loads plus a 16-bit shift.
template <int NW>
MB_DEV void words(const uint8_t* p, uint32_t (&w)[NW]) {
  const uint32_t* a = (const uint32_t*)((uintptr_t)p & ~(uintptr_t)3);
  if (((uintptr_t)p & 2) == 0) {
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = a[i];
  } else {
    uint32_t prev = a[0];
#pragma unroll
    for (int i = 0; i < NW; i++) {
      const uint32_t next = a[i + 1];
      w[i] = __byte_perm(prev, next, 0x5432);
      prev = next;
    }
  }
}

// 6-bit scale / min j of the 12-byte Q4_K / Q5_K scale field (words s0, s1, s2).
MB_DEV void scale_min_k4(int j, uint32_t s0, uint32_t s1, uint32_t s2, int& sc, int& m) {
  auto byte = [&](int k) -> uint32_t { return ((k < 4 ? s0 : (k < 8 ? s1 : s2)) >> ((k & 3) * 8)) & 0xFFu; };
  if (j < 4) {
    sc = byte(j) & 63;
    m = byte(j + 4) & 63;
  } else {
    sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
    m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
  }
}

}  // namespace dec

template <int T>
MB_DEV void decode_unit(const uint8_t* __restrict__ c, int u, float (&y)[32]);

template <>
MB_DEV void decode_unit<MB_GGML_Q4_0>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  uint32_t w[5];  // d, qs[16] (18 bytes from an even address): byte i at w[i >> 2] >> 8(i & 3)
  dec::words<5>(c + u * 18, w);
  const float d = dec::f16(w[0]);
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const int i = 2 + k;
    const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
    y[k] = (float)((int)(byte & 0xF) - 8) * d;
    y[k + 16] = (float)((int)(byte >> 4) - 8) * d;
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q4_1>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  const uint32_t* a = (const uint32_t*)(c + u * 20);  // 4-byte aligned
  const uint32_t h = a[0];
  const float d = dec::f16(h), m = dec::f16(h >> 16);
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const uint32_t byte = (a[1 + (k >> 2)] >> (8 * (k & 3))) & 0xFFu;
    y[k] = fmaf((float)(byte & 0xF), d, m);
    y[k + 16] = fmaf((float)(byte >> 4), d, m);
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q5_0>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  uint32_t w[6];  // d, qh, qs[16] (22 bytes from an even address): byte i at w[i >> 2] >> 8(i & 3)
  dec::words<6>(c + u * 22, w);
  const float d = dec::f16(w[0]);
  const uint32_t qh = (w[0] >> 16) | (w[1] << 16);
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const int i = 6 + k;
    const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
    const int q0 = (int)((byte & 0xF) | (((qh >> k) & 1u) << 4));
    const int q1 = (int)((byte >> 4) | (((qh >> (k + 16)) & 1u) << 4));
    y[k] = (float)(q0 - 16) * d;
    y[k + 16] = (float)(q1 - 16) * d;
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q5_1>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  const uint32_t* a = (const uint32_t*)(c + u * 24);  // 8-byte aligned
  const float d = dec::f16(a[0]), m = dec::f16(a[0] >> 16);
  const uint32_t qh = a[1];
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const uint32_t byte = (a[2 + (k >> 2)] >> (8 * (k & 3))) & 0xFFu;
    const uint32_t q0 = (byte & 0xF) | (((qh >> k) & 1u) << 4);
    const uint32_t q1 = (byte >> 4) | (((qh >> (k + 16)) & 1u) << 4);
    y[k] = fmaf((float)q0, d, m);
    y[k + 16] = fmaf((float)q1, d, m);
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q8_0>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  uint32_t w[9];  // d + qs[32] (34 bytes from an even address)
  dec::words<9>(c + u * 34, w);
  const float d = dec::f16(w[0]);
#pragma unroll
  for (int k = 0; k < 32; k++) {
    const int i = 2 + k;
    const int8_t q = (int8_t)((w[i >> 2] >> (8 * (i & 3))) & 0xFFu);
    y[k] = (float)q * d;
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q4_K>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  const uint4 h = *(const uint4*)c;
  const float d = dec::f16(h.x), dmin = dec::f16(h.x >> 16);
  int sc, m;
  dec::scale_min_k4(u, h.y, h.z, h.w, sc, m);
  const float d1 = d * (float)sc, m1 = dmin * (float)m;
  const uint32_t* qs = (const uint32_t*)(c + 16 + 32 * (u >> 1));
  const int sh = (u & 1) * 4;
#pragma unroll
  for (int k = 0; k < 32; k++) {
    const uint32_t q = (qs[k >> 2] >> (8 * (k & 3) + sh)) & 0xFu;
    y[k] = fmaf(d1, (float)q, -m1);
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q5_K>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  const uint4 h = *(const uint4*)c;
  const float d = dec::f16(h.x), dmin = dec::f16(h.x >> 16);
  int sc, m;
  dec::scale_min_k4(u, h.y, h.z, h.w, sc, m);
  const float d1 = d * (float)sc, m1 = dmin * (float)m;
  const uint32_t* qh = (const uint32_t*)(c + 16);
  const uint32_t* qs = (const uint32_t*)(c + 48 + 32 * (u >> 1));
  const int sh = (u & 1) * 4;
#pragma unroll
  for (int k = 0; k < 32; k++) {
    const uint32_t lo = (qs[k >> 2] >> (8 * (k & 3) + sh)) & 0xFu;
    const uint32_t hb = (qh[k >> 2] >> (8 * (k & 3) + u)) & 1u;
    y[k] = fmaf(d1, (float)(lo | (hb << 4)), -m1);
  }
}

template <>
MB_DEV void decode_unit<MB_GGML_Q6_K>(const uint8_t* __restrict__ c, int u, float (&y)[32]) {
  const int n = u >> 2, g = u & 3;
  const uint32_t* ql = (const uint32_t*)(c + 64 * n + 32 * (g & 1));
  const uint32_t* qh = (const uint32_t*)(c + 128 + 32 * n);
  const int8_t* sc = (const int8_t*)(c + 192 + 8 * n + 2 * g);
  const float d = dec::f16(*(const uint16_t*)(c + 208));
  const float ds0 = d * (float)sc[0], ds1 = d * (float)sc[1];
  const int nsh = (g >> 1) * 4, hsh = 2 * g;
#pragma unroll
  for (int k = 0; k < 32; k++) {
    const uint32_t lo = (ql[k >> 2] >> (8 * (k & 3) + nsh)) & 0xFu;
    const uint32_t hi = (qh[k >> 2] >> (8 * (k & 3) + hsh)) & 3u;
    const int q = (int)(lo | (hi << 4)) - 32;
    y[k] = (k < 16 ? ds0 : ds1) * (float)q;
  }
}

}  // namespace mb
