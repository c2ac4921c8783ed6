// LoRA merge into GGUF weights on the device (flux/lora.rs:651-868, `gguf_lora_var_builder`):
// rows [row0, row0 + nrows) of a weight become requantize(dequant(W) + scale * (B A)), in the
// weight's own GGML type, so a patched tensor keeps its size.
//
// One thread per 256-value chunk of a row (partial chunk at the end of rows that are not a
// multiple of 256: F32 / F16 / BF16 and the 32-value block types). Per value:
//   d = fl(fl(sum_k B[r,k] A[k,c]) * scale)  (the sum by fmaf in ascending k), t = fl(w + d).
// Requantization per block:
//   Q8_0  ggml's reference quantizer: d = amax / 127, q = roundf(x / d) (half away from zero),
//         via x * (1/d) as ggml computes it
//   Q4_0 / Q5_0  ggml's reference quantizer: d = (value of largest |x|) / -8 or -16,
//                q = min(qmax, trunc(x (1/d) + 8.5 or 16.5)) with the unrounded f32 d
//   Q4_1 / Q5_1  ggml's reference quantizer: d = (max - min) / 15 or 31,
//                q = min(qmax, trunc((x - min) (1/d) + 0.5)), the block stores f16 d and min
//   (the K types below are this project's own quantizers: one pass, no scale search)
//   Q4_K / Q5_K  per 32 values min/max -> scale (max - min) / 15 or 31 and min -min; f16 d and
//                dmin = the largest scale / min over 63; 6-bit sc = rint(scale / d), m = rint(min
//                / dmin); q = rint((x + dmin m) / (d sc)), clamped
//   Q6_K  per 16 values the signed absmax / -32; f16 d = largest |scale| / 127; int8
//         sc = rint(scale / d); q = rint(x / (d sc)) + 32, clamped to 0..63
//   F32 / F16 / BF16  stored with round-to-nearest-even
// (rint = round half to even; f16 and bf16 conversions round to nearest even.)
#include <cstring>

#include "common.cuh"
#include "ggml_decode.cuh"
#include "internal.h"

namespace mb {
namespace lora {

MB_DEV uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
MB_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
MB_DEV int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
MB_DEV int rinti(float v) { return __float2int_rn(v); }
MB_DEV void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

MB_DEV void q8_0_block(const float* x, uint8_t* o) {
  float amax = 0.f;
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
  const float d = __fdiv_rn(amax, 127.f);
  const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
  put16(o, f2h(d));
  for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)(int8_t)roundf(__fmul_rn(x[j], id));
}

MB_DEV void q4q5_block(const float* x, uint8_t* o, int bits, bool has_m) {
  const int qmax = (1 << bits) - 1;
  int q[32];
  if (has_m) {
    float mn = INFINITY, mx = -INFINITY;
    for (int j = 0; j < 32; j++) {
      mn = fminf(mn, x[j]);
      mx = fmaxf(mx, x[j]);
    }
    const float d = __fdiv_rn(__fsub_rn(mx, mn), (float)qmax);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    put16(o, f2h(d));
    put16(o + 2, f2h(mn));
    for (int j = 0; j < 32; j++) q[j] = clampi(__float2int_rz(__fadd_rn(__fmul_rn(__fsub_rn(x[j], mn), id), 0.5f)), 0, qmax);
  } else {
    float amax = 0.f, vmax = 0.f;
    for (int j = 0; j < 32; j++)
      if (fabsf(x[j]) > amax) {
        amax = fabsf(x[j]);
        vmax = x[j];
      }
    const int half = 1 << (bits - 1);
    const float d = __fdiv_rn(vmax, (float)(-half));
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    put16(o, f2h(d));
    for (int j = 0; j < 32; j++) q[j] = clampi(__float2int_rz(__fadd_rn(__fmul_rn(x[j], id), (float)half + 0.5f)), 0, qmax);
  }
  uint8_t* qs = o + (has_m ? 4 : 2);
  if (bits == 5) {
    uint32_t qh = 0;
    for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
    for (int b = 0; b < 4; b++) qs[b] = (uint8_t)(qh >> (8 * b));
    qs += 4;
  }
  for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
}

// Q4_K (bits 4) and Q5_K (bits 5) super-block of 256 values.
MB_DEV void qk_block(const float* x, uint8_t* o, int bits) {
  const float qmaxf = bits == 4 ? 15.f : 31.f;
  const int qmax = bits == 4 ? 15 : 31;
  float scale[8], mins[8], max_scale = 0.f, max_min = 0.f;
  for (int j = 0; j < 8; j++) {
    float mn = 0.f, mx = -INFINITY;
    for (int l = 0; l < 32; l++) {
      mn = fminf(mn, x[32 * j + l]);
      mx = fmaxf(mx, x[32 * j + l]);
    }
    if (mx < mn) mx = mn;
    scale[j] = __fdiv_rn(__fsub_rn(mx, mn), qmaxf);
    mins[j] = -mn;
    max_scale = fmaxf(max_scale, scale[j]);
    max_min = fmaxf(max_min, mins[j]);
  }
  const uint16_t dh = f2h(__fdiv_rn(max_scale, 63.f)), mh = f2h(__fdiv_rn(max_min, 63.f));
  const float d = h2f(dh), dmin = h2f(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = d > 0.f ? clampi(rinti(__fdiv_rn(scale[j], d)), 0, 63) : 0;
    m[j] = dmin > 0.f ? clampi(rinti(__fdiv_rn(mins[j], dmin)), 0, 63) : 0;
  }
  put16(o, dh);
  put16(o + 2, mh);
  uint8_t* s = o + 4;
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t* qh = o + 16;
  uint8_t* qs = o + (bits == 4 ? 16 : 48);
  if (bits == 5)
    for (int l = 0; l < 32; l++) qh[l] = 0;
  for (int g = 0; g < 4; g++) {
    for (int l = 0; l < 32; l++) {
      int q2[2];
      for (int h = 0; h < 2; h++) {
        const int j = 2 * g + h;
        const float dl = __fmul_rn(d, (float)sc[j]), ml = __fmul_rn(dmin, (float)m[j]);
        q2[h] = dl > 0.f ? clampi(rinti(__fdiv_rn(__fadd_rn(x[32 * j + l], ml), dl)), 0, qmax) : 0;
        if (bits == 5) qh[l] |= (uint8_t)(((q2[h] >> 4) & 1) << j);
      }
      qs[32 * g + l] = (uint8_t)((q2[0] & 0xF) | ((q2[1] & 0xF) << 4));
    }
  }
}

MB_DEV void q6_k_block(const float* x, uint8_t* o) {
  float sv[16], amax_all = 0.f;
  for (int j = 0; j < 16; j++) {
    float am = 0.f, vm = 0.f;
    for (int l = 0; l < 16; l++)
      if (fabsf(x[16 * j + l]) > am) {
        am = fabsf(x[16 * j + l]);
        vm = x[16 * j + l];
      }
    sv[j] = __fdiv_rn(vm, -32.f);
    if (fabsf(sv[j]) > amax_all) amax_all = fabsf(sv[j]);
  }
  const uint16_t dh = f2h(__fdiv_rn(amax_all, 127.f));
  const float d = h2f(dh);
  int8_t sc[16];
  uint8_t* ql = o;
  uint8_t* qhb = o + 128;
  for (int i = 0; i < 192; i++) o[i] = 0;
  for (int j = 0; j < 16; j++) sc[j] = (int8_t)(d > 0.f ? clampi(rinti(__fdiv_rn(sv[j], d)), -127, 127) : 0);
  auto q_of = [&](int i) -> int {  // quant of value i
    const int j = i >> 4;
    const float ds = __fmul_rn(d, (float)sc[j]);
    return ds != 0.f ? clampi(rinti(__fdiv_rn(x[i], ds)) + 32, 0, 63) : 32;
  };
  for (int n2 = 0; n2 < 2; n2++)
    for (int l = 0; l < 32; l++) {
      const int b = 128 * n2;
      const int q0 = q_of(b + l), q1 = q_of(b + l + 32), q2 = q_of(b + l + 64), q3 = q_of(b + l + 96);
      ql[64 * n2 + l] = (uint8_t)((q0 & 0xF) | ((q2 & 0xF) << 4));
      ql[64 * n2 + l + 32] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      qhb[32 * n2 + l] = (uint8_t)(((q0 >> 4) & 3) | (((q1 >> 4) & 3) << 2) | (((q2 >> 4) & 3) << 4) | (((q3 >> 4) & 3) << 6));
    }
  for (int j = 0; j < 16; j++) o[192 + j] = (uint8_t)sc[j];
  put16(o + 208, dh);
}

MB_DEV uint16_t bf16_rne(float f) {
  uint32_t x = __float_as_uint(f);
  x += 0x7FFFu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

template <int T>
__global__ void k_lora_merge(uint8_t* __restrict__ w, int64_t row_bytes, int64_t n_cols, int64_t row0, int64_t nrows,
                             const float* __restrict__ A, const float* __restrict__ B, int rank, float scale) {
  const int64_t n_chunks = (n_cols + 255) / 256;
  const int64_t total = nrows * n_chunks;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / n_chunks, kc = v % n_chunks;
    const int64_t c0 = kc * 256;
    const int len = (int)(n_cols - c0 < 256 ? n_cols - c0 : 256);
    uint8_t* row = w + (row0 + r) * row_bytes;
    float t[256];
    // dequantize the chunk
    if constexpr (T == MB_GGML_F32) {
      for (int i = 0; i < len; i++) t[i] = ((const float*)row)[c0 + i];
    } else if constexpr (T == MB_GGML_F16) {
      for (int i = 0; i < len; i++) t[i] = __half2float(((const __half*)row)[c0 + i]);
    } else if constexpr (T == MB_GGML_BF16) {
      for (int i = 0; i < len; i++) t[i] = __uint_as_float((uint32_t)((const uint16_t*)row)[c0 + i] << 16);
    } else {
      const uint8_t* chunk = row + kc * kDeviceChunk(T);
      for (int u = 0; u < len / 32; u++) {
        float y[32];
        decode_unit<T>(chunk, u, y);
        for (int i = 0; i < 32; i++) t[32 * u + i] = y[i];
      }
    }
    // add the low-rank delta
    for (int i = 0; i < len; i++) {
      float acc = 0.f;
      for (int k = 0; k < rank; k++) acc = fmaf(B[r * rank + k], A[(int64_t)k * n_cols + c0 + i], acc);
      t[i] = __fadd_rn(t[i], __fmul_rn(acc, scale));
    }
    // requantize into the weight's own type
    if constexpr (T == MB_GGML_F32) {
      for (int i = 0; i < len; i++) ((float*)row)[c0 + i] = t[i];
    } else if constexpr (T == MB_GGML_F16) {
      for (int i = 0; i < len; i++) ((uint16_t*)row)[c0 + i] = f2h(t[i]);
    } else if constexpr (T == MB_GGML_BF16) {
      for (int i = 0; i < len; i++) ((uint16_t*)row)[c0 + i] = bf16_rne(t[i]);
    } else {
      uint8_t* chunk = row + kc * kDeviceChunk(T);
      uint8_t ob[272];
      if constexpr (T == MB_GGML_Q8_0) {
        for (int b = 0; b < len / 32; b++) q8_0_block(t + 32 * b, ob + 34 * b);
      } else if constexpr (T == MB_GGML_Q4_0 || T == MB_GGML_Q4_1 || T == MB_GGML_Q5_0 || T == MB_GGML_Q5_1) {
        constexpr int bits = (T == MB_GGML_Q4_0 || T == MB_GGML_Q4_1) ? 4 : 5;
        constexpr bool has_m = T == MB_GGML_Q4_1 || T == MB_GGML_Q5_1;
        constexpr int bb = kDeviceChunk(T) / 8;
        for (int b = 0; b < len / 32; b++) q4q5_block(t + 32 * b, ob + bb * b, bits, has_m);
      } else if constexpr (T == MB_GGML_Q4_K) {
        qk_block(t, ob, 4);
      } else if constexpr (T == MB_GGML_Q5_K) {
        qk_block(t, ob, 5);
      } else {
        q6_k_block(t, ob);
      }
      // K types: one whole super-block (Q6_K's 14 padding bytes stay as they are); 32-value
      // block types: the blocks of this (possibly partial) chunk
      constexpr bool kSuper = T == MB_GGML_Q4_K || T == MB_GGML_Q5_K || T == MB_GGML_Q6_K;
      const int nb = T == MB_GGML_Q6_K ? 210 : (kSuper ? kDeviceChunk(T) : (len / 32) * (kDeviceChunk(T) / 8));
      for (int i = 0; i < nb; i++) chunk[i] = ob[i];
    }
  }
}

}  // namespace lora

cudaError_t launch_lora_merge(mb_weight* w, int64_t row0, int64_t nrows, const float* A, const float* B, int rank,
                              float scale, cudaStream_t st) {
  using namespace lora;
  const int64_t total = nrows * ((w->n_cols + 255) / 256);
  if (total <= 0) return cudaSuccess;
  const int T = 128;
  const int g = (int)((total + T - 1) / T < 65535 ? (total + T - 1) / T : 65535);
  uint8_t* d = (uint8_t*)w->dev;
#define MB_LORA_CASE(TT)                                                                                     \
  case TT:                                                                                                   \
    k_lora_merge<TT><<<g, T, 0, st>>>(d, w->row_bytes, w->n_cols, row0, nrows, A, B, rank, scale);           \
    break;
  switch (w->type) {
    MB_LORA_CASE(MB_GGML_F32)
    MB_LORA_CASE(MB_GGML_F16)
    MB_LORA_CASE(MB_GGML_BF16)
    MB_LORA_CASE(MB_GGML_Q8_0)
    MB_LORA_CASE(MB_GGML_Q4_0)
    MB_LORA_CASE(MB_GGML_Q4_1)
    MB_LORA_CASE(MB_GGML_Q5_0)
    MB_LORA_CASE(MB_GGML_Q5_1)
    MB_LORA_CASE(MB_GGML_Q4_K)
    MB_LORA_CASE(MB_GGML_Q5_K)
    MB_LORA_CASE(MB_GGML_Q6_K)
    default: return cudaErrorInvalidValue;
  }
#undef MB_LORA_CASE
  return cudaGetLastError();
}

}  // namespace mb

using namespace mb;

extern "C" mb_status mb_weight_lora_merge(mb_weight* w, int64_t row_offset, int64_t rows, const float* A,
                                          const float* B, int rank, float scale, void* stream) {
  MB_CHECK(w, MB_ERR_INVALID, "weight is NULL");
  MB_CHECK(rows >= 0 && row_offset >= 0 && row_offset + rows <= w->n_rows, MB_ERR_INVALID,
           "LoRA row slice [" + std::to_string(row_offset) + ", " + std::to_string(row_offset + rows) +
               ") is outside the weight's " + std::to_string(w->n_rows) + " rows");
  if (rows == 0) return MB_OK;
  MB_CHECK(A && B, MB_ERR_INVALID, "A or B is NULL");
  MB_CHECK(rank > 0 && rows >= 0 && row_offset >= 0 && row_offset + rows <= w->n_rows, MB_ERR_INVALID,
           "LoRA row slice [" + std::to_string(row_offset) + ", " + std::to_string(row_offset + rows) +
               ") is outside the weight's " + std::to_string(w->n_rows) + " rows");
  MB_CUDA(launch_lora_merge(w, row_offset, rows, A, B, rank, scale, (cudaStream_t)stream));
  return MB_OK;
}
