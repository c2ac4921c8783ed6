/*
 * mold-b200 CPU ORACLE — TEST INFRASTRUCTURE ONLY.
 *
 * Nothing in the product path (mold_b200/, include/, the CUDA library) may
 * call, link or load this file. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py use it, and only as the checker.
 *
 * What it restates (reference = utensils/mold, third-party arithmetic pinned in
 * its Cargo.lock):
 *   - GGML block codecs used by candle-core-mold 0.9.10 `QTensor::dequantize`
 *     (called from crates/mold-inference/src/qwen_image/quantized_transformer.rs:60-67
 *     and inside `QMatMul` for FLUX, flux/transformer.rs:64-72). The published
 *     GGML block formats:
 *       Q8_0 : 34 bytes / 32 values  = f16 d, int8 q[32];            x = d*q
 *       Q4_K : 144 bytes / 256 values = f16 d, f16 dmin, u8 scales[12] (packed
 *              6-bit scale/min per 32-value sub-block), u8 qs[128] (nibbles);
 *              x = (d*sc)*q - (dmin*m), multiply then subtract (candle's Rust
 *              code does not contract to FMA).
 *     Pinned: bit-exact against the `gguf` 0.19.0 Python package
 *     (gguf/quants.py Q8_0.quantize_blocks/dequantize_blocks, Q4_K.dequantize_blocks);
 *     fixtures in tests/golden/ with the script that produced them.
 *       Q4_0 : 18 bytes / 32 values  = f16 d, u8 qs[16];                x = d*(q-8)
 *       Q4_1 : 20 bytes / 32 values  = f16 d, f16 m, u8 qs[16];         x = d*q + m
 *       Q5_0 : 22 bytes / 32 values  = f16 d, u32 qh, u8 qs[16];        x = d*(q5-16)
 *       Q5_1 : 24 bytes / 32 values  = f16 d, f16 m, u32 qh, u8 qs[16]; x = d*q5 + m
 *              (value j < 16: low nibble of qs[j], high bit = bit j of qh; value j + 16:
 *              high nibble of qs[j], high bit = bit j + 16 of qh)
 *       Q5_K : 176 bytes / 256 values = f16 d, f16 dmin, u8 scales[12] (as Q4_K),
 *              u8 qh[32], u8 qs[128]; x = (d*sc)*q5 - (dmin*m)
 *       Q6_K : 210 bytes / 256 values = u8 ql[128], u8 qh[64], int8 scales[16], f16 d;
 *              x = (d*sc)*(q6-32)
 *     Every product above is exact in f32 (at most 24 significant bits), so each value is
 *     one rounding of the exact result and does not depend on the evaluation order.
 *   - A Q8_0 quantizer equal to ggml's reference quantizer (amax/127, round half
 *     away from zero), pinned against gguf-py's Q8_0.quantize_blocks.
 *   - ggml's reference quantizers for Q4_0/Q4_1/Q5_0/Q5_1 (pinned against gguf-py), and
 *     quantizers of this project's own for Q5_K/Q6_K (any valid block exercises the same
 *     decode; the decode is what must be bit-exact).
 *   - A Q4_K quantizer of this project's own (per-sub-block min/max, 6-bit
 *     scales relative to the super-block maxima). Any valid Q4_K block
 *     exercises the same decode; only the decode is required to be bit-exact.
 *   - The shared seeded generator (splitmix64 counter hash + Box-Muller) used
 *     for every synthetic tensor in tests and in the CPU baseline.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK8_0 32
#define QK_K 256
#define Q8_0_BYTES 34
#define Q4_K_BYTES 144

/* ---------- IEEE half <-> single (own implementation, RNE) ---------- */
static float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400));
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint16_t sign = (x >> 16) & 0x8000;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0);
  if (ax >= 0x477ff000u) return sign | 0x7c00; /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                      /* result subnormal or zero */
    if (ax < 0x33000000u) return sign;         /* < 2^-25 rounds to 0 */
    uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
    int shift = 126 - (int)e;                  /* 14 + (113 - e) ... */
    shift = (int)(113 - e) + 13;
    uint32_t r = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1))) r++;
    return sign | (uint16_t)r;
  }
  uint32_t r = ((ax >> 13) - (112u << 10));
  uint32_t rem = ax & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r++;
  return sign | (uint16_t)r;
}

void or_f16_to_f32(const uint16_t* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = h2f(in[i]);
}
void or_f32_to_f16(const float* in, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = f2h(in[i]);
}
/* bf16 round-to-nearest-even, returned as f32 values (NaN kept quiet). */
void or_round_bf16(const float* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) {
    uint32_t x;
    memcpy(&x, &in[i], 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) {
      x |= 0x00400000u;
    } else {
      x += 0x7fffu + ((x >> 16) & 1u);
    }
    x &= 0xffff0000u;
    memcpy(&out[i], &x, 4);
  }
}

/* ---------- Q8_0 ---------- */
static float roundf_away(float v) { /* ggml's roundf: half away from zero */
  return roundf(v);
}

void or_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / QK8_0;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const float* xb = x + b * QK8_0;
    uint8_t* ob = out + b * Q8_0_BYTES;
    float amax = 0.f;
    for (int j = 0; j < QK8_0; j++) amax = fmaxf(amax, fabsf(xb[j]));
    float d = amax / 127.f;
    float id = d != 0.f ? 1.0f / d : 0.f;
    uint16_t dh = f2h(d);
    memcpy(ob, &dh, 2);
    for (int j = 0; j < QK8_0; j++) ((int8_t*)(ob + 2))[j] = (int8_t)roundf_away(xb[j] * id);
  }
}

static void dequant_q8_0(const uint8_t* in, int64_t nb, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * Q8_0_BYTES;
    uint16_t dh;
    memcpy(&dh, ib, 2);
    float d = h2f(dh);
    const int8_t* q = (const int8_t*)(ib + 2);
    for (int j = 0; j < QK8_0; j++) out[b * QK8_0 + j] = (float)q[j] * d;
  }
}

/* ---------- Q4_K ---------- */
static void q4k_scale_min(int j, const uint8_t* s, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void or_quantize_q4_k(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / QK_K;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const float* xb = x + b * QK_K;
    uint8_t* ob = out + b * Q4_K_BYTES;
    float scale[8], mins[8];
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
      float mn = 0.f, mx = -INFINITY;
      for (int l = 0; l < 32; l++) {
        float v = xb[32 * j + l];
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
      if (mx < mn) mx = mn;
      scale[j] = (mx - mn) / 15.f;
      mins[j] = -mn;
      max_scale = fmaxf(max_scale, scale[j]);
      max_min = fmaxf(max_min, mins[j]);
    }
    uint16_t dh = f2h(max_scale / 63.f), mh = f2h(max_min / 63.f);
    float d = h2f(dh), dmin = h2f(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
      sc[j] = d > 0.f ? clampi((int)lrintf(scale[j] / d), 0, 63) : 0;
      m[j] = dmin > 0.f ? clampi((int)lrintf(mins[j] / dmin), 0, 63) : 0;
    }
    memcpy(ob, &dh, 2);
    memcpy(ob + 2, &mh, 2);
    uint8_t* s = ob + 4;
    for (int j = 0; j < 4; j++) {
      s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
      s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t q[QK_K];
    for (int j = 0; j < 8; j++) {
      float dl = d * (float)sc[j], ml = dmin * (float)m[j];
      for (int l = 0; l < 32; l++) {
        int v = dl > 0.f ? (int)lrintf((xb[32 * j + l] + ml) / dl) : 0;
        q[32 * j + l] = (uint8_t)clampi(v, 0, 15);
      }
    }
    uint8_t* qs = ob + 16;
    for (int g = 0; g < 4; g++)
      for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
  }
}

static void dequant_q4_k(const uint8_t* in, int64_t nb, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * Q4_K_BYTES;
    uint16_t dh, mh;
    memcpy(&dh, ib, 2);
    memcpy(&mh, ib + 2, 2);
    float d = h2f(dh), dmin = h2f(mh);
    const uint8_t* s = ib + 4;
    const uint8_t* qs = ib + 16;
    float* y = out + b * QK_K;
    for (int g = 0; g < 4; g++) {
      int sc, m;
      q4k_scale_min(2 * g, s, &sc, &m);
      float d1 = d * (float)sc, m1 = dmin * (float)m;
      q4k_scale_min(2 * g + 1, s, &sc, &m);
      float d2 = d * (float)sc, m2 = dmin * (float)m;
      for (int l = 0; l < 32; l++) {
        volatile float p = d1 * (float)(qs[32 * g + l] & 0xF); /* no FMA contraction */
        y[64 * g + l] = p - m1;
      }
      for (int l = 0; l < 32; l++) {
        volatile float p = d2 * (float)(qs[32 * g + l] >> 4);
        y[64 * g + 32 + l] = p - m2;
      }
    }
  }
}

/* ---------- Q4_0 / Q4_1 / Q5_0 / Q5_1 (32-value blocks) ---------- */
static void dequant_q4_01(const uint8_t* in, int64_t nb, float* out, int has_m) {
  const int bytes = has_m ? 20 : 18;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * bytes;
    uint16_t dh, mh = 0;
    memcpy(&dh, ib, 2);
    if (has_m) memcpy(&mh, ib + 2, 2);
    const float d = h2f(dh), m = h2f(mh);
    const uint8_t* qs = ib + (has_m ? 4 : 2);
    float* y = out + b * 32;
    for (int j = 0; j < 16; j++) {
      const int q0 = qs[j] & 0xF, q1 = qs[j] >> 4;
      if (has_m) {
        y[j] = (float)q0 * d + m;
        y[j + 16] = (float)q1 * d + m;
      } else {
        y[j] = (float)(q0 - 8) * d;
        y[j + 16] = (float)(q1 - 8) * d;
      }
    }
  }
}

static void dequant_q5_01(const uint8_t* in, int64_t nb, float* out, int has_m) {
  const int bytes = has_m ? 24 : 22;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * bytes;
    uint16_t dh, mh = 0;
    uint32_t qh;
    memcpy(&dh, ib, 2);
    if (has_m) memcpy(&mh, ib + 2, 2);
    memcpy(&qh, ib + (has_m ? 4 : 2), 4);
    const float d = h2f(dh), m = h2f(mh);
    const uint8_t* qs = ib + (has_m ? 8 : 6);
    float* y = out + b * 32;
    for (int j = 0; j < 16; j++) {
      const int q0 = (qs[j] & 0xF) | (((qh >> j) & 1) << 4);
      const int q1 = (qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
      if (has_m) {
        y[j] = (float)q0 * d + m;
        y[j + 16] = (float)q1 * d + m;
      } else {
        y[j] = (float)(q0 - 16) * d;
        y[j + 16] = (float)(q1 - 16) * d;
      }
    }
  }
}

/* ggml's reference quantizers for the 32-value block types (quantize_row_q4_0_ref and
 * siblings in ggml-quants.c; restated from gguf-py's bit-exact numpy port, gguf/quants.py
 * Q4_0..Q5_1.quantize_blocks, which the tests pin this against):
 *   symmetric (Q4_0 / Q5_0): max = the value of largest |x| (first one), d = max / -8 or -16,
 *     id = 1 / d (0 if d == 0), q = min(qmax, trunc(x id + 8.5 or 16.5))
 *   affine (Q4_1 / Q5_1): d = (max - min) / 15 or 31, id = 1 / d (0 if d == 0),
 *     q = min(qmax, trunc((x - min) id + 0.5)); the block stores f16(d) and f16(min)
 * q is computed with the unrounded f32 d. */
void or_quantize_q4q5(const float* x, int64_t n, uint8_t* out, int bits, int has_m) {
  const int bytes = bits == 4 ? (has_m ? 20 : 18) : (has_m ? 24 : 22);
  const int qmax = (1 << bits) - 1;
  int64_t nb = n / 32;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const float* xb = x + b * 32;
    uint8_t* ob = out + b * bytes;
    int q[32];
    if (has_m) {
      float mn = INFINITY, mx = -INFINITY;
      for (int j = 0; j < 32; j++) { mn = fminf(mn, xb[j]); mx = fmaxf(mx, xb[j]); }
      const float d = (mx - mn) / (float)qmax;
      const float id = d != 0.f ? 1.0f / d : 0.f;
      uint16_t dh = f2h(d), mh = f2h(mn);
      memcpy(ob, &dh, 2);
      memcpy(ob + 2, &mh, 2);
      for (int j = 0; j < 32; j++) {
        const float v = (xb[j] - mn) * id;
        q[j] = clampi((int)(v + 0.5f), 0, qmax);
      }
    } else {
      float amax = 0.f, vmax = 0.f;
      for (int j = 0; j < 32; j++)
        if (fabsf(xb[j]) > amax) { amax = fabsf(xb[j]); vmax = xb[j]; }
      const int half = 1 << (bits - 1);
      const float d = vmax / (float)(-half);
      const float id = d != 0.f ? 1.0f / d : 0.f;
      uint16_t dh = f2h(d);
      memcpy(ob, &dh, 2);
      for (int j = 0; j < 32; j++) {
        const float v = xb[j] * id;
        q[j] = clampi((int)(v + ((float)half + 0.5f)), 0, qmax);
      }
    }
    uint8_t* qs = ob + (has_m ? 4 : 2);
    if (bits == 5) {
      uint32_t qh = 0;
      for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
      memcpy(qs, &qh, 4);
      qs += 4;
    }
    for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
  }
}

/* ---------- Q5_K ---------- */
static void dequant_q5_k(const uint8_t* in, int64_t nb, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * 176;
    uint16_t dh, mh;
    memcpy(&dh, ib, 2);
    memcpy(&mh, ib + 2, 2);
    const float d = h2f(dh), dmin = h2f(mh);
    const uint8_t* s = ib + 4;
    const uint8_t* qh = ib + 16;
    const uint8_t* qs = ib + 48;
    float* y = out + b * QK_K;
    for (int g = 0; g < 4; g++) {
      for (int h = 0; h < 2; h++) {
        int sc, m;
        q4k_scale_min(2 * g + h, s, &sc, &m);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        for (int l = 0; l < 32; l++) {
          const int q = (h ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 0xF)) | (((qh[l] >> (2 * g + h)) & 1) << 4);
          volatile float p = d1 * (float)q; /* exact; no FMA contraction */
          y[64 * g + 32 * h + l] = p - m1;
        }
      }
    }
  }
}

void or_quantize_q5_k(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / QK_K;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const float* xb = x + b * QK_K;
    uint8_t* ob = out + b * 176;
    float scale[8], mins[8], max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
      float mn = 0.f, mx = -INFINITY;
      for (int l = 0; l < 32; l++) { mn = fminf(mn, xb[32 * j + l]); mx = fmaxf(mx, xb[32 * j + l]); }
      if (mx < mn) mx = mn;
      scale[j] = (mx - mn) / 31.f;
      mins[j] = -mn;
      max_scale = fmaxf(max_scale, scale[j]);
      max_min = fmaxf(max_min, mins[j]);
    }
    uint16_t dh = f2h(max_scale / 63.f), mh = f2h(max_min / 63.f);
    const float d = h2f(dh), dmin = h2f(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
      sc[j] = d > 0.f ? clampi((int)lrintf(scale[j] / d), 0, 63) : 0;
      m[j] = dmin > 0.f ? clampi((int)lrintf(mins[j] / dmin), 0, 63) : 0;
    }
    memcpy(ob, &dh, 2);
    memcpy(ob + 2, &mh, 2);
    uint8_t* s = ob + 4;
    for (int j = 0; j < 4; j++) {
      s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
      s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t* qh = ob + 16;
    uint8_t* qs = ob + 48;
    memset(qh, 0, 32);
    for (int g = 0; g < 4; g++) {
      for (int l = 0; l < 32; l++) {
        int q2[2];
        for (int h = 0; h < 2; h++) {
          const int j = 2 * g + h;
          const float dl = d * (float)sc[j], ml = dmin * (float)m[j];
          q2[h] = dl > 0.f ? clampi((int)lrintf((xb[32 * j + l] + ml) / dl), 0, 31) : 0;
          qh[l] |= (uint8_t)(((q2[h] >> 4) & 1) << (2 * g + h));
        }
        qs[32 * g + l] = (uint8_t)((q2[0] & 0xF) | ((q2[1] & 0xF) << 4));
      }
    }
  }
}

/* ---------- Q6_K ---------- */
static void dequant_q6_k(const uint8_t* in, int64_t nb, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const uint8_t* ib = in + b * 210;
    const uint8_t* ql = ib;
    const uint8_t* qh = ib + 128;
    const int8_t* sc = (const int8_t*)(ib + 192);
    uint16_t dh;
    memcpy(&dh, ib + 208, 2);
    const float d = h2f(dh);
    float* y = out + b * QK_K;
    for (int n2 = 0; n2 < 2; n2++) {
      for (int l = 0; l < 32; l++) {
        const int is = l / 16;
        const int q1 = (int)((ql[64 * n2 + l] & 0xF) | (((qh[32 * n2 + l] >> 0) & 3) << 4)) - 32;
        const int q2 = (int)((ql[64 * n2 + l + 32] & 0xF) | (((qh[32 * n2 + l] >> 2) & 3) << 4)) - 32;
        const int q3 = (int)((ql[64 * n2 + l] >> 4) | (((qh[32 * n2 + l] >> 4) & 3) << 4)) - 32;
        const int q4 = (int)((ql[64 * n2 + l + 32] >> 4) | (((qh[32 * n2 + l] >> 6) & 3) << 4)) - 32;
        y[128 * n2 + l] = d * (float)sc[8 * n2 + is + 0] * (float)q1;
        y[128 * n2 + l + 32] = d * (float)sc[8 * n2 + is + 2] * (float)q2;
        y[128 * n2 + l + 64] = d * (float)sc[8 * n2 + is + 4] * (float)q3;
        y[128 * n2 + l + 96] = d * (float)sc[8 * n2 + is + 6] * (float)q4;
      }
    }
  }
}

void or_quantize_q6_k(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / QK_K;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; b++) {
    const float* xb = x + b * QK_K;
    uint8_t* ob = out + b * 210;
    float sv[16], amax_all = 0.f;
    for (int j = 0; j < 16; j++) {
      float am = 0.f, vm = 0.f;
      for (int l = 0; l < 16; l++)
        if (fabsf(xb[16 * j + l]) > am) { am = fabsf(xb[16 * j + l]); vm = xb[16 * j + l]; }
      sv[j] = vm / -32.f;
      if (fabsf(sv[j]) > amax_all) amax_all = fabsf(sv[j]);
    }
    uint16_t dh = f2h(amax_all / 127.f);
    const float d = h2f(dh);
    int8_t* sc = (int8_t*)(ob + 192);
    int q[QK_K];
    for (int j = 0; j < 16; j++) {
      sc[j] = (int8_t)(d > 0.f ? clampi((int)lrintf(sv[j] / d), -127, 127) : 0);
      const float ds = d * (float)sc[j];
      for (int l = 0; l < 16; l++) q[16 * j + l] = ds != 0.f ? clampi((int)lrintf(xb[16 * j + l] / ds) + 32, 0, 63) : 32;
    }
    uint8_t* ql = ob;
    uint8_t* qh = ob + 128;
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int n2 = 0; n2 < 2; n2++)
      for (int l = 0; l < 32; l++) {
        const int* qq = q + 128 * n2;
        ql[64 * n2 + l] = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
        ql[64 * n2 + l + 32] = (uint8_t)((qq[l + 32] & 0xF) | ((qq[l + 96] & 0xF) << 4));
        qh[32 * n2 + l] = (uint8_t)(((qq[l] >> 4) & 3) | (((qq[l + 32] >> 4) & 3) << 2) | (((qq[l + 64] >> 4) & 3) << 4) |
                                    (((qq[l + 96] >> 4) & 3) << 6));
      }
    memcpy(ob + 208, &dh, 2);
  }
}

/* ggml type ids (GGMLQuantizationType): F32=0, F16=1, Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8,
 * Q4_K=12, Q5_K=13, Q6_K=14, BF16=30 */
int or_dequantize(int ggml_type, const uint8_t* in, int64_t n, float* out) {
  switch (ggml_type) {
    case 0: memcpy(out, in, (size_t)n * 4); return 0;
    case 1: or_f16_to_f32((const uint16_t*)in, n, out); return 0;
    case 30:
      for (int64_t i = 0; i < n; i++) {
        uint32_t v = (uint32_t)((const uint16_t*)in)[i] << 16;
        memcpy(&out[i], &v, 4);
      }
      return 0;
    case 8:
      if (n % QK8_0) return -1;
      dequant_q8_0(in, n / QK8_0, out);
      return 0;
    case 12:
      if (n % QK_K) return -1;
      dequant_q4_k(in, n / QK_K, out);
      return 0;
    case 2:
    case 3:
      if (n % 32) return -1;
      dequant_q4_01(in, n / 32, out, ggml_type == 3);
      return 0;
    case 6:
    case 7:
      if (n % 32) return -1;
      dequant_q5_01(in, n / 32, out, ggml_type == 7);
      return 0;
    case 13:
      if (n % QK_K) return -1;
      dequant_q5_k(in, n / QK_K, out);
      return 0;
    case 14:
      if (n % QK_K) return -1;
      dequant_q6_k(in, n / QK_K, out);
      return 0;
    default: return -2;
  }
}

/* ---------- LoRA merge (flux/lora.rs:651-868) ----------
 * Rows [row0, row0 + nrows) of a weight (raw GGUF bytes, n_cols values per row) become
 * quantize(dequant(w) + fl(fl(sum_k B[r,k] A[k,c]) * scale)), the dot product accumulated with
 * fmaf in ascending k; other rows are copied. A is [rank, n_cols], B is [nrows, rank] (f32).
 * The quantizers are the ones above (Q8_0: ggml's reference algorithm). */
int or_lora_merge(int type, const uint8_t* raw, int64_t n_rows, int64_t n_cols, int64_t row0, int64_t nrows,
                  const float* A, const float* B, int rank, float scale, uint8_t* out) {
  int64_t rb;
  switch (type) {
    case 0: rb = n_cols * 4; break;
    case 1: case 30: rb = n_cols * 2; break;
    case 8: rb = n_cols / 32 * 34; break;
    case 12: rb = n_cols / 256 * 144; break;
    case 2: rb = n_cols / 32 * 18; break;
    case 3: rb = n_cols / 32 * 20; break;
    case 6: rb = n_cols / 32 * 22; break;
    case 7: rb = n_cols / 32 * 24; break;
    case 13: rb = n_cols / 256 * 176; break;
    case 14: rb = n_cols / 256 * 210; break;
    default: return -2;
  }
  if (row0 < 0 || nrows < 0 || row0 + nrows > n_rows) return -1;
  memcpy(out, raw, (size_t)(n_rows * rb));
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < nrows; r++) {
    float* t = (float*)malloc((size_t)n_cols * sizeof(float));
    or_dequantize(type, raw + (row0 + r) * rb, n_cols, t);
    for (int64_t c = 0; c < n_cols; c++) {
      float acc = 0.f;
      for (int k = 0; k < rank; k++) acc = fmaf(B[r * rank + k], A[(int64_t)k * n_cols + c], acc);
      volatile float d = acc * scale;
      t[c] = t[c] + d;
    }
    uint8_t* o = out + (row0 + r) * rb;
    switch (type) {
      case 0: memcpy(o, t, (size_t)n_cols * 4); break;
      case 1: or_f32_to_f16(t, n_cols, (uint16_t*)o); break;
      case 30:
        for (int64_t c = 0; c < n_cols; c++) {
          float q;
          or_round_bf16(&t[c], 1, &q);
          uint32_t bits;
          memcpy(&bits, &q, 4);
          ((uint16_t*)o)[c] = (uint16_t)(bits >> 16);
        }
        break;
      case 8: or_quantize_q8_0(t, n_cols, o); break;
      case 12: or_quantize_q4_k(t, n_cols, o); break;
      case 2: or_quantize_q4q5(t, n_cols, o, 4, 0); break;
      case 3: or_quantize_q4q5(t, n_cols, o, 4, 1); break;
      case 6: or_quantize_q4q5(t, n_cols, o, 5, 0); break;
      case 7: or_quantize_q4q5(t, n_cols, o, 5, 1); break;
      case 13: or_quantize_q5_k(t, n_cols, o); break;
      case 14: or_quantize_q6_k(t, n_cols, o); break;
    }
    free(t);
  }
  return 0;
}

/* ---------- shared seeded generator ----------
 * value i of stream `seed` = std * N(0,1) where the normal comes from
 * Box-Muller on two uniforms u1 = (h(2i)>>40 + 1) * 2^-24 and u2 = (h(2i+1)>>40) * 2^-24,
 * h(c) = splitmix64(seed * 0x9E3779B97F4A7C15 + c). Computed in double, stored f32.
 */
static uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void or_randn(uint64_t seed, int64_t n, float std, float* out) {
  uint64_t base = seed * 0x9E3779B97F4A7C15ull;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    uint64_t a = splitmix64(base + 2 * (uint64_t)i), b = splitmix64(base + 2 * (uint64_t)i + 1);
    double u1 = ((double)(a >> 40) + 1.0) * (1.0 / 16777216.0);
    double u2 = (double)(b >> 40) * (1.0 / 16777216.0);
    double r = sqrt(-2.0 * log(u1));
    out[i] = (float)((double)std * r * cos(6.283185307179586 * u2));
  }
}
