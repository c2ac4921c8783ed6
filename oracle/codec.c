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
 *   - A Q8_0 quantizer equal to ggml's reference quantizer (amax/127, round half
 *     away from zero), pinned against gguf-py's Q8_0.quantize_blocks.
 *   - A Q4_K quantizer of this project's own (per-sub-block min/max, 6-bit
 *     scales relative to the super-block maxima). Any valid Q4_K block
 *     exercises the same decode; only the decode is required to be bit-exact.
 *   - The shared seeded generator (splitmix64 counter hash + Box-Muller) used
 *     for every synthetic tensor in tests and in the CPU baseline.
 */
#include <math.h>
#include <stdint.h>
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

/* ggml type ids (GGMLQuantizationType): F32=0, F16=1, Q8_0=8, Q4_K=12, BF16=30 */
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
    default: return -2;
  }
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
