// K3: batched quantized GEMV (M = 1) for the conditioning path: the stems'
// MLPs (time_in / guidance_in / vector_in, flux/offload.rs:583-609; Qwen's timestep MLP)
// and every block's AdaLN modulation silu(vec) -> Linear (flux/offload.rs:117-156,
// qwen_image/quantized_transformer.rs:868-879). All of a step's modulations depend only on
// vec, so they run as ONE launch over a job table (one job per weight), after one small
// launch that stages the input vectors. Weight-bandwidth bound: each weight byte is read
// once, with no shared memory or barrier between the loads; the staged x values a lane
// needs stay in its registers across the rows it serves.
#include "common.cuh"
#include "ggml_decode.cuh"
#include "internal.h"

namespace mb {
namespace gemv {

#ifndef MB_GEMV_WARPS
#define MB_GEMV_WARPS 4
#endif
constexpr int kWarps = MB_GEMV_WARPS;                     // warps per block
constexpr int kRowsPerWarp = kGemvRowsPerBlock / kWarps;  // 8
constexpr int kMaxLen = 4096;
constexpr int kMaxInputs = 4;
// Per staged input: x, its 32-value partial sums, then x as fixed-point digits for the Q4_K and
// Q8_0 paths (kQ4IOff in Q4_K unit order, kQ8IOff in Q8_0 unit order), stored slot-major: piece s of every unit (64 values for Q4_K, 32
// for Q8_0) first, then piece s + 1, ..., so that the lanes of a row group, which take
// consecutive units, read consecutive 16-byte pieces (coalesced) instead of pieces one unit apart.
// The digits: x = S * xi with xi a 24-bit integer (S = max|x| / (2^23 - 1)), xi = d0 2^16 +
// d1 2^8 + d2 (d0 signed, d1 and d2 unsigned bytes); four values' digits are packed per 32-bit
// word, as uint4 (d0 word, d1 word, d2 word, unused) per 4 values. S is stored at kScaleOff.
constexpr int kQ4IOff = kMaxLen + kMaxLen / 32;
constexpr int kQ8IOff = kQ4IOff + kMaxLen;
constexpr int kScaleOff = kQ8IOff + kMaxLen;
constexpr int kStageStride = kScaleOff + 4;


struct Inputs {
  GemvInput in[kMaxInputs];
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

// Stage every input vector once: x = silu?(sum of parts) and its 32-value partial sums
// (the Q4_K min term needs sum(x) per sub-block). Block s handles input s.
__global__ void k_gemv_stage(Inputs ins, float* __restrict__ stage) {
  const GemvInput in = ins.in[blockIdx.x];
  float* xs = stage + (int64_t)blockIdx.x * kStageStride;
  float* xsum = xs + kMaxLen;
  for (int i = threadIdx.x * 4; i < in.len; i += blockDim.x * 4) {
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    // the integer copies: S from the vector's max |x|, then the three digits of round(x / S)
    __shared__ float red[32];
    float mx = 0.f;
    for (int i = threadIdx.x; i < in.len; i += blockDim.x) {
      const float a = fabsf(xs[i]);
      mx = a <= 3.402823466e38f ? fmaxf(mx, a) : __int_as_float(0x7f800000);  // NaN and inf count as inf
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
    // a non-finite x makes S NaN, so the rows' results are NaN as a float product's would be
    const float S = !(mx <= 3.402823466e38f) ? __int_as_float(0x7fc00000) : (mx > 0.f ? mx / 8388607.f : 1.f);
    const float invS = S == S ? 1.f / S : 0.f;
    if (threadIdx.x == 0) xs[kScaleOff] = S;
    for (int i = threadIdx.x * 4; i < in.len; i += blockDim.x * 4) {
      uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        int xi = __float2int_rn(xs[i + t] * invS);
        xi = max(-8388607, min(8388607, xi));
        w0 |= ((uint32_t)(xi >> 16) & 0xFFu) << (8 * t);
        w1 |= ((uint32_t)(xi >> 8) & 0xFFu) << (8 * t);
        w2 |= ((uint32_t)xi & 0xFFu) << (8 * t);
      }
      ((uint4*)(xs + kQ4IOff))[((i & 63) >> 2) * (in.len >> 6) + (i >> 6)] = make_uint4(w0, w1, w2, 0u);
      ((uint4*)(xs + kQ8IOff))[((i & 31) >> 2) * (in.len >> 5) + (i >> 5)] = make_uint4(w0, w1, w2, 0u);
    }
  }
  for (int c = warp; c < in.len / 32; c += blockDim.x >> 5) {

    float v = xs[c * 32 + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) xsum[c] = v;
  }
}

// Reduce a per-lane partial over the LPR lanes of one row group and store the row result.
template <int LPR>
MB_DEV void finish_rows(const float (&acc)[kRowsPerWarp * LPR / 32], int r0, int sub, int sl, int nr,
                        const GemvJob& job) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB;
#pragma unroll
  for (int i = 0; i < RPL; i++) {
    float v = acc[i];
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int rr = sub + i * NSUB;
    if (sl == 0 && rr < nr) job.y[r0 + rr] = v + (job.bias ? job.bias[r0 + rr] : 0.f);
  }
}

MB_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned bytes of a . signed bytes of b + c
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
MB_DEV uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
MB_DEV int dp4a_ss(uint32_t a, uint32_t b, int c) {  // signed bytes . signed bytes + c
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
MB_DEV int dp4a_su(uint32_t a, uint32_t b, int c) {  // signed bytes of a . unsigned bytes of b + c
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K rows on the integer pipe: a group of LPR lanes serves one row; lane sl takes the 64-value
// units sl, sl + LPR, ... (unit = the low and high nibbles of one 32-byte quant run = sub-blocks
// 2g and 2g+1) of its RPL rows. The nibbles (low ones as bytes 0..15, high ones in place as
// 16 q) multiply the three byte digits of the fixed-point x with dp4a, 4 products per
// instruction with exact integer sums; a unit's digit sums are combined in f32 once.
#ifndef MB_GEMV_Q4K_RB
#define MB_GEMV_Q4K_RB 2  // rows per load batch
#endif
template <int LPR>
MB_DEV void rows_q4k_int(const GemvJob& job, const uint8_t* wbase, const float* __restrict__ xs,
                         const float* __restrict__ xsum, int r0, int nr, int lane) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB, RB = RPL < MB_GEMV_Q4K_RB ? RPL : MB_GEMV_Q4K_RB;
  const int sub = lane / LPR, sl = lane % LPR;
  const int U = job.n_cols / 64;
  const float S = xs[kScaleOff];
  float acc[RPL];
#pragma unroll
  for (int i = 0; i < RPL; i++) acc[i] = 0.f;
  for (int u = sl; u < U; u += LPR) {
    const int kb = u >> 2, g = u & 3;
    const uint4* xi = (const uint4*)(xs + kQ4IOff) + u;  // slot s of unit u at xi[s * U]
    const float s_lo = __ldg(xsum + 2 * u), s_hi = __ldg(xsum + 2 * u + 1);
    // rows in batches of RB: all loads of a batch first (rows past the job's end re-read its
    // last row; finish_rows drops them); the unit's digits are read per word and shared by the
    // batch's rows
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += RB) {
      uint4 H[RB], A[RB], B[RB];
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const int rr = min(sub + (i0 + j) * NSUB, nr - 1);
        const uint8_t* b = wbase + (int64_t)rr * job.row_bytes + kb * 144;
        H[j] = *(const uint4*)b;
        A[j] = *(const uint4*)(b + 16 + 32 * g);
        B[j] = *(const uint4*)(b + 32 + 32 * g);
      }
      int l0[RB], h0[RB];
      uint32_t l1[RB], l2[RB], h1[RB], h2[RB];
#pragma unroll
      for (int j = 0; j < RB; j++) l0[j] = h0[j] = 0, l1[j] = l2[j] = h1[j] = h2[j] = 0u;
#pragma unroll
      for (int I = 0; I < 8; I++) {
        const uint4 xl = __ldg(xi + I * U), xh = __ldg(xi + (8 + I) * U);
#pragma unroll
        for (int j = 0; j < RB; j++) {
          const uint32_t W = I < 4 ? (I == 0 ? A[j].x : I == 1 ? A[j].y : I == 2 ? A[j].z : A[j].w)
                                   : (I == 4 ? B[j].x : I == 5 ? B[j].y : I == 6 ? B[j].z : B[j].w);
          const uint32_t lo = W & 0x0F0F0F0Fu, hi = W & 0xF0F0F0F0u;  // hi bytes hold 16 q
          l0[j] = dp4a_us(lo, xl.x, l0[j]);
          l1[j] = dp4a_uu(lo, xl.y, l1[j]);
          l2[j] = dp4a_uu(lo, xl.z, l2[j]);
          h0[j] = dp4a_us(hi, xh.x, h0[j]);
          h1[j] = dp4a_uu(hi, xh.y, h1[j]);
          h2[j] = dp4a_uu(hi, xh.z, h2[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const float dlo = S * ((float)l0[j] * 65536.f + (float)l1[j] * 256.f + (float)l2[j]);
        const float dhi = S * 0.0625f * ((float)h0[j] * 65536.f + (float)h1[j] * 256.f + (float)h2[j]);
        const float d = h16(H[j].x), dmin = h16(H[j].x >> 16);
        int sc0, m0, sc1, m1;
        q4k_sm(2 * g, H[j].y, H[j].z, H[j].w, sc0, m0);
        q4k_sm(2 * g + 1, H[j].y, H[j].z, H[j].w, sc1, m1);
        acc[i0 + j] += d * (float)sc0 * dlo - dmin * (float)m0 * s_lo + d * (float)sc1 * dhi - dmin * (float)m1 * s_hi;
      }
    }
  }
  finish_rows<LPR>(acc, r0, sub, sl, nr, job);
}

// Q8_0 rows on the integer pipe: each block's 32 int8 weights times the three byte digits of the
// fixed-point x (dp4a, exact integer sums), combined in f32 once per block and scaled by d.
template <int LPR>
MB_DEV void rows_q8_int(const GemvJob& job, const uint8_t* wbase, const float* __restrict__ xs, int r0, int nr,
                        int lane) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB, RB = RPL < 4 ? RPL : 4;
  const int sub = lane / LPR, sl = lane % LPR;
  const int U = job.n_cols / 32;
  const float S = xs[kScaleOff];
  float acc[RPL];
#pragma unroll
  for (int i = 0; i < RPL; i++) acc[i] = 0.f;
  for (int u = sl; u < U; u += LPR) {
    uint4 xd[8];
#pragma unroll
    for (int i = 0; i < 8; i++) xd[i] = __ldg((const uint4*)(xs + kQ8IOff) + i * U + u);
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += RB) {
      uint32_t wv[RB][10];
      bool sh[RB];  // the 34-byte block starts 2 bytes into a word
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const int rr = min(sub + (i0 + j) * NSUB, nr - 1);
        const uint8_t* b = wbase + (int64_t)rr * job.row_bytes + u * 34;
        const uint32_t* a4 = (const uint32_t*)((uintptr_t)b & ~(uintptr_t)3);
        sh[j] = ((uintptr_t)b & 3) != 0;
#pragma unroll
        for (int k = 0; k < 10; k++) wv[j][k] = a4[k];
      }
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const float d = sh[j] ? h16(wv[j][0] >> 16) : h16(wv[j][0]);
        int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t q = sh[j] ? wv[j][k + 1] : __byte_perm(wv[j][k], wv[j][k + 1], 0x5432);
          a0 = dp4a_ss(q, xd[k].x, a0);
          a1 = dp4a_su(q, xd[k].y, a1);
          a2 = dp4a_su(q, xd[k].z, a2);
        }
        acc[i0 + j] += d * (S * ((float)a0 * 65536.f + (float)a1 * 256.f + (float)a2));
      }
    }
  }
  finish_rows<LPR>(acc, r0, sub, sl, nr, job);
}

// Q6_K rows (224-byte device chunks of 256 values): unit u = values 32u .. 32u+31 of a chunk,
// x_l = d sc[16-value group] (q6_l - 32). A lane keeps its unit's 32 staged x values in registers
// and serves its rows RB at a time with all their loads issued first; the scales multiply the two
// 16-value partial dots (exact decode is not needed for a float dot product).
template <int LPR>
MB_DEV void rows_q6k(const GemvJob& job, const float* __restrict__ xs, int r0, int nr, int lane) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB, RB = RPL < 4 ? RPL : 4;
  const int sub = lane / LPR, sl = lane % LPR;
  const int U = job.n_cols / 32;
  const uint8_t* wbase = (const uint8_t*)job.w + (int64_t)r0 * job.row_bytes;
  float acc[RPL];
#pragma unroll
  for (int i = 0; i < RPL; i++) acc[i] = 0.f;
  for (int u = sl; u < U; u += LPR) {
    const int c = u >> 3, uu = u & 7, n = uu >> 2, g = uu & 3;
    const int nsh = (g >> 1) * 4, hsh = 2 * g;
    float x[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 t = __ldg((const float4*)(xs + u * 32) + i);
      x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
    }
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += RB) {
      uint4 L0[RB], L1[RB], H0[RB], H1[RB];
      uint32_t SD[RB], DD[RB];
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const int rr = min(sub + (i0 + j) * NSUB, nr - 1);  // rows past the end re-read the last row
        const uint8_t* b = wbase + (int64_t)rr * job.row_bytes + (int64_t)c * 224;
        L0[j] = __ldg((const uint4*)(b + 64 * n + 32 * (g & 1)));
        L1[j] = __ldg((const uint4*)(b + 64 * n + 32 * (g & 1) + 16));
        H0[j] = __ldg((const uint4*)(b + 128 + 32 * n));
        H1[j] = __ldg((const uint4*)(b + 128 + 32 * n + 16));
        SD[j] = __ldg((const uint16_t*)(b + 192 + 8 * n + 2 * g));
        DD[j] = __ldg((const uint16_t*)(b + 208));
      }
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const uint32_t lw[8] = {L0[j].x, L0[j].y, L0[j].z, L0[j].w, L1[j].x, L1[j].y, L1[j].z, L1[j].w};
        const uint32_t hw[8] = {H0[j].x, H0[j].y, H0[j].z, H0[j].w, H1[j].x, H1[j].y, H1[j].z, H1[j].w};
        float dot0 = 0.f, dot1 = 0.f;
#pragma unroll
        for (int k = 0; k < 32; k++) {
          const uint32_t lo = (lw[k >> 2] >> (8 * (k & 3) + nsh)) & 0xFu;
          const uint32_t hi = (hw[k >> 2] >> (8 * (k & 3) + hsh)) & 3u;
          const float q = (float)((int)(lo | (hi << 4)) - 32);
          if (k < 16) dot0 = fmaf(q, x[k], dot0);
          else dot1 = fmaf(q, x[k], dot1);
        }
        const float d = h16(DD[j]);
        const float s0 = (float)(int8_t)(SD[j] & 0xFFu), s1 = (float)(int8_t)(SD[j] >> 8);
        acc[i0 + j] += d * (s0 * dot0 + s1 * dot1);
      }
    }
  }
  finish_rows<LPR>(acc, r0, sub, sl, nr, job);
}

// Q4_1 rows: unit = one 20-byte block (f16 d, f16 m, 16 bytes of nibbles) of 32 values,
// sum_j (d q_j + m) x_j = d sum_j q_j x_j + m sum_j x_j (the staged 32-value partial sums).
template <int LPR>
MB_DEV void rows_q41(const GemvJob& job, const float* __restrict__ xs, const float* __restrict__ xsum, int r0, int nr,
                     int lane) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB, RB = RPL < 4 ? RPL : 4;
  const int sub = lane / LPR, sl = lane % LPR;
  const int U = job.n_cols / 32;
  const uint8_t* wbase = (const uint8_t*)job.w + (int64_t)r0 * job.row_bytes;
  float acc[RPL];
#pragma unroll
  for (int i = 0; i < RPL; i++) acc[i] = 0.f;
  for (int u = sl; u < U; u += LPR) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 t = __ldg((const float4*)(xs + u * 32) + i);
      x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
    }
    const float s = __ldg(xsum + u);
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += RB) {
      uint32_t w[RB][5];  // 20-byte blocks are 4-byte aligned
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const int rr = min(sub + (i0 + j) * NSUB, nr - 1);
        const uint32_t* b = (const uint32_t*)(wbase + (int64_t)rr * job.row_bytes + (int64_t)u * 20);
#pragma unroll
        for (int k = 0; k < 5; k++) w[j][k] = __ldg(b + k);
      }
#pragma unroll
      for (int j = 0; j < RB; j++) {
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const uint32_t byte = (w[j][1 + (k >> 2)] >> (8 * (k & 3))) & 0xFFu;
          dot = fmaf((float)(byte & 0xF), x[k], dot);
          dot = fmaf((float)(byte >> 4), x[k + 16], dot);
        }
        acc[i0 + j] += h16(w[j][0]) * dot + h16(w[j][0] >> 16) * s;
      }
    }
  }
  finish_rows<LPR>(acc, r0, sub, sl, nr, job);
}

// Other chunked types: unit = 32 values decoded by decode_unit<T> straight from global memory.
// A lane serves its rows RB at a time (the RB decodes are independent, so their loads are in flight
// together), reading the unit's staged x values once per row pair.
template <int T, int LPR>
MB_DEV void rows_units(const GemvJob& job, const float* __restrict__ xs, int r0, int nr, int lane) {
  constexpr int NSUB = 32 / LPR, RPL = kRowsPerWarp / NSUB;
  constexpr int RB = T == MB_GGML_Q5_K ? 1 : (RPL < 2 ? RPL : 2);  // Q5_K's decode needs the registers
  const int sub = lane / LPR, sl = lane % LPR;
  const int U = job.n_cols / 32;
  const uint8_t* wbase = (const uint8_t*)job.w + (int64_t)r0 * job.row_bytes;
  float acc[RPL];
#pragma unroll
  for (int i = 0; i < RPL; i++) acc[i] = 0.f;
  for (int u = sl; u < U; u += LPR) {
    const int64_t coff = (int64_t)(u >> 3) * kDeviceChunk(T);
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += RB) {
      float y[RB][32];
#pragma unroll
      for (int j = 0; j < RB; j++) {
        const int rr = min(sub + (i0 + j) * NSUB, nr - 1);  // rows past the end re-read the last row
        decode_unit<T>(wbase + (int64_t)rr * job.row_bytes + coff, u & 7, y[j]);
      }
#pragma unroll
      for (int k4 = 0; k4 < 8; k4++) {
        const float4 t = __ldg((const float4*)(xs + u * 32) + k4);
#pragma unroll
        for (int j = 0; j < RB; j++) {
          float a = acc[i0 + j];
          a = fmaf(y[j][4 * k4], t.x, a);
          a = fmaf(y[j][4 * k4 + 1], t.y, a);
          a = fmaf(y[j][4 * k4 + 2], t.z, a);
          a = fmaf(y[j][4 * k4 + 3], t.w, a);
          acc[i0 + j] = a;
        }
      }
    }
  }
  finish_rows<LPR>(acc, r0, sub, sl, nr, job);
}

template <int T>
MB_DEV void rows_units_any(const GemvJob& job, const float* __restrict__ xs, int r0, int nr, int lane) {
  if ((job.n_cols / 32) % 32 == 0)
    rows_units<T, 32>(job, xs, r0, nr, lane);
  else
    rows_units<T, 16>(job, xs, r0, nr, lane);
}

// F32 / F16 / BF16 rows: the whole warp serves one row at a time.
MB_DEV void rows_plain(const GemvJob& job, const float* __restrict__ xs, int r0, int nr, int lane) {
  const uint8_t* wbase = (const uint8_t*)job.w + (int64_t)r0 * job.row_bytes;
  float acc[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; i++) acc[i] = 0.f;
  for (int c = lane; c < job.n_cols; c += 32) {
    const float xv = __ldg(xs + c);
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; i++) {
      if (i < nr) {
        const uint8_t* row = wbase + (int64_t)i * job.row_bytes;
        float wv;
        if (job.type == MB_GGML_F32) wv = ((const float*)row)[c];
        else if (job.type == MB_GGML_F16) wv = __half2float(((const __half*)row)[c]);
        else wv = __uint_as_float((uint32_t)((const uint16_t*)row)[c] << 16);
        acc[i] = fmaf(wv, xv, acc[i]);
      }
    }
  }
  finish_rows<32>(acc, r0, 0, lane, nr, job);
}

// Kernel instance of a weight type: 2 Q4_K, 0 Q8_0 and the plain types, 1 the decode_unit types.
__host__ __device__ inline int kind_of(int t) {
  return t == MB_GGML_Q4_K ? 2
                           : ((t == MB_GGML_Q8_0 || t == MB_GGML_F32 || t == MB_GGML_F16 || t == MB_GGML_BF16) ? 0 : 1);
}

// One block = kWarps warps x kRowsPerWarp rows of one job (blocks[] = (job, first row)). Three
// kernels (KIND 2: Q4_K; KIND 0: Q8_0 and the plain types; KIND 1: the decode_unit types) so that
// each is compiled for its own paths' registers (the Q4_K kernel, alone, fits more blocks per SM);
// a block whose job is of another kind returns at once.
// Q4_K and Q8_0 blocks first copy their 32 contiguous rows into shared memory with one bulk copy
// (smem_rb bytes per row reserved): the copy engine streams them at full rate, and the lanes then
// read their scattered 16-byte pieces from shared memory (conflict-free) instead of as many
// partially used global sectors.
#ifndef MB_GEMV_MINB
#define MB_GEMV_MINB 3
#endif
#ifndef MB_GEMV_MINB_Q4K
#define MB_GEMV_MINB_Q4K 4
#endif
template <int KIND>
__global__ void __launch_bounds__(kWarps * 32, KIND == 2 ? MB_GEMV_MINB_Q4K : MB_GEMV_MINB)
    k_gemv(const GemvJob* __restrict__ jobs, const int2* __restrict__ blocks, GemvJob inline_job,
           const float* __restrict__ stage, int smem_rb, int* status) {
  extern __shared__ __align__(128) uint8_t sw[];
  __shared__ uint64_t wbar;
  __shared__ int abort_flag;
  const int2 bj = jobs ? blocks[blockIdx.x] : make_int2(0, blockIdx.x * kGemvRowsPerBlock);
  const GemvJob job = jobs ? jobs[bj.x] : inline_job;
  if (kind_of(job.type) != KIND) return;
  const float* xs = stage + (int64_t)job.x_slot * kStageStride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (KIND == 0 || KIND == 2) {
    if (job.type == MB_GGML_Q4_K || job.type == MB_GGML_Q8_0) {
      const int nrb = min(kGemvRowsPerBlock, job.n_rows - bj.y);
      if (job.row_bytes > smem_rb || nrb <= 0) return;  // the launch reserved too little: skip, never overrun
      const uint32_t bytes = (uint32_t)(nrb * job.row_bytes);
      if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(&wbar, 1);
        fence_mbar_init();
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        mbar_expect_tx(&wbar, bytes);
        bulk_load(sw, (const uint8_t*)job.w + (int64_t)bj.y * job.row_bytes, bytes, &wbar);
      }
      if (!mbar_wait(&wbar, 0, &abort_flag, status, kDevTimeoutGemv)) return;
      const int rl = warp * kRowsPerWarp;  // first row of this warp within the block
      if (rl >= nrb) return;
      const int nr = min(kRowsPerWarp, nrb - rl);
      const uint8_t* wb = sw + (int64_t)rl * job.row_bytes;
      const int r0 = bj.y + rl;
      if constexpr (KIND == 2) {
        if ((job.n_cols / 64) % 16 == 0)
          rows_q4k_int<16>(job, wb, xs, xs + kMaxLen, r0, nr, lane);
        else
          rows_q4k_int<32>(job, wb, xs, xs + kMaxLen, r0, nr, lane);
      } else {
        if ((job.n_cols / 32) % 32 == 0)
          rows_q8_int<32>(job, wb, xs, r0, nr, lane);
        else
          rows_q8_int<16>(job, wb, xs, r0, nr, lane);
      }
      return;
    }
  }
  const int r0 = bj.y + warp * kRowsPerWarp;
  if (r0 >= job.n_rows) return;
  const int nr = min(kRowsPerWarp, job.n_rows - r0);
  if constexpr (KIND == 0) {
    rows_plain(job, xs, r0, nr, lane);
  } else if constexpr (KIND == 1) {
    if (job.type == MB_GGML_Q4_0) {
      rows_units_any<MB_GGML_Q4_0>(job, xs, r0, nr, lane);
    } else if (job.type == MB_GGML_Q4_1) {
      if ((job.n_cols / 32) % 32 == 0)
        rows_q41<32>(job, xs, xs + kMaxLen, r0, nr, lane);
      else
        rows_q41<16>(job, xs, xs + kMaxLen, r0, nr, lane);
    } else if (job.type == MB_GGML_Q5_0) {
      rows_units_any<MB_GGML_Q5_0>(job, xs, r0, nr, lane);
    } else if (job.type == MB_GGML_Q5_1) {
      rows_units_any<MB_GGML_Q5_1>(job, xs, r0, nr, lane);
    } else if (job.type == MB_GGML_Q5_K) {
      rows_units_any<MB_GGML_Q5_K>(job, xs, r0, nr, lane);
    } else {
      if ((job.n_cols / 32) % 32 == 0)
        rows_q6k<32>(job, xs, r0, nr, lane);
      else
        rows_q6k<16>(job, xs, r0, nr, lane);
    }
  }
}

}  // namespace gemv

int gemv_kind(int ggml_type) { return gemv::kind_of(ggml_type); }

int64_t gemv_smem_row_bytes(int ggml_type, int64_t row_bytes) {
  return (ggml_type == MB_GGML_Q4_K || ggml_type == MB_GGML_Q8_0) ? row_bytes : 0;
}

// Dynamic shared memory of the KIND 0 / 2 kernels for `smem_rb` bytes per row (their attribute is
// raised once per device to the largest size requested so far).
template <int KIND>
static cudaError_t gemv_smem(int64_t smem_rb, size_t* bytes) {
  *bytes = (size_t)smem_rb * kGemvRowsPerBlock;
  if (*bytes > 200 * 1024) return cudaErrorInvalidValue;
  static size_t done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (*bytes > done[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv::k_gemv<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)*bytes);
    if (e != cudaSuccess) return e;
    done[dev & 63] = *bytes;
  }
  return cudaSuccess;
}

cudaError_t launch_gemv_batch(const GemvJob* jobs_dev, int kinds, const int* block_job_dev, int n_blocks,
                              const GemvInput* inputs, int n_inputs, float* stage, int64_t smem_row_bytes,
                              cudaStream_t st) {
  if (kinds & ~7) return cudaErrorInvalidValue;
  if (n_inputs < 1 || n_inputs > gemv::kMaxInputs || !stage) return cudaErrorInvalidValue;
  gemv::Inputs ins = {};
  for (int i = 0; i < n_inputs; i++) {
    if (inputs[i].len <= 0 || inputs[i].len > gemv::kMaxLen || inputs[i].len % 32) return cudaErrorInvalidValue;
    ins.in[i] = inputs[i];
  }
  gemv::k_gemv_stage<<<n_inputs, 256, 0, st>>>(ins, stage);
  GemvJob dummy = {};
  int* status = device_status_ptr();
  if (kinds & 1) {
    size_t sm = 0;
    cudaError_t e = gemv_smem<0>(smem_row_bytes, &sm);
    if (e != cudaSuccess) return e;
    gemv::k_gemv<0><<<n_blocks, gemv::kWarps * 32, sm, st>>>(jobs_dev, (const int2*)block_job_dev, dummy, stage,
                                                            (int)smem_row_bytes, status);
  }
  if (kinds & 4) {
    size_t sm = 0;
    cudaError_t e = gemv_smem<2>(smem_row_bytes, &sm);
    if (e != cudaSuccess) return e;
    gemv::k_gemv<2><<<n_blocks, gemv::kWarps * 32, sm, st>>>(jobs_dev, (const int2*)block_job_dev, dummy, stage,
                                                            (int)smem_row_bytes, status);
  }
  if (kinds & 2)
    gemv::k_gemv<1><<<n_blocks, gemv::kWarps * 32, 0, st>>>(jobs_dev, (const int2*)block_job_dev, dummy, stage, 0,
                                                           status);
  return cudaGetLastError();
}

size_t gemv_stage_floats() { return (size_t)gemv::kMaxInputs * gemv::kStageStride; }

// Single-weight GEMV without a device job table (mb_qgemv).
cudaError_t launch_gemv_single(const mb_weight* w, const float* x, int apply_silu, const float* bias, float* y,
                               cudaStream_t st) {
  if (w->n_cols > gemv::kMaxLen || w->n_cols % 32) return cudaErrorInvalidValue;
  float* stage = (float*)device_scratch(gemv_stage_floats() * sizeof(float));
  if (!stage) return cudaErrorMemoryAllocation;
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
  gemv::k_gemv_stage<<<1, 256, 0, st>>>(ins, stage);
  const int blocks = (int)((w->n_rows + kGemvRowsPerBlock - 1) / kGemvRowsPerBlock);
  int* status = device_status_ptr();
  const int kind = gemv_kind(w->type);
  if (kind == 0 || kind == 2) {
    const int64_t rb = gemv_smem_row_bytes(w->type, w->row_bytes);
    size_t sm = 0;
    cudaError_t e = kind == 0 ? gemv_smem<0>(rb, &sm) : gemv_smem<2>(rb, &sm);
    if (e != cudaSuccess) return e;
    if (kind == 0)
      gemv::k_gemv<0><<<blocks, gemv::kWarps * 32, sm, st>>>(nullptr, nullptr, j, stage, (int)rb, status);
    else
      gemv::k_gemv<2><<<blocks, gemv::kWarps * 32, sm, st>>>(nullptr, nullptr, j, stage, (int)rb, status);
  } else {
    gemv::k_gemv<1><<<blocks, gemv::kWarps * 32, 0, st>>>(nullptr, nullptr, j, stage, 0, status);
  }
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
