// K2: GGUF-quantized linear y = epilogue(x W^T + b) on tcgen05 / TMEM (sm_100a).
//
// Replaces candle's QMatMul::forward (quantized FLUX, flux/transformer.rs:64-72)
// and QwenLinear::forward (qwen_image/quantized_transformer.rs:54-77).
//
// Design (one persistent CTA per SM, warp-specialised):
//   * The product is computed transposed: D[n, m] = W[n, :] . X[m, :], so the
//     weight tile is the MMA's A operand and lives in TENSOR MEMORY: dequant
//     warps decode raw GGML blocks to bf16 in registers and tcgen05.st them
//     straight into TMEM (one TMEM lane = one weight row). Dequantized weights
//     never touch shared memory, which keeps shared-memory traffic at the X tile
//     (TMA write + MMA read) plus the raw blocks.
//   * X (activations, bf16, K-major) is TMA-loaded with the 128-byte swizzle into
//     an 8-stage ring and read by tcgen05.mma as the B operand.
//   * Raw weight bytes are TMA-loaded in their GGUF layout (Q4_K: whole 144-byte
//     super-blocks, one TMA per 4 stages, scales decoded once per super-block; Q8_0 and
//     the other block types: whole 256-value chunks likewise; BF16: 128 bytes per stage).
//   * Tile = 128 weight rows x 256 activation rows, so each decoded weight feeds
//     256 MACs (the dequant rate needed is 16 values per SM clock at full MMA
//     rate). TMEM: the 128x256 f32 accumulator in columns [0, 256) and an
//     8-deep ring of 64-wide bf16 A stages in [256, 512). The epilogue releases
//     the accumulator as soon as its last columns are in registers.
//   * CTA pairs (default): a cluster of two CTAs on two SMs computes a 256-weight-row x
//     256-activation-row tile with tcgen05.mma.cta_group::2 (M = 256). Each CTA decodes its own
//     128 weight rows into its own TMEM and TMA-loads only its 128-row half of the X tile; the
//     leader's MMAs read both halves, so each SM streams half the activation bytes from L2
//     (the unpaired kernel re-reads the full 256-row X tile per 128 weight rows). Both CTAs'
//     X bytes and decoder arrivals complete on the leader's barriers; the leader's commits
//     arrive on both CTAs' barriers (tcgen05.commit multicast); no TMA load is multicast.
// Warp roles (576 threads): 0 TMA producer, 1 MMA issuer + TMEM owner,
// 2..9 dequant (two threads per weight row, one per K half of a stage),
// 10..17 epilogue (thread = output feature n; stores are coalesced along n).
// Decoding uses sm_100's packed f32x2 FMA/SUB (two exact IEEE ops per instruction).
//
// Bit-exactness: the dequantized value of every weight equals the GGML decode
// (Q4_K: (d*sc)*q - dmin*m with one rounding per operation; Q8_0: d*q) rounded
// to bf16 RNE. d1*q is formed as fma(d1, 2^23+q, -d1*2^23), which is the same
// single rounding of the exact product.
#include "common.cuh"
#include "ggml_decode.cuh"
#include "internal.h"

namespace mb {

namespace gemm {

constexpr int TN = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int TM = 256;  // activation rows per tile (MMA N): every decoded weight feeds 256 rows
constexpr int BK = 64;   // K per stage
// The decoded-A ring in TMEM (32 columns per stage) has the same depth as the X ring in shared
// memory: stage s uses slot s % SX of both, so one "full" and one "empty" barrier per slot cover
// both operands (one barrier wait and one commit per stage in the MMA issuer).
constexpr int kDW = 8;   // dequant warps (2..9)
constexpr int kEW = 8;   // epilogue warps (10..17)
constexpr int kThreads = (2 + kDW + kEW) * 32;
constexpr uint32_t kXStageBytes = TM * BK * 2;  // 32 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = 256;  // first A-stage column (D uses [0, 256))
constexpr int kMaxSX = 4;         // A ring [256, 384)
// Epilogue staging [384, 512): each epilogue warp parks its 128 packed bf16 results (64 words per
// lane) here, so the accumulator is freed without holding them in registers (the kernel's 18
// warps leave 96 registers per thread; a register-resident copy spills).
constexpr uint32_t kTmemStage = kTmemA + kMaxSX * 32;

// Other quantized types: one 256-value chunk per row and raw stage (kDeviceChunk bytes, a
// multiple of 16), decoded per 32-value unit by decode_unit<WT>.
template <int WT>
struct Cfg {
  static constexpr int kRawRow = kDeviceChunk(WT), kSPC = 4, kSR = 3, kSX = 4;
};
template <>
struct Cfg<MB_GGML_Q4_K> {
  static constexpr int kRawRow = 144, kSPC = 4, kSR = 3, kSX = 4;  // whole super-blocks
};
template <>
struct Cfg<MB_GGML_Q8_0> {
  // whole 272-byte chunks of 8 blocks (loaded as 136 16-bit elements: a TMA box is <= 256 wide);
  // measured +10 % over one 80-byte window per stage
  static constexpr int kRawRow = 272, kSPC = 4, kSR = 2, kSX = 4;
};
template <>
struct Cfg<MB_GGML_BF16> {
  static constexpr int kRawRow = 128, kSPC = 1, kSR = 4, kSX = 4;
};

static_assert(Cfg<MB_GGML_Q4_K>::kSX <= kMaxSX && Cfg<MB_GGML_Q8_0>::kSX <= kMaxSX && Cfg<MB_GGML_BF16>::kSX <= kMaxSX &&
                  Cfg<MB_GGML_Q6_K>::kSX <= kMaxSX,
              "A ring must fit below the epilogue staging columns");
static_assert(1024 + 4 * 32768 + 3 * 128 * 224 + 512 <= 232448, "largest raw ring must fit in shared memory");
// X bytes per stage and CTA: a CTA pair splits the tile's 256 activation rows between its two CTAs.
template <bool PAIR>
constexpr uint32_t x_stage_bytes() {
  return PAIR ? kXStageBytes / 2 : kXStageBytes;
}
template <int WT, bool PAIR>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)Cfg<WT>::kSX * x_stage_bytes<PAIR>() + (size_t)Cfg<WT>::kSR * TN * Cfg<WT>::kRawRow + 512;
}

struct Prob {  // one GEMM of a (possibly grouped) launch
  int M, N, K;
  int tiles_m, tiles_n, tile0;  // tile0: first global tile index of this problem
  GemmEpilogue epi;
};
struct Params {
  Prob pr[2];
  int nprob;
  int n_tiles;
  int* status;
};

// ---- packed f32x2 arithmetic (sm_100): two IEEE single-precision ops per instruction ----
MB_DEV uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
MB_DEV uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
MB_DEV uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
MB_DEV uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
MB_DEV uint32_t bf16x2_of(uint64_t v) {  // low float -> low half
  uint32_t r;
  asm("{\n .reg .f32 lo, hi;\n mov.b64 {lo, hi}, %1;\n cvt.rn.bf16x2.f32 %0, hi, lo;\n}\n" : "=r"(r) : "l"(v));
  return r;
}

// ---- Q4_K helpers ----
MB_DEV uint32_t sbyte(uint32_t sy, uint32_t sz, uint32_t sw, int k) {
  uint32_t w = k < 4 ? sy : (k < 8 ? sz : sw);
  return (w >> ((k & 3) * 8)) & 0xFFu;
}
MB_DEV void q4k_scale_min(int j, uint32_t sy, uint32_t sz, uint32_t sw, int& sc, int& m) {
  if (j < 4) {
    sc = sbyte(sy, sz, sw, j) & 63;
    m = sbyte(sy, sz, sw, j + 4) & 63;
  } else {
    sc = (sbyte(sy, sz, sw, j + 4) & 0xF) | ((sbyte(sy, sz, sw, j - 4) >> 6) << 4);
    m = (sbyte(sy, sz, sw, j + 4) >> 4) | ((sbyte(sy, sz, sw, j) >> 6) << 4);
  }
}
MB_DEV float h16(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu))); }

// 4 values (one per byte of `b`, 0..255) -> 2 packed bf16x2 of (d1*b) - m1, each op rounded
// once: d1*b = fma(d1, 2^23 + b, -d1*2^23) is the correctly rounded product.
MB_DEV void dq4(uint32_t b, uint64_t d1, uint64_t c1, uint64_t m1, uint32_t& o0, uint32_t& o1) {
  const float f0 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7440));
  const float f1 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7441));
  const float f2v = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7442));
  const float f3 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7443));
  o0 = bf16x2_of(fsub2(ffma2(d1, f2(f0, f1), c1), m1));
  o1 = bf16x2_of(fsub2(ffma2(d1, f2(f2v, f3), c1), m1));
}

// 4 int8 (bytes of q) -> 2 packed bf16x2 of d*q (exact product, one rounding to bf16).
MB_DEV void dq8(uint32_t q, uint64_t d, uint32_t& o0, uint32_t& o1) {
  const uint32_t b = q ^ 0x80808080u;  // bias to 0..255
  const uint64_t kBias = f2(8388736.f, 8388736.f);  // 2^23 + 128
  const float f0 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7440));
  const float f1 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7441));
  const float f2v = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7442));
  const float f3 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7443));
  o0 = bf16x2_of(fmul2(fsub2(f2(f0, f1), kBias), d));
  o1 = bf16x2_of(fmul2(fsub2(f2(f2v, f3), kBias), d));
}

// ---- packed decoders for the GEMM's per-thread 32-value units (o[16] = 16 bf16 pairs) ----
// 2^23 + b for the four bytes of `b` (each 0..255) as floats.
MB_DEV void magic4(uint32_t b, float& f0, float& f1, float& f2v, float& f3) {
  f0 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7440));
  f1 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7441));
  f2v = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7442));
  f3 = __int_as_float(__byte_perm(b, 0x4B000000u, 0x7443));
}

// Q6_K unit u of a 224-byte chunk: x = (d sc) (q6 - 32); q6 - 32 = (2^23 + q6) - (2^23 + 32) exactly,
// then one rounding of the product.
MB_DEV void dq_unit_q6k(const uint8_t* c, int u, uint32_t (&o)[16]) {
  const int n = u >> 2, g = u & 3;
  const uint4* ql = (const uint4*)(c + 64 * n + 32 * (g & 1));
  const uint4* qh = (const uint4*)(c + 128 + 32 * n);
  const int8_t* sc = (const int8_t*)(c + 192 + 8 * n + 2 * g);
  const float d = h16(*(const uint16_t*)(c + 208));
  const float ds0 = d * (float)sc[0], ds1 = d * (float)sc[1];
  const int nsh = (g >> 1) * 4, hsh = 2 * g;
  const uint64_t off = f2(8388640.f, 8388640.f);  // 2^23 + 32
#pragma unroll
  for (int v = 0; v < 2; v++) {
    const uint4 L = ql[v], Hh = qh[v];
    const uint32_t lw[4] = {L.x, L.y, L.z, L.w}, hw[4] = {Hh.x, Hh.y, Hh.z, Hh.w};
    const uint64_t D = v ? f2(ds1, ds1) : f2(ds0, ds0);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t q = ((lw[i] >> nsh) & 0x0F0F0F0Fu) | (((hw[i] >> hsh) & 0x03030303u) << 4);
      float a0, a1, a2, a3;
      magic4(q, a0, a1, a2, a3);
      o[8 * v + 2 * i] = bf16x2_of(fmul2(fsub2(f2(a0, a1), off), D));
      o[8 * v + 2 * i + 1] = bf16x2_of(fmul2(fsub2(f2(a2, a3), off), D));
    }
  }
}

// Q5_K unit u of a 176-byte chunk: x = d1 q5 - m1 with d1 q5 = fma(d1, 2^23 + q5, -d1 2^23) exact.
MB_DEV void dq_unit_q5k(const uint8_t* c, int u, uint32_t (&o)[16]) {
  const uint4 h = *(const uint4*)c;
  const float d = h16(h.x), dmin = h16(h.x >> 16);
  int sc, m;
  q4k_scale_min(u, h.y, h.z, h.w, sc, m);
  const float d1 = d * (float)sc, m1 = dmin * (float)m;
  const uint64_t D1 = f2(d1, d1), C1 = f2(-(d1 * 8388608.f), -(d1 * 8388608.f)), M1 = f2(m1, m1);
  const uint4* qh = (const uint4*)(c + 16);
  const uint4* qs = (const uint4*)(c + 48 + 32 * (u >> 1));
  const int sh = (u & 1) * 4;
#pragma unroll
  for (int v = 0; v < 2; v++) {
    const uint4 Q = qs[v], Hh = qh[v];
    const uint32_t qw[4] = {Q.x, Q.y, Q.z, Q.w}, hw[4] = {Hh.x, Hh.y, Hh.z, Hh.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t q = ((qw[i] >> sh) & 0x0F0F0F0Fu) | (((hw[i] >> u) & 0x01010101u) << 4);
      dq4(q, D1, C1, M1, o[8 * v + 2 * i], o[8 * v + 2 * i + 1]);
    }
  }
}

// Q4_1 unit u (block u of a 160-byte chunk): x = d q + m with d q exact.
MB_DEV void dq_unit_q41(const uint8_t* c, int u, uint32_t (&o)[16]) {
  const uint32_t* a = (const uint32_t*)(c + u * 20);
  const float d = h16(a[0]), m = h16(a[0] >> 16);
  const uint64_t D = f2(d, d), C = f2(-(d * 8388608.f), -(d * 8388608.f)), Mm = f2(-m, -m);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t w = a[1 + i];
    // values 4i..4i+3 (low nibbles) and 16 + 4i.. (high nibbles); dq4 computes d q - (-m)
    dq4(w & 0x0F0F0F0Fu, D, C, Mm, o[2 * i], o[2 * i + 1]);
    dq4((w >> 4) & 0x0F0F0F0Fu, D, C, Mm, o[8 + 2 * i], o[8 + 2 * i + 1]);
  }
}

// b - bias for the four bytes of b (0..255; bias = 8 or 16), times d, as two packed bf16 pairs:
// both steps are exact (small integers, then an 11-bit x 5-bit product), one rounding to bf16.
MB_DEV void dq_sym(uint32_t b, uint64_t dd, uint64_t bias, uint32_t& o0, uint32_t& o1) {
  float f0, f1, f2v, f3;
  magic4(b, f0, f1, f2v, f3);
  o0 = bf16x2_of(fmul2(fsub2(f2(f0, f1), bias), dd));
  o1 = bf16x2_of(fmul2(fsub2(f2(f2v, f3), bias), dd));
}
// the low bits of nibble-packed bytes plus a fifth bit per byte from 4 bits of qh
MB_DEV uint32_t with_hi_bits(uint32_t nib, uint32_t qh4) {
  return nib | (((qh4 * 0x00204081u) & 0x01010101u) << 4);
}

// Q4_0 unit u (block u: f16 d, 16 bytes of nibbles; 18 bytes at 18u, 2-byte aligned):
// x_j = d (q_j - 8).
MB_DEV void dq_unit_q40(const uint8_t* c, int u, uint32_t (&o)[16]) {
  uint32_t w[5];
  dec::words<5>(c + u * 18, w);
  const float d = h16(w[0]);
  const uint64_t dd = f2(d, d), bias = f2(8388616.f, 8388616.f);  // 2^23 + 8
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t q = __byte_perm(w[k], w[k + 1], 0x5432);
    dq_sym(q & 0x0F0F0F0Fu, dd, bias, o[2 * k], o[2 * k + 1]);
    dq_sym((q >> 4) & 0x0F0F0F0Fu, dd, bias, o[8 + 2 * k], o[8 + 2 * k + 1]);
  }
}

// Q5_0 unit u (block u: f16 d, u32 qh, 16 bytes of nibbles; 22 bytes at 22u):
// x_j = d (q5_j - 16), fifth bit of value j = qh bit j.
MB_DEV void dq_unit_q50(const uint8_t* c, int u, uint32_t (&o)[16]) {
  uint32_t w[6];
  dec::words<6>(c + u * 22, w);
  const float d = h16(w[0]);
  const uint32_t qh = (w[0] >> 16) | (w[1] << 16);
  const uint64_t dd = f2(d, d), bias = f2(8388624.f, 8388624.f);  // 2^23 + 16
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t q = __byte_perm(w[1 + k], w[2 + k], 0x5432);
    dq_sym(with_hi_bits(q & 0x0F0F0F0Fu, (qh >> (4 * k)) & 0xFu), dd, bias, o[2 * k], o[2 * k + 1]);
    dq_sym(with_hi_bits((q >> 4) & 0x0F0F0F0Fu, (qh >> (16 + 4 * k)) & 0xFu), dd, bias, o[8 + 2 * k],
           o[8 + 2 * k + 1]);
  }
}

// Q5_1 unit u (block u: f16 d, f16 m, u32 qh, 16 bytes of nibbles; 24 bytes at 24u, 8-byte
// aligned): x_j = d q5_j + m.
MB_DEV void dq_unit_q51(const uint8_t* c, int u, uint32_t (&o)[16]) {
  const uint32_t* a = (const uint32_t*)(c + u * 24);
  const float d = h16(a[0]), m = h16(a[0] >> 16);
  const uint32_t qh = a[1];
  const uint64_t D = f2(d, d), C = f2(-(d * 8388608.f), -(d * 8388608.f)), Mm = f2(-m, -m);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t q = a[2 + k];
    dq4(with_hi_bits(q & 0x0F0F0F0Fu, (qh >> (4 * k)) & 0xFu), D, C, Mm, o[2 * k], o[2 * k + 1]);
    dq4(with_hi_bits((q >> 4) & 0x0F0F0F0Fu, (qh >> (16 + 4 * k)) & 0xFu), D, C, Mm, o[8 + 2 * k], o[8 + 2 * k + 1]);
  }
}

// Q8_0 unit u (block u, 34 bytes at 34u) of a 272-byte chunk: blocks of even u start 4-byte
// aligned, odd ones 2 bytes past a word boundary.
MB_DEV void dq_unit_q8(const uint8_t* c, int u, uint32_t (&o)[16]) {
  if ((u & 1) == 0) {
    const uint32_t* a = (const uint32_t*)(c + 34 * u);
    const float d = h16(a[0]);
    const uint64_t dd = f2(d, d);
#pragma unroll
    for (int i = 0; i < 8; i++) dq8(__byte_perm(a[i], a[i + 1], 0x5432), dd, o[2 * i], o[2 * i + 1]);
  } else {
    const uint32_t* b = (const uint32_t*)(c + 34 * u - 2);
    const float d = h16(b[0] >> 16);
    const uint64_t dd = f2(d, d);
#pragma unroll
    for (int i = 0; i < 8; i++) dq8(b[1 + i], dd, o[2 * i], o[2 * i + 1]);
  }
}

MB_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
MB_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc)^T
// One stage (4 K16 steps) in one instruction sequence for a whole converged warp: the elected
// lane issues D (+)= A[a0 + 8k] * B[b0 + 32k bytes]^T for k = 0..3 (one election, one predicate).
MB_DEV void umma_ts_stage4(uint32_t d_tmem, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e, t;\n .reg .b32 r, a1, a2, a3;\n .reg .b64 b1, b2, b3;\n"
      " setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, 0, 0;\n"
      " add.u32 a1, %1, 8;\n add.u32 a2, %1, 16;\n add.u32 a3, %1, 24;\n"
      " add.u64 b1, %2, 2;\n add.u64 b2, %2, 4;\n add.u64 b3, %2, 6;\n"
      " elect.sync r|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, t;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, t;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, t;\n}\n" ::"r"(d_tmem),
      "r"(a0), "l"(b0), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same for a CTA pair (issued by the leader): A rows 0-127 come from the leader's TMEM, 128-255 from
// the peer's at the same address; B rows 0-127 from the leader's shared memory, 128-255 from the
// peer's at the same offset; each CTA's TMEM receives its own 128 rows of D.
MB_DEV void umma_ts_stage4_pair(uint32_t d_tmem, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e, t;\n .reg .b32 r, a1, a2, a3;\n .reg .b64 b1, b2, b3;\n"
      " setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, 0, 0;\n"
      " add.u32 a1, %1, 8;\n add.u32 a2, %1, 16;\n add.u32 a3, %1, 24;\n"
      " add.u64 b1, %2, 2;\n add.u64 b2, %2, 4;\n add.u64 b3, %2, 6;\n"
      " elect.sync r|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], [a1], b1, %3, t;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], [a2], b2, %3, t;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], [a3], b3, %3, t;\n}\n" ::"r"(d_tmem),
      "r"(a0), "l"(b0), "r"(idesc), "r"(accumulate)
      : "memory");
}
template <int WT, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    k_qgemm(const __grid_constant__ CUtensorMap tm_x0, const __grid_constant__ CUtensorMap tm_w0,
            const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_w1, const Params p) {
  constexpr int kSR = Cfg<WT>::kSR, SX = Cfg<WT>::kSX, kSPC = Cfg<WT>::kSPC;
  constexpr uint32_t kRawStage = TN * Cfg<WT>::kRawRow;
  constexpr uint32_t kXS = x_stage_bytes<PAIR>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* xs = smem;                                    // SX x (32 or 16) KB, 1024-aligned
  uint8_t* rs = smem + SX * kXS;                         // kSR raw stages
  uint64_t* bars = (uint64_t*)(rs + kSR * kRawStage);
  uint64_t* full = bars;         // X landed (TMA tx) and A decoded (kDW arrivals)
  uint64_t* empty = full + SX;    // the stage's MMAs completed (one commit)
  uint64_t* r_full = empty + SX;
  uint64_t* r_empty = r_full + kSR;
  uint64_t* acc_full = r_empty + kSR;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.n_tiles;
  // CTA pair (PAIR): the cluster's two CTAs share one 256 x 256 tile; rank r decodes weight rows
  // [128 r, 128 r + 128) and loads activation rows [128 r, 128 r + 128); the leader (rank 0) issues
  // the pair's MMAs. Tiles are walked per cluster.
  uint32_t rank = 0;
  if constexpr (PAIR) {
    if (cluster_size() != 2) {  // launched without the cluster shape this code needs
      if (threadIdx.x == 0) atomicExch(p.status, kDevTimeoutGemm);
      return;
    }
    rank = cluster_rank();
  }
  const bool leader = rank == 0;
  const int tile_first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int kTileN = PAIR ? 2 * TN : TN;  // weight rows per tile
  constexpr uint32_t kPairArrivals = PAIR ? 2 : 1;
  // problem of a global tile index and the tile's origin within it
#define TILE_SETUP(tile)                                                   \
  const int pi_ = (p.nprob > 1 && (tile) >= p.pr[1].tile0) ? 1 : 0;      \
  const Prob& P = p.pr[pi_];                                               \
  const int lt_ = (tile) - P.tile0;                                        \
  const int nks = P.K / BK;                                                \
  const CUtensorMap* tm_x = pi_ ? &tm_x1 : &tm_x0;                         \
  const CUtensorMap* tm_w = pi_ ? &tm_w1 : &tm_w0;                         \
  (void)tm_x;                                                              \
  (void)tm_w;                                                              \
  (void)lt_;                                                               \
  (void)nks;

  if (threadIdx.x == 0) {
    // in a pair only the leader's full / acc_empty are waited on; they count both CTAs' arrivals
    for (int i = 0; i < SX; i++) { mbar_init(&full[i], 1 + kPairArrivals * kDW); mbar_init(&empty[i], 1); }
    for (int i = 0; i < kSR; i++) { mbar_init(&r_full[i], 1); mbar_init(&r_empty[i], kDW); }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kPairArrivals * kEW);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x0);
    tma_prefetch_desc(&tm_w0);
    if (p.nprob > 1) {
      tma_prefetch_desc(&tm_x1);
      tma_prefetch_desc(&tm_w1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producers
    // lane 0 streams the activation (X) stages, lane 1 the raw weight chunks; the weight stream
    // runs ahead of X, bounded only by its own ring, so decode never waits behind the X ring.
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = tile_first; tile < n_tiles && ok; tile += tile_step) {
        TILE_SETUP(tile);
        const int m0 = (lt_ % P.tiles_m) * TM + (int)rank * (TM / 2);
        for (int ks = 0; ks < nks && ok; ks++, it++) {
          const uint32_t sx = it % SX, px = (it / SX) & 1;
          if (!(ok = (mbar_wait(&empty[sx], px ^ 1, abort_flag, p.status, kDevTimeoutGemm)))) break;
          if constexpr (PAIR) {
            // both halves complete on the leader's barrier, which expects the pair's bytes
            if (leader) mbar_expect_tx(&full[sx], 2 * kXS);
            tma_load_2d_pair(xs + sx * kXS, tm_x, smem_in_cta(&full[sx], 0), ks * BK, m0);
          } else {
            mbar_expect_tx(&full[sx], kXS);
            tma_load_2d(xs + sx * kXS, tm_x, &full[sx], ks * BK, m0);
          }
        }
      }
    } else if (lane == 1) {
      uint32_t ic = 0;
      bool ok = true;
      for (int tile = tile_first; tile < n_tiles && ok; tile += tile_step) {
        TILE_SETUP(tile);
        const int n0 = (lt_ / P.tiles_m) * kTileN + (int)rank * TN;
        for (int ks = 0; ks < nks && ok; ks += kSPC) {  // one raw chunk (kSPC stages) per 128-row block
          const uint32_t sr = ic % kSR, pr = (ic / kSR) & 1;
          ic++;
          if (!(ok = (mbar_wait(&r_empty[sr], pr ^ 1, abort_flag, p.status, kDevTimeoutGemm)))) break;
          mbar_expect_tx(&r_full[sr], kRawStage);
          uint8_t* rdst = rs + sr * kRawStage;
          if (WT == MB_GGML_Q8_0) {  // 16-bit elements
            tma_load_2d(rdst, tm_w, &r_full[sr], (ks >> 2) * (Cfg<WT>::kRawRow / 2), n0);
          } else if (WT == MB_GGML_BF16) {
            tma_load_2d(rdst, tm_w, &r_full[sr], ks * 128, n0);
          } else {  // one whole 256-value chunk (ks is a multiple of kSPC = 4)
            tma_load_2d(rdst, tm_w, &r_full[sr], (ks >> 2) * Cfg<WT>::kRawRow, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (the leader's, in a pair)
    constexpr uint32_t idesc = idesc_bf16(PAIR ? 2 * TN : TN, TM);
    uint32_t it = 0, tcount = 0;
    bool ok = true;
    for (int tile = tile_first; tile < n_tiles && ok && leader; tile += tile_step, tcount++) {
      TILE_SETUP(tile);
      if (!(ok = (PAIR ? mbar_wait_cl(acc_empty, (tcount & 1) ^ 1, abort_flag, p.status, kDevTimeoutGemm)
                            : mbar_wait(acc_empty, (tcount & 1) ^ 1, abort_flag, p.status, kDevTimeoutGemm))))
        break;
      tc_fence_after();
      for (int ks = 0; ks < nks; ks++, it++) {
        const uint32_t sx = it % SX, px = (it / SX) & 1, sa = sx;
        if (!(ok = (PAIR ? mbar_wait_cl(&full[sx], px, abort_flag, p.status, kDevTimeoutGemm)
                                             : mbar_wait(&full[sx], px, abort_flag, p.status, kDevTimeoutGemm))))
          break;
        tc_fence_after();
        {
          // The whole (converged) warp runs the issue sequence and lane 0 issues the stage's four
          // MMAs under one elect.sync (umma_ts_stage4): every instruction of the issuer costs
          // extra cycles while the decoder warps of its SM sub-partition keep that sub-partition
          // busy. Measured against a lane-0-only branch issuing one MMA per call (~537 issue
          // cycles per 512-cycle stage): one election per MMA +8-12 %, one per stage +2 % more.
          const uint32_t xaddr = smem_u32(xs + sx * kXS);
          // the descriptor's address field is bits 0-13 (bytes >> 4): +32 bytes per K16 step = +2
          static_assert(BK / 16 == 4, "one stage = four K16 MMAs");
          if constexpr (PAIR) {
            umma_ts_stage4_pair(tmem, tmem + kTmemA + sa * 32, sw128_desc(xaddr, 16, 1024), idesc, ks != 0);
            if (lane == 0) umma_commit_pair(&empty[sx], 3);
          } else {
            umma_ts_stage4(tmem, tmem + kTmemA + sa * 32, sw128_desc(xaddr, 16, 1024), idesc, ks != 0);
            if (lane == 0) umma_commit(&empty[sx]);
          }
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) {
        if constexpr (PAIR)
          umma_commit_pair(acc_full, 3);
        else
          umma_commit(acc_full);
      }
      __syncwarp();
    }
  } else if (warp < 2 + kDW) {
    // ------------------------------------------------ dequant: raw GGML -> bf16 -> TMEM
    const int q = warp & 3;               // TMEM lane quarter
    const int hh = (warp - 2) >> 2;       // K half of the stage (32 values)
    const int r = q * 32 + lane;          // weight row within the tile == TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t it = 0, ic = 0;
    bool ok = true;
    for (int tile = tile_first; tile < n_tiles && ok; tile += tile_step) {
      TILE_SETUP(tile);
      for (int kc = 0; kc < nks / kSPC && ok; kc++, ic++) {
        const uint32_t sr = ic % kSR, pr = (ic / kSR) & 1;
        if (!(ok = (mbar_wait(&r_full[sr], pr, abort_flag, p.status, kDevTimeoutGemm)))) break;
        const uint8_t* R = rs + sr * kRawStage;
        // Q4_K: this thread's four sub-blocks (2j + hh, j = 0..3) of the super-block, decoded once.
        // High nibbles (hh = 1) are used in place (16 q) with the scale divided by 16: still exact.
        float d1v[kSPC], m1v[kSPC];
        if (WT == MB_GGML_Q4_K) {
          const uint4 h = *(const uint4*)(R + r * 144);
          const float d = h16(h.x), dmin = h16(h.x >> 16);
#pragma unroll
          for (int j = 0; j < kSPC; j++) {
            int sc, mm;
            q4k_scale_min(2 * j + hh, h.y, h.z, h.w, sc, mm);
            d1v[j] = d * (float)sc;
            m1v[j] = dmin * (float)mm;
            if (hh) d1v[j] *= 0.0625f;
          }
        }
#pragma unroll
        for (int j = 0; j < kSPC; j++, it++) {
          const uint32_t sa = it % SX, pa = (it / SX) & 1;
          uint32_t o[16];
          if constexpr (WT == MB_GGML_Q4_K) {
            const uint4* qp = (const uint4*)(R + r * 144 + 16 + 32 * j);
            const uint4 qa = qp[0], qb = qp[1];
            const float d1 = d1v[j], m1 = m1v[j];
            const float c1 = -(d1 * 8388608.f);
            const uint64_t D1 = f2(d1, d1), C1 = f2(c1, c1), M1 = f2(m1, m1);
            const uint32_t mask = hh ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int i = 0; i < 8; i++) dq4(w[i] & mask, D1, C1, M1, o[2 * i], o[2 * i + 1]);
          } else if constexpr (WT == MB_GGML_Q8_0) {
            dq_unit_q8(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_BF16) {
            const uint4* src = (const uint4*)(R + r * 128 + hh * 64);
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const uint4 v = src[i];
              o[4 * i] = v.x; o[4 * i + 1] = v.y; o[4 * i + 2] = v.z; o[4 * i + 3] = v.w;
            }
          } else if constexpr (WT == MB_GGML_Q6_K) {
            dq_unit_q6k(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_Q5_K) {
            dq_unit_q5k(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_Q4_1) {
            dq_unit_q41(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_Q4_0) {
            dq_unit_q40(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_Q5_0) {
            dq_unit_q50(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else if constexpr (WT == MB_GGML_Q5_1) {
            dq_unit_q51(R + r * Cfg<WT>::kRawRow, 2 * j + hh, o);
          } else {
            float y[32];
            decode_unit<WT>(R + r * Cfg<WT>::kRawRow, 2 * j + hh, y);
#pragma unroll
            for (int i = 0; i < 16; i++) o[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
          }
          if (j == kSPC - 1) {
            // generic-proxy reads of this raw chunk are ordered before the TMA that will refill it
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_empty[sr]);
          }
          if (!(ok = (mbar_wait(&empty[sa], pa ^ 1, abort_flag, p.status, kDevTimeoutGemm)))) break;
          tc_fence_after();
          tmem_st16(tmem + lane_addr + kTmemA + sa * 32 + hh * 16, o);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR)
              mbar_arrive_cluster(smem_in_cta(&full[sa], 0));
            else
              mbar_arrive(&full[sa]);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue (thread = output feature n)
    // both CTAs of a pair release the accumulator on the leader's barrier
    auto release_acc = [](uint64_t* bar) {
      if constexpr (PAIR)
        mbar_arrive_cluster(smem_in_cta(bar, 0));
      else
        mbar_arrive(bar);
    };
    const int q = warp & 3;
    const int ch = (warp - 2 - kDW) >> 2;  // which 128 of the tile's 256 activation rows
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t tcount = 0;
    bool ok = true;
    for (int tile = tile_first; tile < n_tiles && ok; tile += tile_step, tcount++) {
      TILE_SETUP(tile);
      const GemmEpilogue& e = P.epi;
      const int m0 = (lt_ % P.tiles_m) * TM + ch * 128, n0 = (lt_ / P.tiles_m) * kTileN + (int)rank * TN;
      const int n = n0 + q * 32 + lane;
      // per-feature epilogue operands are loaded before the accumulator wait (off the drain path)
      const bool nvalid = n < P.N;
      const float bias = (nvalid && e.bias) ? e.bias[n] : 0.f;
      const float gate = (nvalid && e.kind == MB_EPI_GATE_RESIDUAL) ? e.gate[n] : 0.f;
      if (!(ok = (mbar_wait(acc_full, tcount & 1, abort_flag, p.status, kDevTimeoutGemm)))) break;
      tc_fence_after();
      const bool do_gelu = e.kind == MB_EPI_GELU_TANH && n >= e.gelu_from;
      const bool fast_bf16 = e.out_bf16 && e.kind != MB_EPI_GATE_RESIDUAL && (P.N & 1) == 0;
      if (fast_bf16) {
        // bf16 output: pack the warp's 128 accumulator columns to bf16 pairs (rows m, m+1 of
        // feature n), park them in the TMEM staging columns, free the accumulator, then read them
        // back 16 words at a time and store 32-bit words: lanes 2j / 2j+1 exchange halves so each
        // writes features (n, n+1) of one row.
        const uint32_t stage = tmem + lane_addr + kTmemStage + ch * 64;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_addr + ch * 128 + c * 32, v);
          tmem_wait_ld();
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            float a0 = __uint_as_float(v[2 * j]) + bias, a1 = __uint_as_float(v[2 * j + 1]) + bias;
            if (do_gelu) {
              a0 = gelu_tanh(a0);
              a1 = gelu_tanh(a1);
            }
            o[j] = pack_bf16x2(a0, a1);
          }
          tmem_st16(stage + c * 16, o);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(acc_empty);
        const bool odd = lane & 1;
        const int ncol = n - (odd ? 1 : 0);  // even feature of the pair this lane writes
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t pk[16];
          tmem_ld16(stage + c * 16, pk);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const uint32_t r = pk[j];
            const uint32_t r2 = __shfl_xor_sync(0xffffffffu, r, 1);
            // even lane: (own lo, partner lo) = row m ; odd lane: (partner hi, own hi) = row m + 1
            const uint32_t wv = odd ? __byte_perm(r2, r, 0x7632) : __byte_perm(r, r2, 0x5410);
            const int m = m0 + c * 32 + 2 * j + (odd ? 1 : 0);
            if (m < P.M && ncol < P.N)
              *(uint32_t*)((__nv_bfloat16*)e.y + (int64_t)m * e.ldy + ncol) = wv;
          }
        }
      } else if (e.kind == MB_EPI_GATE_RESIDUAL) {
        // f32 residual output: u = gate * (acc + bias) is parked in the TMEM staging columns as
        // packed bf16 pairs (rows m, m+1), the accumulator is freed, then y = residual + u in f32.
        const uint32_t stage = tmem + lane_addr + kTmemStage + ch * 64;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_addr + ch * 128 + c * 32, v);
          tmem_wait_ld();
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; j++)
            o[j] = pack_bf16x2(gate * (__uint_as_float(v[2 * j]) + bias), gate * (__uint_as_float(v[2 * j + 1]) + bias));
          tmem_st16(stage + c * 16, o);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(acc_empty);
        // y usually aliases res: issue a batch of 16 residual loads before any store so their
        // latencies overlap (the compiler cannot reorder loads past aliasing stores). The TMEM
        // reads stay warp-uniform; only the global accesses depend on the lane's feature.
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t pk[16];
          tmem_ld16(stage + c * 16, pk);
          tmem_wait_ld();
          if (nvalid) {
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
              float rv[16];
#pragma unroll
              for (int i = 0; i < 16; i++) {
                const int m = m0 + c * 32 + hb * 16 + i;
                rv[i] = m < P.M ? e.res[(int64_t)m * e.ldr + n] : 0.f;
              }
#pragma unroll
              for (int i = 0; i < 16; i++) {
                const int m = m0 + c * 32 + hb * 16 + i;
                const uint32_t r = pk[hb * 8 + (i >> 1)];
                if (m < P.M) ((float*)e.y)[(int64_t)m * e.ldy + n] = rv[i] + ((i & 1) ? bf16_hi(r) : bf16_lo(r));
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_addr + ch * 128 + c * 32, v);
          tmem_wait_ld();
          if (c == 3) {  // the accumulator is free as soon as the last columns are in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(acc_empty);
          }
          const int mb = m0 + c * 32;
          if (nvalid) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
              const int m = mb + i;
              if (m < P.M) {
                float a = __uint_as_float(v[i]) + bias;
                if (e.kind == MB_EPI_GATE_RESIDUAL) {
                  const float rv = e.res[(int64_t)m * e.ldr + n];
                  ((float*)e.y)[(int64_t)m * e.ldy + n] = rv + gate * a;
                } else {
                  if (do_gelu) a = gelu_tanh(a);
                  if (e.out_bf16)
                    ((__nv_bfloat16*)e.y)[(int64_t)m * e.ldy + n] = __float2bfloat16_rn(a);
                  else
                    ((float*)e.y)[(int64_t)m * e.ldy + n] = a;
                }
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // a pair's CTAs stay resident until neither can still be reached by the other's arrivals,
  // commits or MMA operand reads
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, kTmemCols);
    else
      tmem_dealloc(tmem, kTmemCols);
  }
}


template <int WT, bool PAIR>
bool make_maps(const mb_weight* w, const void* x, int64_t M, int64_t ldx, CUtensorMap* tx, CUtensorMap* tw) {
  if (!make_tmap_2d(tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)w->n_cols, (uint64_t)M, (uint64_t)ldx * 2, BK,
                    PAIR ? TM / 2 : TM, CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  const uint64_t rb = (uint64_t)w->row_bytes, nr = (uint64_t)w->n_rows;
  const uint32_t box = (uint32_t)Cfg<WT>::kRawRow;
  if (WT == MB_GGML_Q8_0)  // 16-bit elements: the 272-byte box is 136 wide
    return make_tmap_2d(tw, w->dev, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, rb / 2, nr, rb, box / 2, TN,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
  return make_tmap_2d(tw, w->dev, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rb, nr, rb, box, TN, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// 1 (default): CTA pairs (cta_group::2); 0: one CTA per tile (MB_GEMM_PAIR=0). Both give
// bit-identical results. Read once per process.
int gemm_pair_mode() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("MB_GEMM_PAIR");
    mode = (e && e[0] == '0') ? 0 : 1;
  }
  return mode;
}

// Launches one persistent kernel over the tiles of n (1 or 2) GEMMs with the same weight type.
template <int WT, bool PAIR>
cudaError_t launch_t(int n, const GemmProblem* g, cudaStream_t st) {
  constexpr int kTileN = PAIR ? 2 * TN : TN;
  CUtensorMap tx[2], tw[2];
  Params p;
  int tiles = 0;
  for (int i = 0; i < n; i++) {
    if (!make_maps<WT, PAIR>(g[i].w, g[i].x, g[i].M, g[i].ldx, &tx[i], &tw[i])) return cudaErrorInvalidValue;
    Prob& P = p.pr[i];
    P.M = (int)g[i].M;
    P.N = (int)g[i].w->n_rows;
    P.K = (int)g[i].w->n_cols;
    P.tiles_m = (int)((g[i].M + TM - 1) / TM);
    P.tiles_n = (int)((g[i].w->n_rows + kTileN - 1) / kTileN);
    P.tile0 = tiles;
    P.epi = g[i].epi;
    tiles += P.tiles_m * P.tiles_n;
  }
  if (n == 1) {
    tx[1] = tx[0];
    tw[1] = tw[0];
    p.pr[1] = p.pr[0];
  }
  p.nprob = n;
  p.n_tiles = tiles;
  p.status = device_status_ptr();
  constexpr size_t smem = smem_bytes<WT, PAIR>();
  static int attr_done[64];  // per template instance and device: 1 + the co-resident cluster count
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  if (PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemm<WT, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int slots = num_sms();
    if (PAIR) {  // pairs that fit at once (a GPC with an odd SM count leaves one SM out)
      int nc = 0;
      cfg.gridDim = dim3((unsigned)num_sms() & ~1u);
      e = cudaOccupancyMaxActiveClusters(&nc, k_qgemm<WT, PAIR>, &cfg);
      if (e != cudaSuccess) return e;
      if (nc < 1) return cudaErrorInvalidConfiguration;
      slots = nc;
    }
    attr_done[dev & 63] = 1 + slots;
  }
  const int slots = attr_done[dev & 63] - 1;
  const int units = tiles < slots ? tiles : slots;  // CTAs, or CTA pairs
  cfg.gridDim = dim3((unsigned)(PAIR ? 2 * units : units));
  return cudaLaunchKernelEx(&cfg, k_qgemm<WT, PAIR>, tx[0], tw[0], tx[1], tw[1], p);
}

template <int WT>
cudaError_t launch_w(int n, const GemmProblem* g, cudaStream_t st) {
  return gemm_pair_mode() ? launch_t<WT, true>(n, g, st) : launch_t<WT, false>(n, g, st);
}

}  // namespace gemm


cudaError_t launch_qgemm_group(int n, const GemmProblem* g, cudaStream_t st) {
  if (n < 1 || n > 2) return cudaErrorInvalidValue;
  for (int i = 0; i < n; i++)
    if (g[i].M <= 0 || g[i].w->type != g[0].w->type) return cudaErrorInvalidValue;
  switch (g[0].w->type) {
    case MB_GGML_Q4_K: return gemm::launch_w<MB_GGML_Q4_K>(n, g, st);
    case MB_GGML_Q8_0: return gemm::launch_w<MB_GGML_Q8_0>(n, g, st);
    case MB_GGML_BF16: return gemm::launch_w<MB_GGML_BF16>(n, g, st);
    case MB_GGML_Q4_0: return gemm::launch_w<MB_GGML_Q4_0>(n, g, st);
    case MB_GGML_Q4_1: return gemm::launch_w<MB_GGML_Q4_1>(n, g, st);
    case MB_GGML_Q5_0: return gemm::launch_w<MB_GGML_Q5_0>(n, g, st);
    case MB_GGML_Q5_1: return gemm::launch_w<MB_GGML_Q5_1>(n, g, st);
    case MB_GGML_Q5_K: return gemm::launch_w<MB_GGML_Q5_K>(n, g, st);
    case MB_GGML_Q6_K: return gemm::launch_w<MB_GGML_Q6_K>(n, g, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_qgemm(const mb_weight* w, const void* x_bf16, int64_t M, int64_t ldx, const GemmEpilogue& epi,
                         cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  GemmProblem g{w, x_bf16, M, ldx, epi};
  return launch_qgemm_group(1, &g, st);
}

}  // namespace mb
