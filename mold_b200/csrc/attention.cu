// K4: non-causal flash attention, head_dim 128, bf16 in / f32 accumulate, on tcgen05 + TMEM (sm_100a).
//
// Replaces scaled_dot_product_attention (flux/offload.rs:40-54, which materialises
// the [H, L, L] score matrix) and Qwen's masked attention
// (qwen_image/quantized_transformer.rs:799-816) without ever forming L x L.
//
// One CTA = 256 query rows (two 128-row tiles) of one head, sharing every K/V block.
//   warp 0      TMA: both Q tiles once, then K_j and V_j (128 keys) into a 2-deep ring.
//   warps 1, 2  MMA issuers of tile 0 and tile 1. Each KV block is processed as two 64-key
//               sub-blocks whose scores go to the two halves of the tile's S columns, so the
//               tensor core computes S(g + 1) while the softmax works on S(g): per tile, per
//               sub-block g, PV_t(g) then S_t(g + 2).
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: one thread per query row
//               (= TMEM lane) holding the sub-block's 64 scores in registers. Row max, exp2, row
//               sum; P (bf16) is written back into TMEM over the first 32 columns of the S half and consumed
//               directly as the A operand of O += P V (O in TMEM). O is rescaled lazily, only
//               when the row max grows by more than 2^8, which leaves the final O / l unchanged.
//               A fixed share of each row's exp2 is evaluated with a polynomial on the FMA
//               pipe instead of the MUFU unit (which alone would cap the kernel).
//               Two softmax warps per SM sub-partition (not four): every always-ready warp beside
//               the MMA issuer on its sub-partition slows tcgen05.mma issue by ~25 cycles per
//               instruction, and at 64 tensor cycles per 128x128x16 MMA the issuer has no slack.
// TMEM (512 columns): S_0 [0,128) (halves of 64), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// V is consumed in its natural [keys, d] layout as an MN-major B operand.
#include "common.cuh"
#include "internal.h"

namespace mb {
namespace attn {

constexpr int BQ = 128, BKV = 128, D = 128, NT = 2;
constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4-7 softmax tile 0, 8-11 tile 1
constexpr uint32_t kTile = 128 * 128 * 2;  // 32 KB: one 128x128 bf16 tile (two 64-wide swizzle atoms)
constexpr uint32_t kHalf = kTile / 2;      // 16 KB: one 64-wide atom column
constexpr size_t kSmem = 1024 + 6 * (size_t)kTile + 256;
constexpr float kScaleLog2 = 0.12751743082459868f;  // log2(e) / sqrt(128)
constexpr float kRescaleThreshold = 8.f;
#ifndef MB_ATTN_POLY
#define MB_ATTN_POLY 6
#endif
constexpr int kPolyPerChunk = MB_ATTN_POLY;  // of every 32 exponentials, this many use the FMA-pipe polynomial

struct Params {
  int H, Lq, Lk, n_valid, n_kv;
  __nv_bfloat16* out;   // rows [0, split)
  __nv_bfloat16* out2;  // rows [split, Lq), from its row 0
  int64_t ldo;
  int split;
  int* status;
};

// ---- packed f32x2 helpers (sm_100): two IEEE single-precision ops per instruction
MB_DEV uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
MB_DEV void up2(uint64_t v, float& a, float& b) { asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
MB_DEV uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
MB_DEV uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
MB_DEV uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
MB_DEV float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// 2^x for a pair by a degree-3 polynomial (own minimax fit of 2^f on [-1/2, 1/2], max relative
// error 7.5e-5, far below the bf16 rounding P is stored with): x is clamped to >= -126 (masked
// keys give ~1e-38), rounded to n by the 1.5 * 2^23 trick, and 2^n enters the exponent field.
MB_DEV void exp2_poly3(uint64_t x2, float& e0, float& e1) {
  float a, b;
  up2(x2, a, b);
  a = fmaxf(a, -126.f);
  b = fmaxf(b, -126.f);
  const uint64_t xc = pk2(a, b);
  const uint64_t magic = pk2(12582912.f, 12582912.f);
  const uint64_t t2 = add2(xc, magic);
  const uint64_t f = sub2(xc, sub2(t2, magic));
  uint64_t p = fma2(pk2(0.05517132207751274f, 0.05517132207751274f), f, pk2(0.24261054396629333f, 0.24261054396629333f));
  p = fma2(p, f, pk2(0.6932609677314758f, 0.6932609677314758f));
  p = fma2(p, f, pk2(0.9999281167984009f, 0.9999281167984009f));
  float t0, t1, p0, p1;
  up2(t2, t0, t1);
  up2(p, p0, p1);
  e0 = __int_as_float(__float_as_int(p0) + (int)((uint32_t)__float_as_int(t0) << 23));
  e1 = __int_as_float(__float_as_int(p1) + (int)((uint32_t)__float_as_int(t1) << 23));
}

MB_DEV void tmem_st16a(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Elected-lane forms for a converged warp (lane 0 issues): cheaper to issue than a lane-0 branch.
MB_DEV void umma_ss_elect(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n .reg .b32 r;\n setp.ne.b32 p, %4, 0;\n elect.sync r|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
MB_DEV void umma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n .reg .b32 r;\n setp.ne.b32 p, %4, 0;\n elect.sync r|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}



__global__ void __launch_bounds__(kThreads, 1)
    k_attention(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                  // 2 tiles
  uint8_t* sK = smem + 2 * kTile;      // 2 stages
  uint8_t* sV = smem + 4 * kTile;      // 2 stages
  uint64_t* bars = (uint64_t*)(smem + 6 * kTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2] per stage
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [tile][half]
  uint64_t* p_full = bars + 11;   // [tile][half]
  uint64_t* o_full = bars + 15;   // [tile]
  uint64_t* pv_done = bars + 17;  // [tile]: one completion per P V sub-block
  uint32_t* tmem_slot = (uint32_t*)(bars + 19);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, q0 = blockIdx.x * (NT * BQ);
  const int n_kv = p.n_kv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 2);  // one commit per MMA issuer
      mbar_init(&o_full[i], 1);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_expect_tx(q_full, 2 * kTile);
      for (int t = 0; t < NT; t++) {
        tma_load_3d(sQ + t * kTile, &tq, q_full, 0, q0 + t * BQ, h);
        tma_load_3d(sQ + t * kTile + kHalf, &tq, q_full, 64, q0 + t * BQ, h);
      }
      for (int j = 0; j < n_kv; j++) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!(mbar_wait(&kv_empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutAttn))) break;
        mbar_expect_tx(&k_full[s], kTile);
        tma_load_3d(sK + s * kTile, &tk, &k_full[s], 0, j * BKV, h);
        tma_load_3d(sK + s * kTile + kHalf, &tk, &k_full[s], 64, j * BKV, h);
        mbar_expect_tx(&v_full[s], kTile);
        tma_load_3d(sV + s * kTile, &tv, &v_full[s], 0, j * BKV, h);
        tma_load_3d(sV + s * kTile + kHalf, &tv, &v_full[s], 64, j * BKV, h);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // MMA issuer of tile t = warp - 1 (the two issuers sit on different SM sub-partitions).
    // Sub-block g = 2j + hh covers keys 64hh .. 64hh+63 of K/V stage j; its scores go to the
    // tile's S half hh, so S_t(g + 2) is issued while the softmax works on S_t(g + 1).
    const int t = warp - 1;
    constexpr uint32_t idesc_s = idesc_bf16(BQ, 64, false);
    constexpr uint32_t idesc_o = idesc_bf16(BQ, D, true);
    const uint32_t qa = smem_u32(sQ) + t * kTile;
    const int n_sub = 2 * n_kv;
    bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kDevTimeoutAttn);
    // S_t(g) = Q_t K_g^T (64 keys) into S half g & 1
    auto issue_s = [&](int g) {
      const int hh = g & 1;
      {
        const uint32_t ka = smem_u32(sK + ((g >> 1) & 1) * kTile) + hh * 8192;
#pragma unroll
        for (int kk = 0; kk < D / 16; kk++) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          umma_ss_elect(tmem + t * 128 + hh * 64, sw128_desc(qa + off, 16, 1024), sw128_desc(ka + off, 16, 1024),
                        idesc_s, kk > 0);
        }
        if (lane == 0) umma_commit(&s_full[t * 2 + hh]);
      }
      __syncwarp();
    };
    // O_t += P_t(g) V_g with P read from TMEM (bf16 pairs over the first 32 columns of S half g & 1)
    auto issue_pv = [&](int g) {
      const int hh = g & 1;
      {
        const uint32_t va = smem_u32(sV + ((g >> 1) & 1) * kTile);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          // V [keys, d]: MN-major; 64-wide d chunks kHalf apart (LBO), 8-key groups 1024 B apart (SBO).
          const uint64_t bdesc = sw128_desc(va + (hh * 4 + kk) * 16 * 128, kHalf, 1024);
          umma_ts_elect(tmem + 256 + t * 128, tmem + t * 128 + hh * 64 + kk * 8, bdesc, idesc_o,
                        (g > 0 || kk > 0) ? 1u : 0u);
        }
        if (lane == 0) {
          umma_commit(&pv_done[t]);
          if (hh == 1) umma_commit(&kv_empty[(g >> 1) & 1]);
        }
      }
      __syncwarp();
    };
    if (ok && n_kv > 0) {
      if ((ok = mbar_wait(&k_full[0], 0, abort_flag, p.status, kDevTimeoutAttn))) {
        tc_fence_after();
        issue_s(0);
        issue_s(1);
      }
    }
    for (int g = 0; g < n_sub && ok; g++) {
      const int hh = g & 1, j = g >> 1;
      if (hh == 0 && !(ok = (mbar_wait(&v_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))))
        break;
      if (!(ok = (mbar_wait(&p_full[t * 2 + hh], j & 1, abort_flag, p.status, kDevTimeoutAttn)))) break;
      tc_fence_after();
      issue_pv(g);
      if (g + 2 < n_sub) {
        if (hh == 0 &&
            !(ok = (mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))))
          break;
        tc_fence_after();
        issue_s(g + 2);
      }
    }
    if (ok && lane == 0) umma_commit(&o_full[t]);
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- softmax
    // 4 warps per tile; thread = query row = TMEM lane (warp w may only touch lanes 32 (w % 4) ..).
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_addr, tO = tmem + 256 + t * 128 + lane_addr;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int g = 0; g < 2 * n_kv; g++) {
      const int hh = g & 1;
      if (!(ok = (mbar_wait(&s_full[t * 2 + hh], (g >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))))
        break;
      tc_fence_after();
      const uint32_t tSh = tS + hh * 64;
      const int valid = p.n_valid - g * 64;  // keys >= valid are masked
      uint32_t v[2][32];
      tmem_ld32(tSh, v[0]);
      tmem_ld32(tSh + 32, v[1]);
      tmem_wait_ld();
      if (valid < 64) {
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (c * 32 + i >= valid) v[c][i] = __float_as_uint(-INFINITY);
      }
      // row max of the 64 keys: two independent max3 chains
      float mc[2];
#pragma unroll
      for (int c = 0; c < 2; c++) {
        mc[c] = fmaxf(__uint_as_float(v[c][0]), __uint_as_float(v[c][1]));
#pragma unroll
        for (int i = 2; i < 32; i += 2) mc[c] = max3(mc[c], __uint_as_float(v[c][i]), __uint_as_float(v[c][i + 1]));
      }
      const float mx = fmaxf(mc[0], mc[1]);
      const float m_new = fmaxf(m_run, mx * kScaleLog2);
      // lazy rescale: only rows whose max grew by more than 2^8 move their reference point
      const bool need = g == 0 || m_new > m_run + kRescaleThreshold;
      const float alpha = (need && g > 0) ? ex2_approx(m_run - m_new) : 1.f;
      if (need) m_run = m_new;
      const uint64_t sc2 = pk2(kScaleLog2, kScaleLog2), nm2 = pk2(-m_run, -m_run);
      uint64_t sum2 = pk2(0.f, 0.f);
      // exponentials, 32 keys at a time; P of keys 32c .. 32c+31 (16 bf16 pairs) goes to columns
      // [16c, 16c + 16) of the S half, all of which were read above
#pragma unroll
      for (int c = 0; c < 2; c++) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const uint64_t x2 = fma2(pk2(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), sc2, nm2);
          float e0, e1;
          if (2 * i < kPolyPerChunk) {
            exp2_poly3(x2, e0, e1);
          } else {
            float x0, x1;
            up2(x2, x0, x1);
            e0 = ex2_approx(x0);
            e1 = ex2_approx(x1);
          }
          sum2 = add2(sum2, pk2(e0, e1));
          pk[i] = pack_bf16x2(e0, e1);
        }
        tmem_st16a(tSh + c * 16, pk);
      }
      float sa, sb;
      up2(sum2, sa, sb);
      if (g > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O_t must hold P V of sub-block g - 1 before it is rescaled (S_t(g) was issued before
        // that P V, so its completion does not imply it)
        if (!(ok = mbar_wait(&pv_done[t], (g - 1) & 1, abort_flag, p.status, kDevTimeoutAttn))) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_wait_st();
      l_run = l_run * alpha + (sa + sb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t * 2 + hh]);
    }
    if (ok) ok = mbar_wait(&o_full[t], 0, abort_flag, p.status, kDevTimeoutAttn);
    if (ok) {
      tc_fence_after();
      const int qrow = q0 + t * BQ + r;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow =
          (qrow < p.split ? p.out + (int64_t)qrow * p.ldo : p.out2 + (int64_t)(qrow - p.split) * p.ldo) + (int64_t)h * D;
#pragma unroll 1
      for (int c = 0; c < 4; c++) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
        if (qrow < p.Lq) {
#pragma unroll
          for (int u = 0; u < 4; u++) {
            uint4 w4;
            w4.x = pack_bf16x2(__uint_as_float(o[8 * u + 0]) * inv, __uint_as_float(o[8 * u + 1]) * inv);
            w4.y = pack_bf16x2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv);
            w4.z = pack_bf16x2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv);
            w4.w = pack_bf16x2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv);
            *(uint4*)(orow + c * 32 + u * 8) = w4;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn


cudaError_t launch_attention(const void* q, const void* k, const void* v, int H, int64_t Lq, int64_t Lk,
                             int64_t n_valid, void* out, int64_t ldo, cudaStream_t st, int64_t split_row,
                             void* out2) {
  using namespace attn;
  CUtensorMap tq, tk, tv;
  const uint64_t rs = D * 2;
  if (!make_tmap_3d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)Lq, (uint64_t)H, rs, rs * Lq, 64, BQ, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)Lk, (uint64_t)H, rs, rs * Lk, 64, BKV, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, (uint64_t)Lk, (uint64_t)H, rs, rs * Lk, 64, BKV, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  Params p;
  p.H = H;
  p.Lq = (int)Lq;
  p.Lk = (int)Lk;
  p.n_valid = (int)n_valid;
  p.n_kv = (int)((n_valid + BKV - 1) / BKV);
  p.out = (__nv_bfloat16*)out;
  p.out2 = (__nv_bfloat16*)(out2 ? out2 : out);
  p.split = (split_row < 0 || split_row > Lq) ? (int)Lq : (int)split_row;
  p.ldo = ldo;
  p.status = device_status_ptr();
  static int attr_done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return e;
    attr_done[dev & 63] = 1;
  }
  dim3 grid((unsigned)((Lq + NT * BQ - 1) / (NT * BQ)), (unsigned)H);
  k_attention<<<grid, kThreads, kSmem, st>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace mb
