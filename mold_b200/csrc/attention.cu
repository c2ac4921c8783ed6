// K4: non-causal flash attention, head_dim 128, bf16 in / f32 accumulate, on tcgen05 + TMEM (sm_100a).
//
// Replaces scaled_dot_product_attention (flux/offload.rs:40-54, which materialises
// the [H, L, L] score matrix) and Qwen's masked attention
// (qwen_image/quantized_transformer.rs:799-816) without ever forming L x L.
//
// One CTA = 128 query rows of one head. Warp roles (192 threads):
//   warp 0   TMA: Q once, then K_j and V_j (128 keys each) into a 2-deep ring.
//   warp 1   MMA: S_j = Q K_j^T into TMEM (two S buffers, so S_{j+1} runs on the
//            tensor core while softmax works on S_j), then O += P_j V_j with O in TMEM.
//   warps 2-5 softmax, one thread per query row (= TMEM lane): row max, exp2,
//            row sum, P_j (bf16) into shared memory in the UMMA K-major 128B-swizzled
//            layout. O is rescaled lazily: only when the running max grows by more
//            than 2^8 (FA4-style), which leaves the final O / l unchanged.
// V is consumed in its natural [keys, d] layout as an MN-major B operand.
#include "common.cuh"
#include "internal.h"

namespace mb {
namespace attn {

constexpr int BQ = 128, BKV = 128, D = 128;
constexpr int kThreads = 192;
constexpr uint32_t kTile = 128 * 128 * 2;  // 32 KB: one 128x128 bf16 tile (two 64-wide swizzle atoms)
constexpr uint32_t kHalf = kTile / 2;      // 16 KB: one 64-wide atom column
constexpr size_t kSmem = 1024 + 7 * (size_t)kTile + 256;
constexpr float kScaleLog2 = 0.12751743082459868f;  // log2(e) / sqrt(128)
constexpr float kRescaleThreshold = 8.f;

struct Params {
  int H, Lq, Lk, n_valid, n_kv;
  __nv_bfloat16* out;
  int64_t ldo;
  int* status;
};

__global__ void __launch_bounds__(kThreads, 1)
    k_attention(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTile;          // 2 stages
  uint8_t* sV = smem + 3 * kTile;      // 2 stages
  uint8_t* sP = smem + 5 * kTile;      // 2 buffers
  uint64_t* bars = (uint64_t*)(smem + 7 * kTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* v_full = bars + 3;   // [2]
  uint64_t* kv_empty = bars + 5; // [2]
  uint64_t* s_full = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;   // [2]
  uint64_t* p_empty = bars + 11; // [2]
  uint64_t* o_full = bars + 13;
  uint32_t* tmem_slot = (uint32_t*)(bars + 14);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, q0 = blockIdx.x * BQ;
  const int n_kv = p.n_kv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(o_full, 1);
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
  const uint32_t tS = tmem, tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_expect_tx(q_full, kTile);
      tma_load_3d(sQ, &tq, q_full, 0, q0, h);
      tma_load_3d(sQ + kHalf, &tq, q_full, 64, q0, h);
      for (int j = 0; j < n_kv; j++) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1, abort_flag, p.status, kDevTimeoutAttn)) break;
        mbar_expect_tx(&k_full[s], kTile);
        tma_load_3d(sK + s * kTile, &tk, &k_full[s], 0, j * BKV, h);
        tma_load_3d(sK + s * kTile + kHalf, &tk, &k_full[s], 64, j * BKV, h);
        mbar_expect_tx(&v_full[s], kTile);
        tma_load_3d(sV + s * kTile, &tv, &v_full[s], 0, j * BKV, h);
        tma_load_3d(sV + s * kTile + kHalf, &tv, &v_full[s], 64, j * BKV, h);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = idesc_bf16(BQ, BKV, false);
    constexpr uint32_t idesc_o = idesc_bf16(BQ, D, true);
    bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kDevTimeoutAttn);
    const uint32_t qa = smem_u32(sQ);
    for (int j = 0; j <= n_kv && ok; j++) {
      if (j < n_kv) {
        const int s = j & 1;
        if (!(ok = mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ka = smem_u32(sK + s * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; kk++) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_f16(tS + s * 128, sw128_desc(qa + off, 16, 1024), sw128_desc(ka + off, 16, 1024), idesc_s, kk > 0);
          }
          umma_commit(&s_full[s]);
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int jj = j - 1, b = jj & 1;
        const uint32_t ph = (jj >> 1) & 1;
        if (!(ok = mbar_wait(&p_full[b], ph, abort_flag, p.status, kDevTimeoutAttn))) break;
        if (!(ok = mbar_wait(&v_full[b], ph, abort_flag, p.status, kDevTimeoutAttn))) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t pa = smem_u32(sP + b * kTile), va = smem_u32(sV + b * kTile);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; kk++) {
            const uint64_t adesc = sw128_desc(pa + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            // V [keys, d]: MN-major; 64-wide d chunks kHalf apart (LBO), 8-key groups 1024 B apart (SBO).
            const uint64_t bdesc = sw128_desc(va + kk * 16 * 128, kHalf, 1024);
            umma_f16(tO, adesc, bdesc, idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&p_empty[b]);
          umma_commit(&kv_empty[b]);
        }
        __syncwarp();
      }
    }
    if (ok && lane == 0) umma_commit(o_full);
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; j++) {
      const int s = j & 1;
      if (!(ok = mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))) break;
      tc_fence_after();
      const int valid = p.n_valid - j * BKV;  // keys >= valid are masked in this block
      const uint32_t sa = tS + s * 128 + lane_addr;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld32(sa + c * 32, v);
        tmem_wait_ld();
        if (valid >= BKV) {
#pragma unroll
          for (int i = 0; i < 32; i++) mx = fmaxf(mx, __uint_as_float(v[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (c * 32 + i < valid) mx = fmaxf(mx, __uint_as_float(v[i]));
        }
      }
      const float m_new = fmaxf(m_run, mx * kScaleLog2);
      if (j == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const int jp = j - 1;
          if (!(ok = mbar_wait(&p_empty[jp & 1], (jp >> 1) & 1, abort_flag, p.status, kDevTimeoutAttn))) break;
          tc_fence_after();
          const float alpha = need ? ex2_approx(m_run - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < 4; c++) {
            uint32_t o[32];
            tmem_ld32(tO + lane_addr + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + lane_addr + c * 32, o);
          }
          tmem_wait_st();
          l_run *= alpha;
          if (need) m_run = m_new;
        }
      }
      if (j >= 2) {
        if (!(ok = mbar_wait(&p_empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status, kDevTimeoutAttn))) break;
      }
      uint8_t* prow = sP + s * kTile + r * 128;
      const int sw = r & 7;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld32(sa + c * 32, v);
        tmem_wait_ld();
        float e[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const float x = __uint_as_float(v[i]) * kScaleLog2 - m_run;
          e[i] = (valid >= BKV || c * 32 + i < valid) ? ex2_approx(x) : 0.f;
          sum += e[i];
        }
        // keys c*32 .. c*32+31 -> atom column (c >> 1), 16-byte chunks (c & 1)*4 .. +3
        uint8_t* base = prow + (c >> 1) * kHalf;
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const int chunk = (c & 1) * 4 + t;
          uint4 u;
          u.x = pack_bf16x2(e[8 * t + 0], e[8 * t + 1]);
          u.y = pack_bf16x2(e[8 * t + 2], e[8 * t + 3]);
          u.z = pack_bf16x2(e[8 * t + 4], e[8 * t + 5]);
          u.w = pack_bf16x2(e[8 * t + 6], e[8 * t + 7]);
          *(uint4*)(base + ((chunk ^ sw) << 4)) = u;
        }
      }
      l_run += sum;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    if (ok) ok = mbar_wait(o_full, 0, abort_flag, p.status, kDevTimeoutAttn);
    if (ok) {
      tc_fence_after();
      const int qrow = q0 + r;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)qrow * p.ldo + (int64_t)h * D;
#pragma unroll 1
      for (int c = 0; c < 4; c++) {
        uint32_t o[32];
        tmem_ld32(tO + lane_addr + c * 32, o);
        tmem_wait_ld();
        if (qrow < p.Lq) {
#pragma unroll
          for (int t = 0; t < 4; t++) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(o[8 * t + 0]) * inv, __uint_as_float(o[8 * t + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(o[8 * t + 2]) * inv, __uint_as_float(o[8 * t + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(o[8 * t + 4]) * inv, __uint_as_float(o[8 * t + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(o[8 * t + 6]) * inv, __uint_as_float(o[8 * t + 7]) * inv);
            *(uint4*)(orow + c * 32 + t * 8) = u;
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
                             int64_t n_valid, void* out, int64_t ldo, cudaStream_t st) {
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
  dim3 grid((unsigned)((Lq + BQ - 1) / BQ), (unsigned)H);
  k_attention<<<grid, kThreads, kSmem, st>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace mb
