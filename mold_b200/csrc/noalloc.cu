// mb_qlinear_f32_static: the f32-input quantized linear without any device allocation.
//
// mb_qlinear with an f32 x first casts x to bf16 into a per-device scratch buffer
// that the library grows with cudaMalloc. Some callers cannot allow that: callers
// whose device memory is handed out by their own pool or arena and must not be
// fragmented or grown behind their back, and hosts that forbid allocation after
// start-up (a fixed memory budget per process, measured once at start). This entry point
// stages the bf16 copy of x in a fixed array that lives in the library's own
// device image instead, so it never calls cudaMalloc, cudaFree or any allocating
// routine.
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace mb {
namespace {

// Staging buffer for the bf16 copy of x: 8 MiB = 4,194,304 bf16 values (M * K).
// Every GPU that loads the library holds it until the process exits. All calls on a
// device share it, so calls whose execution overlaps on the GPU race on it.
constexpr size_t kStaticElems = (size_t)4 << 20;
static __device__ __align__(256) __nv_bfloat16 g_static_x[kStaticElems];

// Host code cannot use g_static_x's name as a device address; the address is looked
// up once per device (with that device current) and cached here.
std::mutex g_mu;
void* g_addr[64];

cudaError_t static_buffer(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_x);
    if (e != cudaSuccess) return e;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" mb_status mb_qlinear_f32_static(const mb_weight* w, const float* x, int64_t M, int64_t ldx, void* y,
                                           int y_dtype, int64_t ldy, const float* bias, int epilogue,
                                           int64_t gelu_from, const float* gate, const float* residual, int64_t ldr,
                                           void* stream) {
  MB_CHECK(w && x && y, MB_ERR_INVALID, "weight, x or y is NULL");
  MB_CHECK(M >= 0, MB_ERR_INVALID, "M must be >= 0");
  MB_CHECK(gemm_type_supported(w->type), MB_ERR_UNSUPPORTED,
           "mb_qlinear_f32_static supports BF16 and the quantized types Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, "
           "Q6_K (got ggml type " + std::to_string(w->type) + ")");
  const int64_t K = w->n_cols, N = w->n_rows;
  MB_CHECK(K > 0 && K % 64 == 0, MB_ERR_INVALID, "K must be a positive multiple of 64");
  // Bound M by division so that no product of caller-supplied sizes can wrap.
  MB_CHECK(M <= (int64_t)(kStaticElems / (size_t)K), MB_ERR_INVALID,
           "mb_qlinear_f32_static: M = " + std::to_string(M) + " rows of K = " + std::to_string(K) +
               " exceed the fixed staging buffer of " + std::to_string(kStaticElems) +
               " values (8 MiB, M * K must be <= that); use mb_qlinear for larger inputs");
  MB_CHECK(w->type == MB_GGML_BF16 || K % 256 == 0, MB_ERR_INVALID, "quantized K must be a multiple of 256");
  MB_CHECK(M < (1LL << 31) && N < (1LL << 31), MB_ERR_INVALID, "M and N must fit in 31 bits");
  MB_CHECK(ldx >= K && ldx % 4 == 0 && ((uintptr_t)x & 15) == 0, MB_ERR_INVALID,
           "x must be 16-byte aligned with ldx >= K and ldx % 4 == 0");
  MB_CHECK(ldy >= N, MB_ERR_INVALID, "ldy must be >= N");
  MB_CHECK(y_dtype == MB_DT_BF16 || y_dtype == MB_DT_F32, MB_ERR_INVALID, "y_dtype must be BF16 or F32");
  MB_CHECK(epilogue >= MB_EPI_NONE && epilogue <= MB_EPI_GATE_RESIDUAL, MB_ERR_INVALID, "unknown epilogue");
  if (epilogue == MB_EPI_GATE_RESIDUAL) {
    MB_CHECK(y_dtype == MB_DT_F32 && gate && residual && ldr >= N, MB_ERR_INVALID,
             "gate-residual epilogue needs f32 y, gate, residual and ldr >= N");
  }
  MB_CHECK(device_status_ready(), MB_ERR_NOT_READY,
           "call mb_init on this device before mb_qlinear_f32_static (mb_init does the one-time allocations)");
  if (M == 0) return MB_OK;
  void* xb = nullptr;
  MB_CUDA(static_buffer(&xb));
  cudaStream_t st = (cudaStream_t)stream;
  // The staged rows [0, M) x [0, K) are fully overwritten by the cast; nothing needs clearing.
  MB_CUDA(launch_cast_f32_bf16(x, M, K, ldx, xb, K, st));
  GemmEpilogue e;
  e.kind = epilogue;
  e.out_bf16 = y_dtype == MB_DT_BF16;
  e.gelu_from = epilogue == MB_EPI_GELU_TANH ? gelu_from : (int64_t)1 << 40;
  e.y = y;
  e.ldy = ldy;
  e.bias = bias;
  e.gate = gate;
  e.res = residual;
  e.ldr = ldr;
  MB_CUDA(launch_qgemm(w, xb, M, K, e, st));
  return MB_OK;
}
