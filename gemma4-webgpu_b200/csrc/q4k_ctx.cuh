// The library context (opaque q4k_ctx of include/q4k.h) and shared helpers of
// the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/q4k.h"
#include "q4k_engine.cuh"
#include "q4k_kernels.cuh"

struct q4k_ctx {
  int device = 0;
  int sm_count = 0;
  q4k::SelectScratch select;
  // Single-call scratch: prepared activations of one GEMV and their scales.
  uint2* xfrag = nullptr;
  size_t xfrag_cap = 0;  // bytes
  float* inv_scale = nullptr;  // [kCtxScaleSlots]: 1/scale per activation row
  unsigned long long* row_slots = nullptr;  // [kMaxSelectRows][256]: q4k_select_rows keys
  uint32_t* row_counters = nullptr;         // [kMaxSelectRows]
  void* scratch = nullptr;     // the one allocation holding all of the above
  char err[512] = {0};
};

namespace q4k {

// Prepared-activation scratch a context allocates once (q4k_create), and the
// activation rows one single call prepares at most (per-row scales).
constexpr size_t kCtxXfragBytes = 16u << 20;
constexpr uint32_t kCtxScaleSlots = 1024;

inline int ctx_fail(q4k_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->err, sizeof(ctx->err), fmt, ap);
    va_end(ap);
  }
  return code;
}

inline int ctx_cuda(q4k_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) {
    ctx->err[0] = 0;
    return Q4K_OK;
  }
  return ctx_fail(ctx, Q4K_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

inline uint32_t tiles_of(uint32_t M) { return (M + kTileRows - 1) / kTileRows; }

// q4k_gemv hands requests of at least this many activation rows to the GEMM.
constexpr uint32_t kGemmMinRows = 64;

// Batched Q4_K GEMM (tcgen05, q4k_gemm.cu): y[t][m] = sum_k w16[m][k] x[t][k]
// for T activation rows, on the context's scratch.  parts = 2: x enters as
// exact f16 hi + lo parts; parts = 1: x rounded once to f16 (after its
// power-of-two row scale), half the tensor-core work.
int run_gemm(q4k_ctx* ctx, const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
             cudaStream_t s, uint32_t parts = 2);

// ---- multi-matrix GEMM launches (plans with batch >= kGemmMinRows) ------------
// Every matrix of a plan stage runs in ONE gemm_kernel launch whose CTAs each
// take one tile (256 weight rows x a token tile) from a host-made tile table,
// after one preparation launch has turned every distinct activation of the
// stage (x, or gelu_mul(gate, up)) into its B operand.

// One matrix: y[t][m] = sum_k w16[m][k] x[t][k] for t < T, m < M.
struct alignas(16) GemmTask {
  const CUtensorMap* amap;  // the raw Q4_K matrix (gemm_weight_map), device memory
  const CUtensorMap* bmap;  // its activation operand (gemm_operand_map), device memory
  float* y;                 // [T][M]
  const float* inv_scale;   // [T]: 1/scale of each activation row (the operand's)
  uint32_t M, N, T;         // N: the K range of this task (k0 .. k0 + N)
  uint32_t tile_tokens;     // activation rows per tile (gemm_tile_tokens)
  uint32_t k0;              // first K element of the range (a multiple of 256)
  uint32_t accumulate;      // 1: add into y (zeroed by the stage's preparation), one of a K split
};

// One activation operand: mode 0 from x [T][N]; mode 1 gelu_mul(gate, up)
// [T][N] (shaders/gelu_mul.wgsl), stored to act when act != null.  Mode 2
// has no operand: it zeroes act [T][N], the output of a K-split matrix.
struct alignas(16) GemmJob {
  const float* x;
  const float* gate;
  const float* up;
  float* act;
  void* operand;     // f16 [parts*T][N] in the weight tiles' K order
  float* inv_scale;  // [T]
  uint32_t N, mode;
};

// Activation rows per token tile of a T-row launch: all of them when they
// make at most 128 operand rows (parts per activation row; the tensor-memory
// A form), else 256 operand rows.
uint32_t gemm_tile_tokens(uint32_t parts, uint32_t T);
// Rows of the weight-row tile (the A operand's M per CTA).
uint32_t gemm_tile_rows();
size_t gemm_operand_bytes(uint32_t N, uint32_t T, uint32_t parts);
cudaError_t gemm_weight_map(CUtensorMap* map, const void* w, uint32_t M, uint32_t N);
cudaError_t gemm_operand_map(CUtensorMap* map, const void* operand, uint32_t N, uint32_t T, uint32_t parts);
// One CTA per (job, token); `max_n` = the widest job, `aligned` = every
// pointer of every job 16-byte aligned (then each input is read once).
cudaError_t launch_gemm_prep(const GemmJob* jobs, uint32_t n_jobs, uint32_t T, uint32_t parts, uint32_t max_n,
                             bool aligned, int device, cudaStream_t s);
cudaError_t launch_gemm_tasks(const GemmTask* tasks, const uint2* tiles, uint32_t n_tiles, uint32_t parts,
                              uint32_t tile_tokens, uint32_t sms, int device, uint32_t* status, uint32_t spin,
                              cudaStream_t s);

}  // namespace q4k
