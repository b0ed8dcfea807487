// extern "C" entry points of libq4k.so (declared in include/q4k.h):
// argument validation, context and scratch ownership, error reporting.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/q4k.h"
#include "q4k_kernels.cuh"

struct q4k_ctx {
  int device = 0;
  int sm_count = 0;
  q4k::SelectScratch select;
  void* scratch = nullptr;
  char err[512] = {0};
};

namespace {

int fail(q4k_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->err, sizeof(ctx->err), fmt, ap);
    va_end(ap);
  }
  return code;
}

int cuda_status(q4k_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) {
    ctx->err[0] = 0;
    return Q4K_OK;
  }
  return fail(ctx, Q4K_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Shape and pointer checks shared by the matmul entry points.
int check_matmul(q4k_ctx* ctx, const void* w, const float* x, const float* y, uint32_t M, uint32_t N,
                 uint32_t batch) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!w || !x || !y) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer (w=%p x=%p y=%p)", w, x, (const void*)y);
  if (N == 0 || N % Q4K_QK != 0)
    return fail(ctx, Q4K_ERR_INVALID_ARG, "N=%u is not a positive multiple of %d (Q4_K super-block)", N, Q4K_QK);
  if (batch == 0) return fail(ctx, Q4K_ERR_INVALID_ARG, "batch must be >= 1");
  if (!aligned16(w) || !aligned16(x) || !aligned16(y))
    return fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned (w=%p x=%p y=%p)", w, x,
                (const void*)y);
  if ((uint64_t)M * batch > 0xffffffffull)
    return fail(ctx, Q4K_ERR_INVALID_ARG, "M*batch=%llu exceeds 2^32-1", (unsigned long long)M * batch);
  return Q4K_OK;
}

}  // namespace

extern "C" {

int q4k_version(void) { return 100; }

int q4k_create(int device, q4k_ctx** out) {
  if (!out) return Q4K_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return Q4K_ERR_CUDA;
  if (device < 0 || device >= n) return Q4K_ERR_INVALID_ARG;
  if (cudaSetDevice(device) != cudaSuccess) return Q4K_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return Q4K_ERR_CUDA;
  if (prop.major != 10) return Q4K_ERR_UNSUPPORTED;  // built for sm_100a only
  q4k_ctx* ctx = new q4k_ctx();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  if (cudaMalloc(&ctx->scratch, q4k::kSelectScratchBytes) != cudaSuccess) {
    delete ctx;
    return Q4K_ERR_CUDA;
  }
  ctx->select.slots = static_cast<unsigned long long*>(ctx->scratch);
  ctx->select.counter = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->scratch) + 256 * 8);
  if (q4k::init_select_scratch(ctx->select, nullptr) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(ctx->scratch);
    delete ctx;
    return Q4K_ERR_CUDA;
  }
  *out = ctx;
  return Q4K_OK;
}

void q4k_destroy(q4k_ctx* ctx) {
  if (!ctx) return;
  if (ctx->scratch) cudaFree(ctx->scratch);
  delete ctx;
}

const char* q4k_last_error(const q4k_ctx* ctx) { return ctx ? ctx->err : "null context"; }

int q4k_gemv(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
             void* stream) {
  int rc = check_matmul(ctx, w, x, y, M, N, batch);
  if (rc != Q4K_OK) return rc;
  if (M == 0) return Q4K_OK;
  return cuda_status(ctx,
                     q4k::launch_gemv(static_cast<const uint8_t*>(w), x, y, M, N, batch, N, M, 0,
                                      static_cast<cudaStream_t>(stream)),
                     "q4k_gemv launch");
}

int q4k_matmul_quant(q4k_ctx* ctx, const float* input, const void* weight, float* output, uint32_t M, uint32_t N,
                     void* stream) {
  return q4k_gemv(ctx, weight, input, output, M, N, 1, stream);
}

int q4k_dequant_f16(q4k_ctx* ctx, const void* w, uint16_t* out, uint64_t n_blocks, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n_blocks == 0) return Q4K_OK;
  if (!w || !out) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(w) || !aligned16(out)) return fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  if (n_blocks > (1ull << 36)) return fail(ctx, Q4K_ERR_INVALID_ARG, "n_blocks too large");
  return cuda_status(ctx,
                     q4k::launch_dequant_f16(static_cast<const uint8_t*>(w), out, n_blocks,
                                             static_cast<cudaStream_t>(stream)),
                     "q4k_dequant_f16 launch");
}

int q4k_logit_softcap(q4k_ctx* ctx, float* logits, uint32_t n, float cap, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n == 0) return Q4K_OK;
  if (!logits) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!(cap > 0.0f)) return fail(ctx, Q4K_ERR_INVALID_ARG, "cap must be > 0 (the engine skips the pass otherwise)");
  return cuda_status(ctx, q4k::launch_softcap(logits, n, cap, static_cast<cudaStream_t>(stream)),
                     "q4k_logit_softcap launch");
}

int q4k_argmax(q4k_ctx* ctx, const float* logits, uint32_t n, uint32_t* result, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!logits || !result) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return cuda_status(ctx, q4k::launch_argmax(logits, n, result, static_cast<cudaStream_t>(stream)),
                     "q4k_argmax launch");
}

int q4k_topk256(q4k_ctx* ctx, const float* logits, uint32_t n, float* result, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!logits || !result) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return cuda_status(ctx, q4k::launch_topk256(logits, n, result, static_cast<cudaStream_t>(stream)),
                     "q4k_topk256 launch");
}

int q4k_gelu_mul(q4k_ctx* ctx, const float* gate, const float* up, float* out, uint32_t n, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n == 0) return Q4K_OK;
  if (!gate || !up || !out) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return cuda_status(ctx, q4k::launch_gelu_mul(gate, up, out, n, static_cast<cudaStream_t>(stream)),
                     "q4k_gelu_mul launch");
}

int q4k_lmhead_select(q4k_ctx* ctx, const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                      uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                      void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!w || !x || !cand_val || !cand_idx || !argmax) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (N == 0 || N % Q4K_QK != 0)
    return fail(ctx, Q4K_ERR_INVALID_ARG, "N=%u is not a positive multiple of %d", N, Q4K_QK);
  if (V == 0) return fail(ctx, Q4K_ERR_INVALID_ARG, "V must be >= 1");
  if ((uint64_t)row_offset + V >= (1ull << 31))
    return fail(ctx, Q4K_ERR_INVALID_ARG, "row_offset + V must be < 2^31");
  if (!aligned16(w) || !aligned16(x) || (logits && !aligned16(logits)))
    return fail(ctx, Q4K_ERR_INVALID_ARG, "w, x and logits must be 16-byte aligned");
  return cuda_status(ctx,
                     q4k::launch_lmhead_select(static_cast<const uint8_t*>(w), x, V, N, cap, row_offset, logits,
                                               cand_val, cand_idx, argmax, ctx->select,
                                               static_cast<cudaStream_t>(stream)),
                     "q4k_lmhead_select launch");
}

int q4k_merge_candidates(q4k_ctx* ctx, const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                         uint32_t* out_idx, uint32_t* argmax, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!vals || !idx || !out_val || !out_idx || !argmax) return fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (G == 0 || G > 4096) return fail(ctx, Q4K_ERR_INVALID_ARG, "G=%u out of range [1, 4096]", G);
  return cuda_status(ctx,
                     q4k::launch_merge_candidates(vals, idx, G, out_val, out_idx, argmax,
                                                  static_cast<cudaStream_t>(stream)),
                     "q4k_merge_candidates launch");
}

}  // extern "C"
