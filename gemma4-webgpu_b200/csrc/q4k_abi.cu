// extern "C" entry points of libq4k.so (declared in include/q4k.h): argument
// validation, context and scratch ownership, error reporting.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "q4k_ctx.cuh"

using namespace q4k;

namespace {

// Shape and pointer checks shared by the matmul entry points.
int check_matmul(q4k_ctx* ctx, const void* w, const float* x, const float* y, uint32_t M, uint32_t N,
                 uint32_t batch) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!w || !x || !y)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer (w=%p x=%p y=%p)", w, (const void*)x, (const void*)y);
  if (N == 0 || N % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "N=%u is not a positive multiple of %d (Q4_K super-block)", N,
                    Q4K_QK);
  if (batch == 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "batch must be >= 1");
  if (!aligned16(w) || !aligned16(x) || !aligned16(y))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned (w=%p x=%p y=%p)", w,
                    (const void*)x, (const void*)y);
  if ((uint64_t)M * batch > 0xffffffffull || (uint64_t)N * batch > 0xffffffffull)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "M*batch or N*batch exceeds 2^32-1");
  return Q4K_OK;
}

// The engine path for batch <= 16 when the prepared activation fits the
// context scratch; otherwise the scratch-free warp-per-row kernel.
int run_gemv(q4k_ctx* ctx, const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
             cudaStream_t s) {
  uint32_t done = 0;
  while (done < batch) {
    const uint32_t b = (batch - done) > (uint32_t)kMaxTokens ? (uint32_t)kMaxTokens : (batch - done);
    const float* xc = x + (uint64_t)done * N;
    float* yc = y + (uint64_t)done * M;
    if (xfrag_bytes(N, b) <= ctx->xfrag_cap) {
      CUtensorMap map;
      uint32_t tile_bytes = 0;
      cudaError_t e = encode_weight_map(&map, w, M, N, &tile_bytes);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemv weight tensor map");
      JobList jl{};
      jl.n = 1;
      jl.inl.x = xc;
      jl.inl.xfrag = ctx->xfrag;
      jl.inl.inv_scale = ctx->inv_scale;
      jl.inl.N = N;
      jl.inl.mode = 0;
      // the engine prepares the activation itself when it fits each CTA's cache
      const bool prep = xfrag_bytes(N, b) <= engine_xcache_bytes(false);
      if (!prep) {
        e = launch_xprep(jl, b, s);
        if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemv activation prep launch");
      }
      TaskList tl{};
      tl.prep = prep ? 1u : 0u;
      tl.inl_job = jl.inl;
      tl.n = 1;
      tl.inl.w = w;
      tl.inl.xfrag = ctx->xfrag;
      tl.inl.inv_scale = ctx->inv_scale;
      tl.inl.y = yc;
      tl.inl.M = M;
      tl.inl.N = N;
      tl.inl.item_begin = 0;
      tl.inl.item_end = tiles_of(M);
      tl.inl.kind = kTaskPlain;
      tl.inl.tile_bytes = tile_bytes;
      tl.total_items = tiles_of(M);
      tl.total_cost = tiles_of(M) * (N / Q4K_QK);
      // long rows (e.g. the FFN down projection): 4 warps share each tile,
      // one K quarter each, as plans do for such stages
      const uint32_t nb = N / Q4K_QK;
      tl.ksplit = (b <= 4 && nb >= 16 && nb % 4 == 0) ? 4u : 0u;
      tl.pairs = pairs_of(N, tl.ksplit, tile_bytes) ? 1u : 0u;
      e = launch_engine(tl, map, b, false, ctx->select, ctx->sm_count, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemv engine launch");
    } else {
      cudaError_t e = launch_gemv(w, xc, yc, M, N, b, N, M, 0, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemv launch");
    }
    done += b;
  }
  ctx->err[0] = 0;
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
  const size_t sel_bytes = 256 * sizeof(unsigned long long) + 256;
  const size_t scale_bytes = kCtxScaleSlots * sizeof(float);
  const size_t rows_bytes = kMaxSelectRows * 256 * sizeof(unsigned long long) + 256;
  const size_t total = sel_bytes + scale_bytes + kCtxXfragBytes + rows_bytes;
  if (cudaMalloc(&ctx->scratch, total) != cudaSuccess) {
    delete ctx;
    return Q4K_ERR_CUDA;
  }
  char* base = static_cast<char*>(ctx->scratch);
  ctx->select.slots = reinterpret_cast<unsigned long long*>(base);
  ctx->select.counter = reinterpret_cast<uint32_t*>(base + 256 * 8);
  ctx->select.status = reinterpret_cast<uint32_t*>(base + 256 * 8 + 4);
  ctx->inv_scale = reinterpret_cast<float*>(base + sel_bytes);
  ctx->xfrag = reinterpret_cast<uint2*>(base + sel_bytes + scale_bytes);
  ctx->xfrag_cap = kCtxXfragBytes;
  ctx->row_slots = reinterpret_cast<unsigned long long*>(base + sel_bytes + scale_bytes + kCtxXfragBytes);
  ctx->row_counters = reinterpret_cast<uint32_t*>(ctx->row_slots + kMaxSelectRows * 256);
  if (init_select_scratch(ctx->select, nullptr) != cudaSuccess ||
      init_row_slots(ctx->row_slots, ctx->row_counters, kMaxSelectRows, nullptr) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
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

int q4k_set_wait_limit(q4k_ctx* ctx, uint32_t polls) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  ctx->select.spin_limit = polls;  // 0: the built-in default
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_check(q4k_ctx* ctx) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_check synchronize");
  uint32_t status = 0;
  e = cudaMemcpy(&status, ctx->select.status, sizeof(status), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_check status read");
  if (status != 0) {
    const uint32_t zero = 0;
    cudaMemcpy(ctx->select.status, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    if (status & 1u)
      return ctx_fail(ctx, Q4K_ERR_TIMEOUT,
                      "a kernel gave up a bounded wait (its weight copies, a K-split partner or a peer rank's "
                      "candidates did not arrive within the wait limit); its outputs are invalid");
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "a token id was >= vocab in q4k_ple_stage1; that token's outputs are NaN");
  }
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_gemv(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
             void* stream) {
  int rc = check_matmul(ctx, w, x, y, M, N, batch);
  if (rc != Q4K_OK) return rc;
  if (M == 0) return Q4K_OK;
  if (batch >= kGemmMinRows)
    return run_gemm(ctx, static_cast<const uint8_t*>(w), x, y, M, N, batch, static_cast<cudaStream_t>(stream));
  return run_gemv(ctx, static_cast<const uint8_t*>(w), x, y, M, N, batch, static_cast<cudaStream_t>(stream));
}

int q4k_gemm(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
             void* stream) {
  int rc = check_matmul(ctx, w, x, y, M, N, T);
  if (rc != Q4K_OK) return rc;
  if (M == 0) return Q4K_OK;
  return run_gemm(ctx, static_cast<const uint8_t*>(w), x, y, M, N, T, static_cast<cudaStream_t>(stream));
}

int q4k_gemm_f16x(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
                  void* stream) {
  int rc = check_matmul(ctx, w, x, y, M, N, T);
  if (rc != Q4K_OK) return rc;
  if (M == 0) return Q4K_OK;
  return run_gemm(ctx, static_cast<const uint8_t*>(w), x, y, M, N, T, static_cast<cudaStream_t>(stream), 1u);
}

int q4k_matmul_quant(q4k_ctx* ctx, const float* input, const void* weight, float* output, uint32_t M, uint32_t N,
                     void* stream) {
  return q4k_gemv(ctx, weight, input, output, M, N, 1, stream);
}

int q4k_dequant_f16(q4k_ctx* ctx, const void* w, uint16_t* out, uint64_t n_blocks, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n_blocks == 0) return Q4K_OK;
  if (!w || !out) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(w) || !aligned16(out)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  if (n_blocks > (1ull << 36)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "n_blocks too large");
  return ctx_cuda(ctx,
                  launch_dequant_f16(static_cast<const uint8_t*>(w), out, n_blocks,
                                     static_cast<cudaStream_t>(stream)),
                  "q4k_dequant_f16 launch");
}

int q4k_logit_softcap(q4k_ctx* ctx, float* logits, uint32_t n, float cap, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n == 0) return Q4K_OK;
  if (!logits) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!(cap > 0.0f))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "cap must be > 0 (the engine skips the pass otherwise)");
  return ctx_cuda(ctx, launch_softcap(logits, n, cap, static_cast<cudaStream_t>(stream)),
                  "q4k_logit_softcap launch");
}

int q4k_argmax(q4k_ctx* ctx, const float* logits, uint32_t n, uint32_t* result, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!logits || !result) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return ctx_cuda(ctx, launch_argmax(logits, n, result, static_cast<cudaStream_t>(stream)), "q4k_argmax launch");
}

int q4k_topk256(q4k_ctx* ctx, const float* logits, uint32_t n, float* result, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!logits || !result) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return ctx_cuda(ctx, launch_topk256(logits, n, result, static_cast<cudaStream_t>(stream)), "q4k_topk256 launch");
}

int q4k_select_rows(q4k_ctx* ctx, float* logits, uint32_t B, uint32_t n, float cap, float* cand_val,
                    uint32_t* cand_idx, uint32_t* argmax, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!logits || !cand_val || !cand_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (B == 0 || B > kMaxSelectRows)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "q4k_select_rows: B=%u outside [1, %u]", B, kMaxSelectRows);
  if (n == 0 || n >= (1u << 31)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "q4k_select_rows: n=%u out of range", n);
  return ctx_cuda(ctx,
                  launch_select_rows(logits, B, n, cap, ctx->row_slots, ctx->row_counters, cand_val, cand_idx, argmax,
                                     ctx->sm_count, static_cast<cudaStream_t>(stream)),
                  "q4k_select_rows launch");
}

int q4k_gelu_mul(q4k_ctx* ctx, const float* gate, const float* up, float* out, uint32_t n, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (n == 0) return Q4K_OK;
  if (!gate || !up || !out) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  return ctx_cuda(ctx, launch_gelu_mul(gate, up, out, n, static_cast<cudaStream_t>(stream)), "q4k_gelu_mul launch");
}

int q4k_lmhead_select(q4k_ctx* ctx, const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                      uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                      void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!w || !x || !cand_val || !cand_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (N == 0 || N % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "N=%u is not a positive multiple of %d", N, Q4K_QK);
  if (V == 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "V must be >= 1");
  if ((uint64_t)row_offset + V >= (1ull << 31))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "row_offset + V must be < 2^31");
  if (!aligned16(w) || !aligned16(x) || (logits && !aligned16(logits)))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "w, x and logits must be 16-byte aligned");
  if (xfrag_bytes(N, 1) > ctx->xfrag_cap)
    return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "N=%u exceeds the context's activation scratch", N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap map;
  uint32_t tile_bytes = 0;
  cudaError_t e = encode_weight_map(&map, w, V, N, &tile_bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_lmhead_select weight tensor map");
  JobList jl{};
  jl.n = 1;
  jl.inl.x = x;
  jl.inl.xfrag = ctx->xfrag;
  jl.inl.inv_scale = ctx->inv_scale;
  jl.inl.N = N;
  const bool prep = xfrag_bytes(N, 1) <= engine_xcache_bytes(true);
  if (!prep) {
    e = launch_xprep(jl, 1, s);
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_lmhead_select activation prep launch");
  }
  TaskList tl{};
  tl.prep = prep ? 1u : 0u;
  tl.inl_job = jl.inl;
  tl.n = 1;
  tl.inl.w = static_cast<const uint8_t*>(w);
  tl.inl.xfrag = ctx->xfrag;
  tl.inl.inv_scale = ctx->inv_scale;
  tl.inl.logits = logits;
  tl.inl.cand_val = cand_val;
  tl.inl.cand_idx = cand_idx;
  tl.inl.argmax = argmax;
  tl.inl.M = V;
  tl.inl.N = N;
  tl.inl.item_begin = 0;
  tl.inl.item_end = tiles_of(V);
  tl.inl.kind = kTaskSelect;
  tl.inl.row_offset = row_offset;
  tl.inl.cap = cap;
  tl.inl.tile_bytes = tile_bytes;
  tl.total_items = tiles_of(V);
  tl.total_cost = tiles_of(V) * (N / Q4K_QK);
  tl.pairs = pairs_of(N, 0, tile_bytes) ? 1u : 0u;
  return ctx_cuda(ctx, launch_engine(tl, map, 1, true, ctx->select, ctx->sm_count, s), "q4k_lmhead_select launch");
}

int q4k_merge_candidates(q4k_ctx* ctx, const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                         uint32_t* out_idx, uint32_t* argmax, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!vals || !idx || !out_val || !out_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (G == 0 || G > 4096) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "G=%u out of range [1, 4096]", G);
  return ctx_cuda(ctx,
                  launch_merge_candidates(vals, idx, G, out_val, out_idx, argmax, static_cast<cudaStream_t>(stream)),
                  "q4k_merge_candidates launch");
}

}  // extern "C"
