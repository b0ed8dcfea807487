// Q6_K entry points of libq4k.so: the load-time repack of GGUF Q6_K bytes
// into the device layout (q6k_dequant.cuh), the weight probe, and the GEMV /
// fused LM head, which run on the engine's Q6_K variant.
//
// Reference: Q6_K tensors are decoded on the CPU at load (src/gguf.ts:316-368,
// via tensorToF16 src/engine.ts:570-578), uploaded as f16 and multiplied by
// the same matmul_quant pipelines as Q4_K ones (shaders/matmul_quant.wgsl);
// Q4_K_M files use Q6_K for some matmuls (docs/findings/why-q4km.md:33).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_ctx.cuh"
#include "q6k_dequant.cuh"

using namespace q4k;

namespace {

// One 32-bit word of a body per thread (GGUF super-blocks are 2-byte
// aligned: two 16-bit loads), then one d per thread into the d plane.
__global__ void q6k_repack_kernel(const uint16_t* __restrict__ src, uint32_t* __restrict__ bodies,
                                  uint16_t* __restrict__ dplane, uint32_t M, uint32_t nb) {
  const uint64_t n_blocks = (uint64_t)M * nb;
  const uint64_t n_words = n_blocks * kQ6BodyWords;
  const uint32_t mp = q6k_dpitch(M);
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words; i += stride) {
    const uint64_t blk = i / kQ6BodyWords, j = i % kQ6BodyWords;
    const uint16_t* s = src + blk * (kQ6BlockBytes / 2) + 2 * j;
    bodies[i] = (uint32_t)s[0] | ((uint32_t)s[1] << 16);
  }
  const uint64_t n_d = (uint64_t)nb * mp;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_d; i += stride) {
    const uint32_t b = (uint32_t)(i / mp), m = (uint32_t)(i % mp);
    dplane[i] = m < M ? src[((uint64_t)m * nb + b) * (kQ6BlockBytes / 2) + kQ6BodyBytes / 2] : (uint16_t)0;
  }
}

// Weight probe: every weight of the device layout through the engine's
// decode (the exact form), written in row-major k order.  Thread = (row,
// super-block, lane role c, word w): the 8 weights a GEMV lane c derives
// from word w.
__global__ void q6k_dequant_kernel(const uint8_t* __restrict__ w, uint16_t* __restrict__ out, uint32_t M,
                                   uint32_t nb) {
  const uint64_t n = (uint64_t)M * nb * 32;
  const uint32_t mp = q6k_dpitch(M);
  const uint16_t* dplane = reinterpret_cast<const uint16_t*>(w + (uint64_t)M * nb * kQ6BodyBytes);
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t wd = (uint32_t)(i & 7u), c = (uint32_t)((i >> 3) & 3u);
    const uint64_t blk = i >> 5;
    const uint32_t m = (uint32_t)(blk / nb), b = (uint32_t)(blk % nb);
    const uint8_t* body = w + blk * kQ6BodyBytes;
    const uint32_t h = c >> 1;
    const uint32_t ql0 = *reinterpret_cast<const uint32_t*>(body + 64 * h + 4 * wd);
    const uint32_t ql1 = *reinterpret_cast<const uint32_t*>(body + 64 * h + 32 + 4 * wd);
    const uint32_t qh = *reinterpret_cast<const uint32_t*>(body + 128 + 32 * h + 4 * wd);
    const uint32_t scw = *reinterpret_cast<const uint32_t*>(body + 192 + 4 * c);
    const float d4 = 4.0f * __half2float(__ushort_as_half(dplane[(uint64_t)b * mp + m]));
    const Q6Consts k = q6_consts(scw, wd >> 2, d4);
    const WordPairs p = dequant6_word<true>(ql0, ql1, qh, (c & 1u) * 4u, k);
    uint16_t* o = out + (uint64_t)m * nb * 256 + (uint64_t)b * 256 + 64 * c + 4 * wd;
    o[0] = (uint16_t)(p.lo02 & 0xffffu);
    o[2] = (uint16_t)(p.lo02 >> 16);
    o[1] = (uint16_t)(p.lo13 & 0xffffu);
    o[3] = (uint16_t)(p.lo13 >> 16);
    o[32] = (uint16_t)(p.hi02 & 0xffffu);
    o[34] = (uint16_t)(p.hi02 >> 16);
    o[33] = (uint16_t)(p.hi13 & 0xffffu);
    o[35] = (uint16_t)(p.hi13 >> 16);
  }
}

uint32_t grid_for(uint64_t n, int sm_count) {
  const uint64_t g = (n + 255) / 256;
  const uint64_t cap = (uint64_t)sm_count * 8;
  return (uint32_t)(g < 1 ? 1 : (g > cap ? cap : g));
}

int check_q6_shape(q4k_ctx* ctx, const void* w, uint32_t M, uint32_t N) {
  if (!w) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null weight pointer");
  if (M == 0 || N == 0 || N % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "M=%u N=%u: M must be >= 1 and N a positive multiple of %d", M, N,
                    Q4K_QK);
  if (!aligned16(w)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "device-layout weights must be 16-byte aligned");
  return Q4K_OK;
}

}  // namespace

extern "C" {

uint64_t q4k_q6k_device_bytes(uint32_t M, uint32_t N) { return N % Q4K_QK ? 0 : q6k_device_bytes(M, N); }

int q4k_q6k_repack(q4k_ctx* ctx, const void* w_gguf, void* w_dev, uint32_t M, uint32_t N, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  int r = check_q6_shape(ctx, w_dev, M, N);
  if (r) return r;
  if (!w_gguf || ((uintptr_t)w_gguf & 1u))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "GGUF Q6_K bytes must be a non-null, 2-byte aligned pointer");
  const uint32_t nb = N / Q4K_QK;
  uint8_t* dst = static_cast<uint8_t*>(w_dev);
  const uint64_t work = (uint64_t)M * nb * kQ6BodyWords;
  q6k_repack_kernel<<<grid_for(work, ctx->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w_gguf), reinterpret_cast<uint32_t*>(dst),
      reinterpret_cast<uint16_t*>(dst + (uint64_t)M * nb * kQ6BodyBytes), M, nb);
  return ctx_cuda(ctx, cudaGetLastError(), "q4k_q6k_repack launch");
}

int q4k_q6k_dequant_f16(q4k_ctx* ctx, const void* w_dev, uint32_t M, uint32_t N, uint16_t* out, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  int r = check_q6_shape(ctx, w_dev, M, N);
  if (r) return r;
  if (!out) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null output pointer");
  const uint32_t nb = N / Q4K_QK;
  const uint64_t work = (uint64_t)M * nb * 32;
  q6k_dequant_kernel<<<grid_for(work, ctx->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w_dev), out, M, nb);
  return ctx_cuda(ctx, cudaGetLastError(), "q4k_q6k_dequant_f16 launch");
}

int q4k_q6k_gemv(q4k_ctx* ctx, const void* w_dev, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
                 void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  int r = check_q6_shape(ctx, w_dev, M, N);
  if (r) return r;
  if (!x || !y) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer (x=%p y=%p)", (const void*)x, (void*)y);
  if (batch == 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "batch must be >= 1");
  if (!aligned16(x) || !aligned16(y)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  if ((uint64_t)M * batch > 0xffffffffull || (uint64_t)N * batch > 0xffffffffull)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "M*batch or N*batch exceeds 2^32-1");
  if (xfrag_bytes(N, 1) > ctx->xfrag_cap)
    return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "N=%u exceeds the context's activation scratch", N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap maps[2];
  uint32_t tile_bytes = 0;
  cudaError_t e = encode_q6k_maps(maps, w_dev, M, N, &tile_bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_q6k_gemv weight tensor maps");
  uint32_t done = 0;
  while (done < batch) {
    uint32_t b = (batch - done) > (uint32_t)kMaxTokens ? (uint32_t)kMaxTokens : (batch - done);
    while (xfrag_bytes(N, b) > ctx->xfrag_cap) --b;
    JobList jl{};
    jl.n = 1;
    jl.inl.x = x + (uint64_t)done * N;
    jl.inl.xfrag = ctx->xfrag;
    jl.inl.inv_scale = ctx->inv_scale;
    jl.inl.N = N;
    const bool prep = xfrag_bytes(N, b) <= engine_xcache_bytes(false, kFmtQ6K);
    if (!prep) {
      e = launch_xprep(jl, b, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_q6k_gemv activation prep launch");
    }
    TaskList tl{};
    tl.fmt = kFmtQ6K;
    tl.prep = prep ? 1u : 0u;
    tl.inl_job = jl.inl;
    tl.n = 1;
    tl.inl.w = static_cast<const uint8_t*>(w_dev);
    tl.inl.xfrag = ctx->xfrag;
    tl.inl.inv_scale = ctx->inv_scale;
    tl.inl.y = y + (uint64_t)done * M;
    tl.inl.M = M;
    tl.inl.N = N;
    tl.inl.item_begin = 0;
    tl.inl.item_end = tiles_of(M);
    tl.inl.kind = kTaskPlain;
    tl.inl.tile_bytes = tile_bytes;
    tl.total_items = tiles_of(M);
    tl.total_cost = tiles_of(M) * (N / Q4K_QK);
    e = launch_engine(tl, maps[0], b, false, ctx->select, ctx->sm_count, s, &maps[1]);
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_q6k_gemv engine launch");
    done += b;
  }
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_q6k_lmhead_select(q4k_ctx* ctx, const void* w_dev, const float* x, uint32_t V, uint32_t N, float cap,
                          uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                          void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  int r = check_q6_shape(ctx, w_dev, V, N);
  if (r) return r;
  if (!x || !cand_val || !cand_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if ((uint64_t)row_offset + V >= (1ull << 31))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "row_offset + V must be < 2^31");
  if (!aligned16(x) || (logits && !aligned16(logits)))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "x and logits must be 16-byte aligned");
  if (xfrag_bytes(N, 1) > ctx->xfrag_cap)
    return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "N=%u exceeds the context's activation scratch", N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap maps[2];
  uint32_t tile_bytes = 0;
  cudaError_t e = encode_q6k_maps(maps, w_dev, V, N, &tile_bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_q6k_lmhead_select weight tensor maps");
  JobList jl{};
  jl.n = 1;
  jl.inl.x = x;
  jl.inl.xfrag = ctx->xfrag;
  jl.inl.inv_scale = ctx->inv_scale;
  jl.inl.N = N;
  const bool prep = xfrag_bytes(N, 1) <= engine_xcache_bytes(true, kFmtQ6K);
  if (!prep) {
    e = launch_xprep(jl, 1, s);
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_q6k_lmhead_select activation prep launch");
  }
  TaskList tl{};
  tl.fmt = kFmtQ6K;
  tl.prep = prep ? 1u : 0u;
  tl.inl_job = jl.inl;
  tl.n = 1;
  tl.inl.w = static_cast<const uint8_t*>(w_dev);
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
  return ctx_cuda(ctx, launch_engine(tl, maps[0], 1, true, ctx->select, ctx->sm_count, s, &maps[1]),
                  "q4k_q6k_lmhead_select launch");
}

}  // extern "C"
