// Per-layer embeddings (PLE) of Gemma-4-E2B, stage 1, for sm_100a.
//
// The reference decodes the 1.6 GB Q5_K table per_layer_token_embd at load
// time into one f16 buffer per layer (streamDecodePleQ5_K,
// src/engine.ts:642-721: row v of the table holds `layers` consecutive
// 176-byte super-blocks, block L is layer L's 256 values; decodeQ5_KBlock,
// src/gguf.ts:218-256, then f32ToF16Array), and per token runs
// shaders/ple_stage1_fuse.wgsl once per layer (src/engine.ts:1528-1535):
//
//   rms = sqrt(sum_i projected[L*D+i]^2 / D + eps)
//   ple_inputs[L*D+i] = ((projected[L*D+i] / rms) * norm_w[i]
//                        + embed_L[token*D+i] * sqrt(D)) * inverseSqrt(2)
//
// Here the table stays Q5_K in HBM as the file stores it.  One launch covers
// every layer of T tokens: CTA (L, t) stages token t's super-block of layer
// L (176 bytes) in shared memory, each of its 256 threads decodes one
// element exactly as the upload would have stored it (f16_rne of the f32
// value d*sc*q - dmin*m, q the 5-bit quant), and the CTA applies the fused
// normalisation.  The token ids are read from device memory, so the argmax
// of the previous step can feed the next one without a host round trip (as
// src/engine.ts:1719-1727 copies it into the uniforms).  f32 products and
// sums are written with explicit round-to-nearest intrinsics (no FMA
// contraction) in the shader's order, including the 256-lane tree sum.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_ctx.cuh"
#include "q4k_device.cuh"

namespace q4k {
namespace {

constexpr uint32_t kQ5Bytes = 176;
constexpr uint32_t kPleDim = 256;  // per_layer_input_dim: one super-block per layer

// Element i (0..255) of a Q5_K super-block held in `b` (src/gguf.ts:233-254):
// group g = i/64 takes the low nibbles of qs[32g + l] (j < 32) or the high
// nibbles (j >= 32), plus bit 2g (low) or 2g+1 (high) of qh[l] as the 16s
// bit; sub-block 2g or 2g+1 gives (sc, m).  Returns the f16 bits of
// f16_rne(f32(d*sc*q - dmin*m)): d*sc and dmin*m are exact in f32 and the
// fma rounds the exact value once, like the reference's f64 expression
// stored into a Float32Array.
__device__ __forceinline__ uint16_t q5k_element_f16(const uint8_t* b, uint32_t i) {
  const uint32_t g = i >> 6, j = i & 63u, l = j & 31u, hi = j >> 5;
  const uint32_t qs = b[48 + 32 * g + l];
  const uint32_t nib = hi ? (qs >> 4) : (qs & 15u);
  const uint32_t q = nib + (((b[16 + l] >> (2 * g + hi)) & 1u) << 4);
  const uint32_t sb = 2 * g + hi;
  const uint8_t* s = b + 4;
  uint32_t sc, m;
  if (sb < 4) {
    sc = s[sb] & 63u;
    m = s[sb + 4] & 63u;
  } else {
    sc = (s[sb + 4] & 15u) | ((s[sb - 4] >> 6) << 4);
    m = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4);
  }
  const float d = half_bits_to_float((uint32_t)b[0] | ((uint32_t)b[1] << 8));
  const float dmin = half_bits_to_float((uint32_t)b[2] | ((uint32_t)b[3] << 8));
  return weight_f16_bits(d * (float)sc, dmin * (float)m, q);
}

// Thread per element; the debug view of the decoded table (q4k_q5k_dequant_f16).
__global__ void __launch_bounds__(256) q5k_dequant_kernel(const uint8_t* w, uint16_t* out, uint64_t n_blocks) {
  const uint64_t blk = blockIdx.x;
  if (blk >= n_blocks) return;
  __shared__ __align__(16) uint8_t sb[kQ5Bytes];
  if (threadIdx.x < kQ5Bytes / 16)
    reinterpret_cast<uint4*>(sb)[threadIdx.x] = reinterpret_cast<const uint4*>(w + blk * kQ5Bytes)[threadIdx.x];
  __syncthreads();
  out[blk * kPleDim + threadIdx.x] = q5k_element_f16(sb, threadIdx.x);
}

// CTA (L, t): layer L of token t.  status bit 1: a token id >= vocab (that
// token's outputs are NaN).
__global__ void __launch_bounds__(kPleDim) ple_stage1_kernel(const uint8_t* table, const uint32_t* tokens,
                                                             uint32_t vocab, uint32_t layers, const float* projected,
                                                             const uint16_t* norm_w, float eps, float* out,
                                                             uint32_t* status) {
  __shared__ __align__(16) uint8_t sb[kQ5Bytes];
  __shared__ float s_sum[kPleDim];
  const uint32_t L = blockIdx.x, t = blockIdx.y, i = threadIdx.x;
  const uint32_t token = tokens[t];
  const uint64_t base = ((uint64_t)t * layers + L) * kPleDim;
  if (token >= vocab) {
    out[base + i] = __int_as_float(0x7fc00000);
    if (i == 0 && L == 0) atomicOr(status, 2u);
    return;
  }
  if (i < kQ5Bytes / 16)
    reinterpret_cast<uint4*>(sb)[i] =
        reinterpret_cast<const uint4*>(table + ((uint64_t)token * layers + L) * kQ5Bytes)[i];
  const float v = projected[base + i];
  s_sum[i] = __fmul_rn(v, v);
  __syncthreads();
  // shaders/ple_stage1_fuse.wgsl:27-30: strides 128, 64, ..., 1
  for (uint32_t stride = kPleDim / 2; stride > 0; stride >>= 1) {
    if (i < stride) s_sum[i] = __fadd_rn(s_sum[i], s_sum[i + stride]);
    __syncthreads();
  }
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s_sum[0], (float)kPleDim), eps));
  const float nw = half_bits_to_float(norm_w[i]);
  const float e = half_bits_to_float(q5k_element_f16(sb, i));
  const float proj_normed = __fmul_rn(__fdiv_rn(v, rms), nw);
  const float embed_val = __fmul_rn(e, 16.0f);  // sqrt(f32(256)) = 16 exactly
  out[base + i] = __fmul_rn(__fadd_rn(proj_normed, embed_val), 0.70710678118654752f);
}

}  // namespace
}  // namespace q4k

using namespace q4k;

extern "C" int q4k_q5k_dequant_f16(q4k_ctx* ctx, const void* w, uint16_t* out, uint64_t n_blocks, void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!w || !out) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(w)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "Q5_K data must be 16-byte aligned");
  if (n_blocks == 0) return Q4K_OK;
  if (n_blocks > 0x7fffffffull) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "too many blocks");
  q5k_dequant_kernel<<<(uint32_t)n_blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w), out, n_blocks);
  return ctx_cuda(ctx, cudaGetLastError(), "q4k_q5k_dequant_f16 launch");
}

extern "C" int q4k_ple_stage1(q4k_ctx* ctx, const void* table, const uint32_t* token_ids, uint32_t T, uint32_t vocab,
                              uint32_t layers, const float* projected, const uint16_t* norm_w, float eps, float* out,
                              void* stream) {
  if (!ctx) return Q4K_ERR_INVALID_ARG;
  if (!table || !token_ids || !projected || !norm_w || !out)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(table)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "Q5_K table must be 16-byte aligned");
  if (vocab == 0 || layers == 0 || layers > 65535u || T > 65535u)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "ple_stage1: vocab=%u layers=%u T=%u out of range", vocab, layers, T);
  if (T == 0) return Q4K_OK;
  ple_stage1_kernel<<<dim3(layers, T), kPleDim, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(table), token_ids, vocab, layers, projected, norm_w, eps, out, ctx->select.status);
  return ctx_cuda(ctx, cudaGetLastError(), "q4k_ple_stage1 launch");
}
