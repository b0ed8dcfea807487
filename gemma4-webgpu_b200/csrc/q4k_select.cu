// LM-head consumers of the matmul: softcap, argmax, topk256 (per-residue max),
// gelu_mul and the cross-rank candidate merge.  The fused LM head (matmul +
// softcap + selection in one launch) is the engine's select task
// (q4k_engine.cu).
//
// Selection semantics (shaders/argmax.wgsl:7-34, shaders/topk256.wgsl:5-21):
//   * residue candidate t (t = 0..255) = first strict maximum over indices
//     i = t, t+256, ... starting from (-1e30, 0): the maximum under float '>',
//     ties to the lower index, NaN never wins;
//   * argmax = the residue candidate that the reference's tree over the 256
//     lanes leaves in lane 0: a value moves to the lower lane only when
//     strictly greater, so tied residues meet at their lowest differing bit
//     and the one with a 0 there wins (residue_argmax runs that same tree).
// Both are associative merges, so any partition of the indices (CTAs, warps,
// GPUs) gives bit-identical candidates.
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_device.cuh"
#include "q4k_kernels.cuh"

namespace q4k {
namespace {

constexpr float kFloor = -1e30f;  // the reference scans start here (argmax.wgsl:12)

// Shared-memory argmax over 256 residue candidates with the reference's tree:
// the partner wins only when strictly greater (argmax.wgsl:21-27).  Called by
// all threads of a >= 256-thread block; returns the winner to thread 0.
__device__ uint32_t residue_argmax(float* s_v, uint32_t* s_i) {
  const uint32_t t = threadIdx.x;
  for (uint32_t stride = 128; stride > 0; stride >>= 1) {
    if (t < stride && s_v[t + stride] > s_v[t]) {
      s_v[t] = s_v[t + stride];
      s_i[t] = s_i[t + stride];
    }
    __syncthreads();
  }
  return s_i[0];
}

// ---- standalone reference operators ---------------------------------------

__global__ void softcap_kernel(float* __restrict__ logits, uint32_t n, float cap) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    logits[i] = softcap(logits[i], cap);
}

// One 1024-thread block: thread t scans residue t%256, quarter t/256 of the
// index sequence; quarters merge per residue, then the argmax tree.
// mode 0 writes the argmax u32, mode 1 the topk256 buffer f32[512]
// (val, bitcast(idx)) as shaders/topk256.wgsl:19-20 lays it out.
__global__ void __launch_bounds__(1024) select_kernel(const float* __restrict__ logits, uint32_t n, int mode,
                                                      uint32_t* __restrict__ argmax_out,
                                                      float* __restrict__ topk_out) {
  __shared__ float s_v[1024];
  __shared__ uint32_t s_i[1024];
  const uint32_t t = threadIdx.x, r = t & 255u, q = t >> 8;
  float bv = kFloor;
  uint32_t bi = 0u;
  for (uint32_t i = r + 256u * q; i < n; i += 1024u) {
    const float v = logits[i];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  s_v[t] = bv;
  s_i[t] = bi;
  __syncthreads();
  if (t < 256) {
#pragma unroll
    for (int k = 1; k < 4; ++k)
      if (better(s_v[t + 256 * k], s_i[t + 256 * k], bv, bi)) {
        bv = s_v[t + 256 * k];
        bi = s_i[t + 256 * k];
      }
  }
  __syncthreads();
  if (t < 256) {
    s_v[t] = bv;
    s_i[t] = bi;
    if (mode == 1) {
      topk_out[2 * t] = bv;
      topk_out[2 * t + 1] = __uint_as_float(bi);
    }
  }
  __syncthreads();
  if (mode == 0) {
    const uint32_t am = residue_argmax(s_v, s_i);
    if (t == 0) *argmax_out = am;
  }
}

// Softcap + topk256 + argmax for B rows in one launch (the batch-B tail of
// sampleNextTokenSubmit, src/engine.ts:1686-1741): CTA (c, row) scans
// 256-element groups [c*gpc, (c+1)*gpc) of its row, thread t keeping residue
// t's first strict maximum (softcapping and storing the logits on the way
// when cap > 0, as logit_softcap.wgsl does in place), publishes it as an
// order key with atomicMax into the row's 256 slots, and the last CTA of the
// row (completion counter) turns the keys into the candidates and runs the
// reference's argmax tree, then puts the slots and counter back to their
// between-calls state.
__global__ void __launch_bounds__(256) select_rows_kernel(float* __restrict__ logits, uint32_t n, float cap,
                                                          uint32_t gpc, unsigned long long* __restrict__ slots,
                                                          uint32_t* __restrict__ counters, float* __restrict__ cand_val,
                                                          uint32_t* __restrict__ cand_idx,
                                                          uint32_t* __restrict__ argmax_out) {
  __shared__ float s_v[256];
  __shared__ uint32_t s_i[256];
  __shared__ uint32_t s_last;
  const uint32_t row = blockIdx.y, t = threadIdx.x;
  float* L = logits + (size_t)row * n;
  const uint32_t groups = (n + 255u) / 256u;
  const uint32_t g0 = blockIdx.x * gpc, g1 = min(groups, g0 + gpc);
  float bv = kFloor;
  uint32_t bi = 0u;
  for (uint32_t g = g0; g < g1; ++g) {
    const uint32_t i = g * 256u + t;
    if (i < n) {
      float v = L[i];
      if (cap > 0.0f) {
        v = softcap(v, cap);
        L[i] = v;
      }
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
  unsigned long long* S = slots + (size_t)row * 256u;
  if (!(bv == kFloor && bi == 0u)) atomicMax(&S[t], sel_key(bv, bi));
  __threadfence();
  __syncthreads();
  if (t == 0) s_last = (atomicAdd(&counters[row], 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float v;
  uint32_t i;
  sel_unkey(atomicExch(&S[t], sel_key(kFloor, 0u)), v, i);
  cand_val[(size_t)row * 256u + t] = v;
  cand_idx[(size_t)row * 256u + t] = i;
  s_v[t] = v;
  s_i[t] = i;
  __syncthreads();
  const uint32_t am = residue_argmax(s_v, s_i);
  if (t == 0) {
    argmax_out[row] = am;
    counters[row] = 0u;
  }
}

__global__ void init_row_slots_kernel(unsigned long long* slots, uint32_t* counters) {
  slots[blockIdx.x * 256u + threadIdx.x] = sel_key(kFloor, 0u);
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

// shaders/gelu_mul.wgsl:14-16.
__global__ void gelu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                float* __restrict__ out, uint32_t n) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = gelu_mul_value(gate[i], up[i]);
}

// Cross-rank merge: G candidate sets of 256 -> one, plus argmax.
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ vals, const uint32_t* __restrict__ idx,
                                                    uint32_t G, float* __restrict__ out_val,
                                                    uint32_t* __restrict__ out_idx, uint32_t* __restrict__ argmax_out) {
  __shared__ float s_v[256];
  __shared__ uint32_t s_i[256];
  const uint32_t t = threadIdx.x;
  float bv = kFloor;
  uint32_t bi = 0u;
  for (uint32_t g = 0; g < G; ++g) {
    const float v = vals[g * 256u + t];
    const uint32_t i = idx[g * 256u + t];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  out_val[t] = bv;
  out_idx[t] = bi;
  s_v[t] = bv;
  s_i[t] = bi;
  __syncthreads();
  const uint32_t am = residue_argmax(s_v, s_i);
  if (t == 0) *argmax_out = am;
}

}  // namespace

cudaError_t launch_softcap(float* logits, uint32_t n, float cap, cudaStream_t s) {
  uint32_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  if (grid == 0) grid = 1;
  softcap_kernel<<<grid, 256, 0, s>>>(logits, n, cap);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, uint32_t n, uint32_t* result, cudaStream_t s) {
  select_kernel<<<1, 1024, 0, s>>>(logits, n, 0, result, nullptr);
  return cudaGetLastError();
}

cudaError_t launch_topk256(const float* logits, uint32_t n, float* result512, cudaStream_t s) {
  select_kernel<<<1, 1024, 0, s>>>(logits, n, 1, nullptr, result512);
  return cudaGetLastError();
}

cudaError_t launch_gelu_mul(const float* gate, const float* up, float* out, uint32_t n, cudaStream_t s) {
  uint32_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  if (grid == 0) grid = 1;
  gelu_mul_kernel<<<grid, 256, 0, s>>>(gate, up, out, n);
  return cudaGetLastError();
}

cudaError_t init_row_slots(unsigned long long* slots, uint32_t* counters, uint32_t rows, cudaStream_t s) {
  init_row_slots_kernel<<<rows, 256, 0, s>>>(slots, counters);
  return cudaGetLastError();
}

cudaError_t launch_select_rows(float* logits, uint32_t B, uint32_t n, float cap, unsigned long long* slots,
                               uint32_t* counters, float* cand_val, uint32_t* cand_idx, uint32_t* argmax, int sms,
                               cudaStream_t s) {
  const uint32_t groups = (n + 255u) / 256u;
  uint32_t per_row = (2u * (uint32_t)sms) / B;  // about two CTAs per SM over all rows
  per_row = per_row == 0 ? 1u : per_row;
  const uint32_t gpc = (groups + per_row - 1) / per_row;
  const uint32_t ctas = (groups + gpc - 1) / gpc;
  select_rows_kernel<<<dim3(ctas, B), 256, 0, s>>>(logits, n, cap, gpc, slots, counters, cand_val, cand_idx, argmax);
  return cudaGetLastError();
}

cudaError_t launch_merge_candidates(const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                                    uint32_t* out_idx, uint32_t* argmax, cudaStream_t s) {
  merge_kernel<<<1, 256, 0, s>>>(vals, idx, G, out_val, out_idx, argmax);
  return cudaGetLastError();
}

}  // namespace q4k
