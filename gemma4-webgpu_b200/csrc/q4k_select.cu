// LM-head consumers of the matmul: softcap, argmax, topk256 (per-residue max),
// gelu_mul, the fused LM head, and the cross-rank candidate merge.
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

// 64-bit order key of a (value, global index) candidate for atomicMax: a larger
// key is a larger value, then a lower index.  -0.0 and +0.0 order equal; the
// low bit keeps the sign of a zero so the exact value comes back out.
// Requires index < 2^31.
__device__ __forceinline__ unsigned long long pack_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  const uint32_t neg_zero = (b == 0x80000000u) ? 1u : 0u;
  if (neg_zero) b = 0u;
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | ((unsigned long long)(0x7fffffffu - idx) << 1) | neg_zero;
}

__device__ __forceinline__ void unpack_key(unsigned long long k, float& v, uint32_t& idx) {
  const uint32_t ord = (uint32_t)(k >> 32);
  uint32_t b = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
  if (k & 1ull) b = 0x80000000u;
  v = __uint_as_float(b);
  idx = 0x7fffffffu - (uint32_t)((k >> 1) & 0x7fffffffu);
}

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

// ---- fused LM head -------------------------------------------------------

// One warp per vocabulary row (rows strided over the persistent grid); the
// row's logit is softcapped, optionally stored, and folded into the warp's
// private per-residue best (shared memory, no races).  Each CTA then merges
// its warps and publishes 256 atomicMax keys; the last CTA to finish turns
// the keys into candidates + argmax and resets the keys and the counter, so
// the scratch is ready for the next call without a memset.
constexpr int kSelWarps = 8;

__global__ void __launch_bounds__(kSelWarps * 32) lmhead_select_kernel(
    const uint8_t* __restrict__ w, const float* __restrict__ x, uint32_t V, uint32_t N, float cap,
    uint32_t row_offset, float* __restrict__ logits_opt, float* __restrict__ cand_val,
    uint32_t* __restrict__ cand_idx, uint32_t* __restrict__ argmax_out, unsigned long long* __restrict__ slots,
    uint32_t* __restrict__ counter) {
  __shared__ float s_bv[kSelWarps][256];
  __shared__ uint32_t s_bi[kSelWarps][256];
  __shared__ uint32_t s_last;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  for (uint32_t r = lane; r < 256; r += 32) {
    s_bv[warp][r] = kFloor;
    s_bi[warp][r] = 0u;
  }
  __syncwarp();

  const uint32_t nb = N / kQK;
  const uint64_t row_bytes = (uint64_t)nb * kBlockBytes;
  const uint64_t total_warps = (uint64_t)gridDim.x * kSelWarps;
  for (uint64_t row = (uint64_t)blockIdx.x * kSelWarps + warp; row < V; row += total_warps) {
    const uint8_t* wr = w + row * row_bytes;
    float acc = 0.0f;
    for (uint32_t u = lane; u < 4u * nb; u += 32u) {
      const uint32_t blk_i = u >> 2, g = u & 3u;
      const uint8_t* blk = wr + (uint64_t)blk_i * kBlockBytes;
      const uint4 h = *reinterpret_cast<const uint4*>(blk);
      const ScaleMin4 sm = unpack_scale_min(h.y, h.z, h.w);
      const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
      uint32_t sc0, m0, sc1, m1;
      scale_min(sm, 2 * g, sc0, m0);
      scale_min(sm, 2 * g + 1, sc1, m1);
      const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0;
      const float ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
      const uint4 qa = ldg_nc_v4(blk + 16 + 32 * g);
      const uint4 qb = ldg_nc_v4(blk + 32 + 32 * g);
      const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const uint32_t k0 = blk_i * kQK + 64 * g;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 xl = *reinterpret_cast<const float4*>(x + k0 + 4 * i);
        const float4 xh = *reinterpret_cast<const float4*>(x + k0 + 32 + 4 * i);
        const float xlv[4] = {xl.x, xl.y, xl.z, xl.w}, xhv[4] = {xh.x, xh.y, xh.z, xh.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = (qw[i] >> (8 * j)) & 0xffu;
          acc = fmaf(weight_f16r(ds0, dm0, byte & 15u), xlv[j], acc);
          acc = fmaf(weight_f16r(ds1, dm1, byte >> 4), xhv[j], acc);
        }
      }
    }
    float v = warp_sum(acc);
    if (lane == 0) {
      if (cap > 0.0f) v = softcap(v, cap);
      if (logits_opt) logits_opt[row] = v;
      const uint32_t gi = row_offset + (uint32_t)row;
      const uint32_t res = gi & 255u;
      if (better(v, gi, s_bv[warp][res], s_bi[warp][res])) {
        s_bv[warp][res] = v;
        s_bi[warp][res] = gi;
      }
    }
  }
  __syncthreads();

  // CTA merge (thread t = residue t), then one atomicMax per residue.
  const uint32_t t = threadIdx.x;
  if (t < 256) {
    float bv = s_bv[0][t];
    uint32_t bi = s_bi[0][t];
#pragma unroll
    for (int k = 1; k < kSelWarps; ++k)
      if (better(s_bv[k][t], s_bi[k][t], bv, bi)) {
        bv = s_bv[k][t];
        bi = s_bi[k][t];
      }
    if (!(bv == kFloor && bi == 0u)) atomicMax(&slots[t], pack_key(bv, bi));
  }
  __threadfence();
  __syncthreads();
  if (t == 0) s_last = (atomicAdd(counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA: keys -> candidates, argmax, reset.
  float* f_v = &s_bv[0][0];
  uint32_t* f_i = &s_bi[0][0];
  if (t < 256) {
    const unsigned long long k = atomicExch(&slots[t], pack_key(kFloor, 0u));
    float v;
    uint32_t i;
    unpack_key(k, v, i);
    cand_val[t] = v;
    cand_idx[t] = i;
    f_v[t] = v;
    f_i[t] = i;
  }
  __syncthreads();
  const uint32_t am = residue_argmax(f_v, f_i);
  if (t == 0) {
    *argmax_out = am;
    *counter = 0u;
  }
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

// shaders/gelu_mul.wgsl:14-16.
__global__ void gelu_mul_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                float* __restrict__ out, uint32_t n) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float g = gate[i];
    float a = k0 * g * (1.0f + k1 * g * g);
    a = a < -15.0f ? -15.0f : (a > 15.0f ? 15.0f : a);
    out[i] = (0.5f * g * (1.0f + tanhf(a))) * up[i];
  }
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

__global__ void init_slots_kernel(unsigned long long* slots, uint32_t* counter) {
  slots[threadIdx.x] = pack_key(kFloor, 0u);
  if (threadIdx.x == 0) *counter = 0u;
}

int g_sm_count = 0;

int sm_count() {
  if (g_sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  return g_sm_count;
}

}  // namespace

cudaError_t init_select_scratch(const SelectScratch& sc, cudaStream_t s) {
  init_slots_kernel<<<1, 256, 0, s>>>(sc.slots, sc.counter);
  return cudaGetLastError();
}

cudaError_t launch_lmhead_select(const uint8_t* w, const float* x, uint32_t V, uint32_t N, float cap,
                                 uint32_t row_offset, float* logits_opt, float* cand_val, uint32_t* cand_idx,
                                 uint32_t* argmax, const SelectScratch& scratch, cudaStream_t s) {
  const uint32_t rows_per_cta = kSelWarps;
  uint32_t grid = (V + rows_per_cta - 1) / rows_per_cta;
  const uint32_t cap_grid = (uint32_t)sm_count() * 8u;
  if (grid > cap_grid) grid = cap_grid;
  if (grid == 0) grid = 1;
  lmhead_select_kernel<<<grid, kSelWarps * 32, 0, s>>>(w, x, V, N, cap, row_offset, logits_opt, cand_val, cand_idx,
                                                       argmax, scratch.slots, scratch.counter);
  return cudaGetLastError();
}

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

cudaError_t launch_merge_candidates(const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                                    uint32_t* out_idx, uint32_t* argmax, cudaStream_t s) {
  merge_kernel<<<1, 256, 0, s>>>(vals, idx, G, out_val, out_idx, argmax);
  return cudaGetLastError();
}

}  // namespace q4k
