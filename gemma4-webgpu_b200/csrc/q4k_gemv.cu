// Q4_K GEMV on CUDA cores: the drop-in for shaders/matmul_quant.wgsl and
// shaders/matmul_quant_mr4.wgsl (same y = sum_k f32(w16[m,k]) * x[k], f32
// accumulation), reading the 144-byte Q4_K super-blocks directly instead of a
// pre-dequantized f16 buffer.
//
// Mapping ("rowwarp"): one warp per output row; lane l takes 32-byte qs groups
// u = l, l+32, ... of the row (group = half of the 64 weights of sub-blocks
// 2g and 2g+1 of block u/4), decodes the block header, dequantizes its 64
// weights to f16-rounded f32 in registers and FMAs them with x; a warp
// shuffle reduces the 32 lane partials.  x is read through the L1/L2 (every
// warp of the GPU reads the same vector).
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_device.cuh"
#include "q4k_kernels.cuh"

namespace q4k {
namespace {

template <int BT>
__global__ void __launch_bounds__(256) gemv_rowwarp_kernel(const uint8_t* __restrict__ w,
                                                           const float* __restrict__ x, float* __restrict__ y,
                                                           uint32_t M, uint32_t N, uint32_t ldx, uint32_t ldy) {
  const uint32_t warps = blockDim.x >> 5;
  const uint64_t row = (uint64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= M) return;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t nb = N / kQK;
  const uint8_t* wr = w + row * (uint64_t)nb * kBlockBytes;

  float acc[BT];
#pragma unroll
  for (int b = 0; b < BT; ++b) acc[b] = 0.0f;

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
      float wl[4], wh[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (qw[i] >> (8 * j)) & 0xffu;
        wl[j] = weight_f16r(ds0, dm0, byte & 15u);
        wh[j] = weight_f16r(ds1, dm1, byte >> 4);
      }
#pragma unroll
      for (int b = 0; b < BT; ++b) {
        const float4 xl = *reinterpret_cast<const float4*>(x + (uint64_t)b * ldx + k0 + 4 * i);
        const float4 xh = *reinterpret_cast<const float4*>(x + (uint64_t)b * ldx + k0 + 32 + 4 * i);
        acc[b] = fmaf(wl[0], xl.x, acc[b]);
        acc[b] = fmaf(wl[1], xl.y, acc[b]);
        acc[b] = fmaf(wl[2], xl.z, acc[b]);
        acc[b] = fmaf(wl[3], xl.w, acc[b]);
        acc[b] = fmaf(wh[0], xh.x, acc[b]);
        acc[b] = fmaf(wh[1], xh.y, acc[b]);
        acc[b] = fmaf(wh[2], xh.z, acc[b]);
        acc[b] = fmaf(wh[3], xh.w, acc[b]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < BT; ++b) {
    const float s = warp_sum(acc[b]);
    if (lane == 0) y[(uint64_t)b * ldy + row] = s;
  }
}

template <int BT>
cudaError_t launch_rowwarp(const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t ldx,
                           uint32_t ldy, cudaStream_t s) {
  const uint32_t threads = 256, rows_per_cta = threads / 32;
  const uint32_t grid = (M + rows_per_cta - 1) / rows_per_cta;
  gemv_rowwarp_kernel<BT><<<grid, threads, 0, s>>>(w, x, y, M, N, ldx, ldy);
  return cudaGetLastError();
}

// One thread per 8 weights: Q4_K -> f16 bit patterns (debug / parity entry).
__global__ void dequant_f16_kernel(const uint8_t* __restrict__ w, uint16_t* __restrict__ out, uint64_t n_blocks) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t blk_i = t >> 5;  // 32 threads per block of 256 weights
  if (blk_i >= n_blocks) return;
  const uint32_t part = (uint32_t)(t & 31u);  // 4 bytes of qs each
  const uint8_t* blk = w + blk_i * kBlockBytes;
  const uint4 h = *reinterpret_cast<const uint4*>(blk);
  const ScaleMin4 sm = unpack_scale_min(h.y, h.z, h.w);
  const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
  const uint32_t g = part >> 3, l0 = (part & 7u) * 4;  // group, first byte in group
  uint32_t sc0, m0, sc1, m1;
  scale_min(sm, 2 * g, sc0, m0);
  scale_min(sm, 2 * g + 1, sc1, m1);
  const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0;
  const float ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
  const uint32_t q = *reinterpret_cast<const uint32_t*>(blk + 16 + 32 * g + l0);
  uint16_t lo[4], hi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t byte = (q >> (8 * j)) & 0xffu;
    lo[j] = weight_f16_bits(ds0, dm0, byte & 15u);
    hi[j] = weight_f16_bits(ds1, dm1, byte >> 4);
  }
  uint16_t* o = out + blk_i * kQK + 64 * g + l0;
  *reinterpret_cast<uint2*>(o) = make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
  *reinterpret_cast<uint2*>(o + 32) =
      make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
}

}  // namespace

cudaError_t launch_gemv(const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
                        uint32_t ldx, uint32_t ldy, int variant, cudaStream_t s) {
  (void)variant;
  // Batches are processed in chunks of 8/4/2/1 activation rows; every chunk
  // streams the weights once.
  uint32_t done = 0;
  while (done < batch) {
    const uint32_t left = batch - done;
    const float* xc = x + (uint64_t)done * ldx;
    float* yc = y + (uint64_t)done * ldy;
    cudaError_t e;
    uint32_t step;
    if (left >= 8) {
      e = launch_rowwarp<8>(w, xc, yc, M, N, ldx, ldy, s);
      step = 8;
    } else if (left >= 4) {
      e = launch_rowwarp<4>(w, xc, yc, M, N, ldx, ldy, s);
      step = 4;
    } else if (left >= 2) {
      e = launch_rowwarp<2>(w, xc, yc, M, N, ldx, ldy, s);
      step = 2;
    } else {
      e = launch_rowwarp<1>(w, xc, yc, M, N, ldx, ldy, s);
      step = 1;
    }
    if (e != cudaSuccess) return e;
    done += step;
  }
  return cudaSuccess;
}

cudaError_t launch_dequant_f16(const uint8_t* w, uint16_t* out, uint64_t n_blocks, cudaStream_t s) {
  const uint64_t threads = n_blocks * 32;
  const uint32_t tpb = 256;
  const uint64_t grid = (threads + tpb - 1) / tpb;
  dequant_f16_kernel<<<(unsigned)grid, tpb, 0, s>>>(w, out, n_blocks);
  return cudaGetLastError();
}

}  // namespace q4k
