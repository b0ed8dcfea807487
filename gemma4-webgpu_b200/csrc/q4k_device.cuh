// Device-side building blocks shared by the Q4_K kernels.
//
// Q4_K super-block (src/gguf.ts:157-210, 144 bytes, 256 weights):
//   bytes 0..1   f16 d        bytes 2..3  f16 dmin
//   bytes 4..15  8 x (6-bit scale, 6-bit min), packed (getScaleMin, :175-182)
//   bytes 16..143 qs: group g (0..3) = qs[32g .. 32g+31]; low nibble of qs[32g+l]
//                is element 64g+l (sub-block 2g), high nibble is element
//                64g+32+l (sub-block 2g+1).
//
// Weight semantics (what the reference GPU multiplies): w = f16_rne(f32(d*sc*q - dmin*m)).
// d*sc and dmin*m are exact in f32 (11 x 6 significant bits), so
// fmaf(d*sc, q, -(dmin*m)) rounds the exact value once to f32, the same f32
// the reference stores after evaluating d1*q - min1 in f64 (src/gguf.ts:194-204).
// __float2half_rn is the IEEE round-to-nearest-even of Float16Array.set.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace q4k {

constexpr int kQK = 256;          // weights per super-block
constexpr int kBlockBytes = 144;  // bytes per super-block

// The 8 (scale, min) pairs of a block as four byte-packed words:
// sc[0..3], m[0..3], sc[4..7], m[4..7] (byte j of each word = sub-block j%4).
struct ScaleMin4 {
  uint32_t sc_lo, m_lo, sc_hi, m_hi;
};

__device__ __forceinline__ ScaleMin4 unpack_scale_min(uint32_t w0, uint32_t w1, uint32_t w2) {
  ScaleMin4 r;
  r.sc_lo = w0 & 0x3f3f3f3fu;
  r.m_lo = w1 & 0x3f3f3f3fu;
  r.sc_hi = (w2 & 0x0f0f0f0fu) | ((w0 >> 2) & 0x30303030u);
  r.m_hi = ((w2 >> 4) & 0x0f0f0f0fu) | ((w1 >> 2) & 0x30303030u);
  return r;
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xffu; }

// (scale, min) of sub-block j (0..7).
__device__ __forceinline__ void scale_min(const ScaleMin4& s, int j, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = byte_of(s.sc_lo, j);
    m = byte_of(s.m_lo, j);
  } else {
    sc = byte_of(s.sc_hi, j - 4);
    m = byte_of(s.m_hi, j - 4);
  }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu)));
}

// The reference weight value for nibble q with per-sub-block ds = d*sc and
// dm = dmin*m: f16-rounded, returned as f32.
__device__ __forceinline__ float weight_f16r(float ds, float dm, uint32_t q) {
  return __half2float(__float2half_rn(fmaf(ds, (float)q, -dm)));
}

__device__ __forceinline__ uint16_t weight_f16_bits(float ds, float dm, uint32_t q) {
  return __half_as_ushort(__float2half_rn(fmaf(ds, (float)q, -dm)));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Softcap of shaders/logit_softcap.wgsl:13-15: tanh(clamp(v/cap, -15, 15))*cap.
// The clamp is written with comparisons so a NaN logit stays NaN (and then
// never wins a selection), as in the CPU restatement.
__device__ __forceinline__ float softcap(float v, float cap) {
  float t = v / cap;
  t = t < -15.0f ? -15.0f : (t > 15.0f ? 15.0f : t);
  return tanhf(t) * cap;
}

// shaders/gelu_mul.wgsl:14-16: GELU(tanh)(g) * u.  One definition shared by
// the gelu_mul op and the activation preparation that evaluates it on the
// fly, so both produce the same bits.
__device__ __forceinline__ float gelu_mul_value(float g, float u) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float a = k0 * g * (1.0f + k1 * g * g);
  a = a < -15.0f ? -15.0f : (a > 15.0f ? 15.0f : a);
  return (0.5f * g * (1.0f + tanhf(a))) * u;
}

// Selection order of the reference's argmax / topk256 scans
// (shaders/argmax.wgsl:12-20, topk256.wgsl:10-17): a first strict maximum over
// ascending indices, started at (-1e30, 0), equals the maximum under float
// '>' with ties going to the lower index.  `better` is that order; NaN never
// wins because every comparison with it is false.
__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// Order key for the cross-warp atomicMax merge of selection candidates:
// larger value first, then lower index; -0.0 orders with +0.0 and keeps its
// sign in bit 0.  Index < 2^31.
__device__ __forceinline__ unsigned long long sel_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  const uint32_t neg_zero = (b == 0x80000000u) ? 1u : 0u;
  if (neg_zero) b = 0u;
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | ((unsigned long long)(0x7fffffffu - idx) << 1) | neg_zero;
}

__device__ __forceinline__ void sel_unkey(unsigned long long k, float& v, uint32_t& idx) {
  const uint32_t ord = (uint32_t)(k >> 32);
  uint32_t b = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
  if (k & 1ull) b = 0x80000000u;
  v = __uint_as_float(b);
  idx = 0x7fffffffu - (uint32_t)((k >> 1) & 0x7fffffffu);
}

}  // namespace q4k
