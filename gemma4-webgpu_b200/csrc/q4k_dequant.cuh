// Exact reference weights from Q4_K nibbles on the CUDA cores, 8 per 32-bit
// word (shared by the GEMV engine and the GEMM's A-operand producers).
//
// w16 = f16_rne(f32(d*sc*q - dmin*m)) (src/gguf.ts:168-210 + 425-473):
//   1. nibble pairs -> f16 magic values 1024+q      (one LOP3 per pair)
//   2. HFMA2 (1024+q)*sc - 1024*sc = sc*q, exact   (one per pair)
//   3. mixed FMA d(f16)*(sc*q)(f16) - dmin*m (f32) = f32(d*sc*q - dmin*m), the
//      exact product rounded once, as the reference's f64 expression then
//      Float32Array store rounds it
//   4. cvt.rn.f16x2.f32 -> the f16 weight pair (round to nearest even)
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_device.cuh"

namespace q4k {

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// d(f32) = a(f16) * b(f16) + c(f32), one rounding (sm_100 mixed-precision FMA).
__device__ __forceinline__ float fma_h_h_f(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// ---- per (row, super-block) constants ------------------------------------------

// What one lane needs to dequantize its qs group c of one row's block:
// sub-block j0 = 2c (low nibbles) and j1 = 2c+1 (high nibbles).
struct RowConsts {
  uint32_t sc0, nsc0;  // f16x2 (sc_j0, sc_j0), (-1024 sc_j0, ...)
  uint32_t sc1, nsc1;  // f16x2 (sc_j1/16, ...), (-64 sc_j1, ...)
  float ndm0, ndm1;    // -dmin*m_j0, -dmin*m_j1 (exact in f32)
  uint16_t d;          // f16 bits of d
};

// prmt selector picking bytes (2(c&1), 2(c&1)+1) of a packed scale word --
// the (scale, min) slots of sub-blocks 2c, 2c+1 -- into bytes 0 and 2, zeros
// elsewhere.
__host__ __device__ constexpr uint32_t scale_sel(uint32_t c) {
  return (c & 1u) ? ((4u << 12) | (3u << 8) | (4u << 4) | 2u) : ((4u << 12) | (1u << 8) | (4u << 4) | 0u);
}

__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// sel = scale_sel(c).  Every step is exact: the 6-bit values enter as f16
// magic numbers (1024 + v, or -(1024 + v) with the sign byte 0xE4), which one
// f16 add turns into v; the products by -1024, 1/16 and -64 are powers of
// two applied to values of at most 6 significant bits.
__device__ __forceinline__ RowConsts row_consts(const uint4& h, uint32_t c, uint32_t sel) {
  RowConsts r;
  const ScaleMin4 sm = unpack_scale_min(h.y, h.z, h.w);
  const uint32_t scw = c < 2 ? sm.sc_lo : sm.sc_hi;
  const uint32_t mw = c < 2 ? sm.m_lo : sm.m_hi;
  // sel picks bytes (s, s+1) into halves 0 and 1 (s = 2(c&1)); sel ^ 0x100
  // broadcasts byte s, sel | 1 broadcasts byte s+1
  const uint32_t s0 = prmt(scw, 0x64646464u, sel ^ 0x100u);  // (1024 + sc_j0) x2
  const uint32_t s1 = prmt(scw, 0x64646464u, sel | 1u);      // (1024 + sc_j1) x2
  r.sc0 = hadd2(s0, 0xE400E400u);                            // sc_j0 x2
  r.nsc0 = hmul2(r.sc0, 0xE400E400u);                        // -1024 sc_j0
  r.sc1 = hfma2(s1, 0x2C002C00u, 0xD400D400u);               // (1024 + sc)/16 - 64 = sc_j1/16
  r.nsc1 = hmul2(r.sc1, 0xE400E400u);                        // -64 sc_j1
  const uint32_t nm = hadd2(prmt(mw, 0xE4E4E4E4u, sel), 0x64006400u);  // (-m_j0, -m_j1)
  const uint16_t dmin = (uint16_t)(h.x >> 16);
  r.ndm0 = fma_h_h_f(dmin, (uint16_t)(nm & 0xffffu), 0.0f);  // -dmin*m, exact
  r.ndm1 = fma_h_h_f(dmin, (uint16_t)(nm >> 16), 0.0f);
  r.d = (uint16_t)(h.x & 0xffffu);
  return r;
}

// One 32-bit word of nibbles (bytes b0..b3 of one row) -> four f16x2 weight
// pairs: lo02 = (w[b0 lo], w[b2 lo]), lo13 = (w[b1 lo], w[b3 lo]), and the
// same for the high nibbles.  Low nibbles belong to sub-block j0, high to j1.
// One PTX block, so the f16 halves feed the mixed FMAs without integer
// extraction.
struct WordPairs {
  uint32_t lo02, lo13, hi02, hi13;
};

__device__ __forceinline__ WordPairs dequant_word(uint32_t v, const RowConsts& r) {
  WordPairs o;
  asm("{\n\t"
      ".reg .b32 v8, m0, m1, m2, m3, p0, p1, p2, p3;\n\t"
      ".reg .b16 a0, a1, b0, b1, c0, c1, d0, d1;\n\t"
      ".reg .f32 e0, e1, e2, e3, e4, e5, e6, e7;\n\t"
      "shr.b32 v8, %4, 8;\n\t"
      "lop3.b32 m0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"   // (v & mask) | magic
      "lop3.b32 m1, v8, 0x000F000F, 0x64006400, 0xEA;\n\t"
      "lop3.b32 m2, %4, 0x00F000F0, 0x64006400, 0xEA;\n\t"
      "lop3.b32 m3, v8, 0x00F000F0, 0x64006400, 0xEA;\n\t"
      "fma.rn.f16x2 p0, m0, %5, %6;\n\t"                    // sc*q, exact
      "fma.rn.f16x2 p1, m1, %5, %6;\n\t"
      "fma.rn.f16x2 p2, m2, %7, %8;\n\t"
      "fma.rn.f16x2 p3, m3, %7, %8;\n\t"
      "mov.b32 {a0, a1}, p0;\n\t"
      "mov.b32 {b0, b1}, p1;\n\t"
      "mov.b32 {c0, c1}, p2;\n\t"
      "mov.b32 {d0, d1}, p3;\n\t"
      "fma.rn.f32.f16 e0, %11, a0, %9;\n\t"                 // d*sc*q - dmin*m, one rounding
      "fma.rn.f32.f16 e1, %11, a1, %9;\n\t"
      "fma.rn.f32.f16 e2, %11, b0, %9;\n\t"
      "fma.rn.f32.f16 e3, %11, b1, %9;\n\t"
      "fma.rn.f32.f16 e4, %11, c0, %10;\n\t"
      "fma.rn.f32.f16 e5, %11, c1, %10;\n\t"
      "fma.rn.f32.f16 e6, %11, d0, %10;\n\t"
      "fma.rn.f32.f16 e7, %11, d1, %10;\n\t"
      "cvt.rn.f16x2.f32 %0, e1, e0;\n\t"                     // f16 RNE, (lo, hi) halves
      "cvt.rn.f16x2.f32 %1, e3, e2;\n\t"
      "cvt.rn.f16x2.f32 %2, e5, e4;\n\t"
      "cvt.rn.f16x2.f32 %3, e7, e6;\n\t"
      "}"
      : "=r"(o.lo02), "=r"(o.lo13), "=r"(o.hi02), "=r"(o.hi13)
      : "r"(v), "r"(r.sc0), "r"(r.nsc0), "r"(r.sc1), "r"(r.nsc1), "f"(r.ndm0), "f"(r.ndm1), "h"(r.d));
  return o;
}

}  // namespace q4k
