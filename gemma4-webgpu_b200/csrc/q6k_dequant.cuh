// Exact reference weights from Q6_K super-blocks on the CUDA cores (shared by
// the GEMV engine and the weight-probe kernel).
//
// Reference semantics (src/gguf.ts:316-368 then f32ToF16Array :425-473):
//   w16 = f16_rne(f32(d * sc * (q - 32)))
// with d the block's f16 scale, sc the int8 scale of the weight's 16-element
// sub-block and q its 6-bit quant (4 bits of ql, 2 bits of qh).  The product
// is exact in f32 (d has 11 significant bits, |sc*(q-32)| <= 4096), so the
// reference's f64 evaluation and Float32Array store give exactly d*sc*(q-32).
//
// Device layout ("Q6_K planar", written once at load by q4k_q6k_repack from
// the GGUF bytes -- the counterpart of the reference's load-time
// dequantizeQ6_K + f32ToF16Array upload):
//   bodies  [M][N/256][208]  bytes 0..207 of each GGUF super-block
//                            (ql[128] | qh[64] | int8 scales[16])
//   d plane [N/256][Mp]      f16 d of super-block b of row m at [b][m],
//                            Mp = M rounded up to 8 (zero padded)
// Bodies stay 16-byte aligned (208 = 13 * 16), so tiles of them move by TMA;
// the d plane's rows are 16-byte multiples, so a tile's 16 d values are one
// 32-byte box.  The size is the GGUF size plus at most 14 bytes per
// super-block column.
//
// Per 32-bit word: lane (g, c) owns the 64 weights 64c..64c+63 of a block
// (the same k positions as a Q4_K lane): half h = c/2, quarters 2(c&1) and
// 2(c&1)+1 of that half.  Word w (columns l = 4w..4w+3 of the half) gives 8
// weights per row: 4 of the low quarter (k = 64c+4w+j) and 4 of the high
// quarter (k = 64c+32+4w+j), j = 0..3 -- the Q4_K engine's k-steps w and
// w+8, so both formats read the same prepared activations.
//   1. 6-bit quants of 4 columns as bytes: nibbles (shifted down 4 bits in
//      odd lanes) | 2 bits of qh << 4                    (9 ALU ops)
//   2. each byte into an f32 magic 0x42XX0000 = 32 + q/4 (one PRMT per weight)
//   3. fma.rn.f32x2: (32 + q/4) * 4*d*sc - 160*d*sc = d*sc*(q-32), exact
//      (one FFMA2 per weight pair)
//   4. cvt.rn.f16x2.f32 -> the f16 weight pair (round to nearest even)
// The fused step 3 matches the reference for every finite d, except that an
// exactly zero weight comes out +0 (the reference's sign of zero follows d,
// sc and q-32).  The exact variant (EXACT = true) evaluates (32 + q/4 - 40) *
// 4*d*sc instead: every bit, signed zeros, infinities and NaN included.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_dequant.cuh"

namespace q4k {

constexpr uint32_t kQ6BlockBytes = 210;  // GGUF super-block
constexpr uint32_t kQ6BodyBytes = 208;   // device body: ql | qh | scales
constexpr uint32_t kQ6BodyWords = kQ6BodyBytes / 4;

// Entries per row of the d plane (M rounded up to 8: 16-byte rows).
__host__ __device__ inline uint32_t q6k_dpitch(uint32_t M) { return (M + 7u) & ~7u; }

// Bytes of the device layout of an M x N Q6_K matrix.
__host__ __device__ inline uint64_t q6k_device_bytes(uint32_t M, uint32_t N) {
  const uint64_t nb = N >> 8;
  return (uint64_t)M * nb * kQ6BodyBytes + nb * q6k_dpitch(M) * 2u;
}

__device__ __forceinline__ uint64_t f32x2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}

// One row's constants for one 16-column half of a lane's block: the scale
// pairs (4*d*sc, 4*d*sc) and (-160*d*sc, ...) of its low and high quarter.
struct Q6Consts {
  uint64_t dlo, clo, dhi, chi;
};

// scw: the lane's scale word (bytes 4c..4c+3 of the scales: low quarter
// columns 0-15, 16-31, high quarter columns 0-15, 16-31); is: column half;
// d4 = 4*d as f32.
__device__ __forceinline__ Q6Consts q6_consts(uint32_t scw, uint32_t is, float d4) {
  const float slo = (float)(int8_t)(scw >> (8u * is));
  const float shi = (float)(int8_t)(scw >> (16u + 8u * is));
  const float dlo = d4 * slo, dhi = d4 * shi;  // exact: 11 x 8 significant bits
  const float clo = -40.0f * dlo, chi = -40.0f * dhi;
  Q6Consts k;
  k.dlo = f32x2(dlo, dlo);
  k.clo = f32x2(clo, clo);
  k.dhi = f32x2(dhi, dhi);
  k.chi = f32x2(chi, chi);
  return k;
}

// Word w of a lane's half-block (ql0 = ql bytes 4w..4w+3 of the half, ql1 =
// the bytes 32 further, qh = qh bytes 4w..4w+3 of the half; sh = 4 in odd
// lanes, else 0) -> four f16x2 weight pairs in the Q4_K engine's order:
// lo02 = (w[col 0], w[col 2]), lo13 = (w[col 1], w[col 3]) of the low
// quarter, hi02 / hi13 of the high quarter.
template <bool EXACT>
__device__ __forceinline__ WordPairs dequant6_word(uint32_t ql0, uint32_t ql1, uint32_t qh, uint32_t sh,
                                                   const Q6Consts& k) {
  WordPairs o;
  if constexpr (!EXACT) {
    asm("{\n\t"
        ".reg .b32 a0, a1, hq, t4, t2, lo, hi, v0, v1, v2, v3, u0, u1, u2, u3;\n\t"
        ".reg .b32 e0, e1, e2, e3, f0, f1, f2, f3;\n\t"
        ".reg .b64 p02, p13, r02, r13, s02, s13, x02, x13, y02, y13;\n\t"
        "shr.b32 a0, %4, %7;\n\t"
        "shr.b32 a1, %5, %7;\n\t"
        "shr.b32 hq, %6, %7;\n\t"
        "shl.b32 t4, hq, 4;\n\t"
        "shl.b32 t2, hq, 2;\n\t"
        "lop3.b32 lo, a0, t4, 0x0F0F0F0F, 0xE4;\n\t"  // (a & c) | (b & ~c)
        "and.b32 lo, lo, 0x3F3F3F3F;\n\t"
        "lop3.b32 hi, a1, t2, 0x0F0F0F0F, 0xE4;\n\t"
        "and.b32 hi, hi, 0x3F3F3F3F;\n\t"
        "prmt.b32 v0, lo, 0x42000000, 0x7044;\n\t"      // 0x42qq0000 = 32 + q/4
        "prmt.b32 v1, lo, 0x42000000, 0x7144;\n\t"
        "prmt.b32 v2, lo, 0x42000000, 0x7244;\n\t"
        "prmt.b32 v3, lo, 0x42000000, 0x7344;\n\t"
        "prmt.b32 u0, hi, 0x42000000, 0x7044;\n\t"
        "prmt.b32 u1, hi, 0x42000000, 0x7144;\n\t"
        "prmt.b32 u2, hi, 0x42000000, 0x7244;\n\t"
        "prmt.b32 u3, hi, 0x42000000, 0x7344;\n\t"
        "mov.b64 p02, {v0, v2};\n\t"
        "mov.b64 p13, {v1, v3};\n\t"
        "mov.b64 r02, {u0, u2};\n\t"
        "mov.b64 r13, {u1, u3};\n\t"
        "fma.rn.f32x2 s02, p02, %8, %9;\n\t"             // d*sc*(q-32), exact
        "fma.rn.f32x2 s13, p13, %8, %9;\n\t"
        "fma.rn.f32x2 x02, r02, %10, %11;\n\t"
        "fma.rn.f32x2 x13, r13, %10, %11;\n\t"
        "mov.b64 {e0, e2}, s02;\n\t"
        "mov.b64 {e1, e3}, s13;\n\t"
        "mov.b64 {f0, f2}, x02;\n\t"
        "mov.b64 {f1, f3}, x13;\n\t"
        "cvt.rn.f16x2.f32 %0, e2, e0;\n\t"               // f16 RNE, (lo, hi) halves
        "cvt.rn.f16x2.f32 %1, e3, e1;\n\t"
        "cvt.rn.f16x2.f32 %2, f2, f0;\n\t"
        "cvt.rn.f16x2.f32 %3, f3, f1;\n\t"
        "}"
        : "=r"(o.lo02), "=r"(o.lo13), "=r"(o.hi02), "=r"(o.hi13)
        : "r"(ql0), "r"(ql1), "r"(qh), "r"(sh), "l"(k.dlo), "l"(k.clo), "l"(k.dhi), "l"(k.chi));
  } else {
    asm("{\n\t"
        ".reg .b32 a0, a1, hq, t4, t2, lo, hi, v0, v1, v2, v3, u0, u1, u2, u3;\n\t"
        ".reg .b32 e0, e1, e2, e3, f0, f1, f2, f3;\n\t"
        ".reg .b64 p02, p13, r02, r13, s02, s13, x02, x13, m40;\n\t"
        "mov.b64 m40, {0xC2200000, 0xC2200000};\n\t"    // (-40, -40)
        "shr.b32 a0, %4, %7;\n\t"
        "shr.b32 a1, %5, %7;\n\t"
        "shr.b32 hq, %6, %7;\n\t"
        "shl.b32 t4, hq, 4;\n\t"
        "shl.b32 t2, hq, 2;\n\t"
        "lop3.b32 lo, a0, t4, 0x0F0F0F0F, 0xE4;\n\t"
        "and.b32 lo, lo, 0x3F3F3F3F;\n\t"
        "lop3.b32 hi, a1, t2, 0x0F0F0F0F, 0xE4;\n\t"
        "and.b32 hi, hi, 0x3F3F3F3F;\n\t"
        "prmt.b32 v0, lo, 0x42000000, 0x7044;\n\t"
        "prmt.b32 v1, lo, 0x42000000, 0x7144;\n\t"
        "prmt.b32 v2, lo, 0x42000000, 0x7244;\n\t"
        "prmt.b32 v3, lo, 0x42000000, 0x7344;\n\t"
        "prmt.b32 u0, hi, 0x42000000, 0x7044;\n\t"
        "prmt.b32 u1, hi, 0x42000000, 0x7144;\n\t"
        "prmt.b32 u2, hi, 0x42000000, 0x7244;\n\t"
        "prmt.b32 u3, hi, 0x42000000, 0x7344;\n\t"
        "mov.b64 p02, {v0, v2};\n\t"
        "mov.b64 p13, {v1, v3};\n\t"
        "mov.b64 r02, {u0, u2};\n\t"
        "mov.b64 r13, {u1, u3};\n\t"
        "add.rn.f32x2 p02, p02, m40;\n\t"                // q/4 - 8, exact, +0 at q = 32
        "add.rn.f32x2 p13, p13, m40;\n\t"
        "add.rn.f32x2 r02, r02, m40;\n\t"
        "add.rn.f32x2 r13, r13, m40;\n\t"
        "mul.rn.f32x2 s02, p02, %8;\n\t"                 // (q/4 - 8) * 4*d*sc
        "mul.rn.f32x2 s13, p13, %8;\n\t"
        "mul.rn.f32x2 x02, r02, %9;\n\t"
        "mul.rn.f32x2 x13, r13, %9;\n\t"
        "mov.b64 {e0, e2}, s02;\n\t"
        "mov.b64 {e1, e3}, s13;\n\t"
        "mov.b64 {f0, f2}, x02;\n\t"
        "mov.b64 {f1, f3}, x13;\n\t"
        "cvt.rn.f16x2.f32 %0, e2, e0;\n\t"
        "cvt.rn.f16x2.f32 %1, e3, e1;\n\t"
        "cvt.rn.f16x2.f32 %2, f2, f0;\n\t"
        "cvt.rn.f16x2.f32 %3, f3, f1;\n\t"
        "}"
        : "=r"(o.lo02), "=r"(o.lo13), "=r"(o.hi02), "=r"(o.hi13)
        : "r"(ql0), "r"(ql1), "r"(qh), "r"(sh), "l"(k.dlo), "l"(k.dhi));
  }
  return o;
}

}  // namespace q4k
