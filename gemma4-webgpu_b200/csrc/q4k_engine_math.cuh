// Device math of the GEMV engines shared by the plan engine (q4k_engine.cu)
// and the chained decode step (q4k_chain.cu): the register-A tensor-core MAC,
// the per-token power-of-two scale of the activation split, and one Q4_K
// super-block of a lane's two tile rows (exact f16 weights, q4k_dequant.cuh).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_dequant.cuh"

namespace q4k {
namespace {

// Not volatile: a pure function of its operands, so the compiler may
// schedule it freely among the shared-memory loads and the dequantization.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint2 b) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

__device__ __forceinline__ uint32_t word_of(const uint4& a, const uint4& b, int w) {
  switch (w) {
    case 0: return a.x;
    case 1: return a.y;
    case 2: return a.z;
    case 3: return a.w;
    case 4: return b.x;
    case 5: return b.y;
    case 6: return b.z;
    default: return b.w;
  }
}

// Power-of-two scale s with max|x| * s < 2^15 (exponent clamped), as
// (s, 1/s).
__device__ __forceinline__ float2 token_scale(float mx) {
  int e = 0, sexp = 0;
  if (mx > 0.0f && mx <= 3.402823466e38f) {
    frexpf(mx, &e);  // mx < 2^e
    sexp = 15 - e;
    sexp = sexp > 100 ? 100 : (sexp < -100 ? -100 : sexp);
  }
  return make_float2(ldexpf(1.0f, sexp), ldexpf(1.0f, -sexp));
}

// The 96 bytes of one super-block a lane needs: both rows' header and qs group.
struct BlockRegs {
  uint4 ha, hb, qa0, qa1, qb0, qb1;
};

// Shared-memory loads as plain C++ loads (pointers into the kernel's
// dynamic shared memory, so they compile to LDS): the compiler keeps them
// after the stage's barrier wait and before the stage is handed back (both
// asm statements clobber memory) and is otherwise free to schedule them.
__device__ __forceinline__ uint4 sld128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ BlockRegs read_block(const uint8_t* ra_p, const uint8_t* rb_p, uint32_t c) {
  BlockRegs r;
  r.ha = sld128(ra_p);
  r.hb = sld128(rb_p);
  r.qa0 = sld128(ra_p + 16 + 32 * c);
  r.qa1 = sld128(ra_p + 32 + 32 * c);
  r.qb0 = sld128(rb_p + 16 + 32 * c);
  r.qb1 = sld128(rb_p + 32 + 32 * c);
  return r;
}

// This lane's B fragments of k-steps w and w+8 (one 16-byte load): from the
// CTA's shared-memory activation cache (SX) or from global memory.
template <bool SX>
__device__ __forceinline__ uint4 load_frag(const uint8_t* p) {
  if constexpr (SX) return *reinterpret_cast<const uint4*>(p);
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// The math of one super-block: 2 rows x 64 weights per lane -> 16 (or 16*NT)
// mma.sync.  base[n]: address of this lane's fragments of word 0 of the
// block; COLS > 0 fixes the column count (batch = COLS/2 <= 4), making every
// word offset an immediate.
template <int NT, int COLS, bool SX>
__device__ __forceinline__ void block_math(float (&acc)[NT][2][4], const BlockRegs& R, uint32_t c, uint32_t bsel,
                                           const uint8_t* const (&base)[NT], const uint32_t (&wstep)[NT]) {
  const RowConsts ka = row_consts(R.ha, c, bsel);
  const RowConsts kb = row_consts(R.hb, c, bsel);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const WordPairs A = dequant_word(word_of(R.qa0, R.qa1, w), ka);
    const WordPairs B = dequant_word(word_of(R.qb0, R.qb1, w), kb);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint32_t ws = COLS > 0 ? (uint32_t)COLS * 64u : wstep[n];
      const uint4 f = load_frag<SX>(base[n] + w * ws);
      mma_16816(acc[n][0], A.lo02, B.lo02, A.lo13, B.lo13, make_uint2(f.x, f.y));
      mma_16816(acc[n][1], A.hi02, B.hi02, A.hi13, B.hi13, make_uint2(f.z, f.w));
    }
  }
}

}  // namespace
}  // namespace q4k
