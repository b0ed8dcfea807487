// Q4_K GEMV engine for sm_100a.
//
// y[t, m] = sum_k f32(w16[m, k]) * x[t, k], w16 = f16_rne(f32(d*sc*q - dmin*m))
// (the weight the reference GPU multiplies: src/gguf.ts:168-210 + 425-473,
// shaders/matmul_quant.wgsl:35), for t < batch <= 16.
//
// Work decomposition: a persistent grid of 8-warp CTAs walks a list of work
// items; an item is a 16-row tile of one GEMV task (tasks = the GEMVs of one
// launch: a single call, or every GEMV of a plan stage).  A warp owns one
// item at a time and streams the tile's 144-byte super-blocks straight from
// HBM into registers with 128-bit loads, one block ahead of the math.
//
// Per item, lane (g = lane/4, c = lane%4) owns rows g and g+8 of the tile and
// qs group c (sub-blocks 2c, 2c+1) of every super-block.  For each 32-bit word
// of nibbles it produces the exact reference weights on the CUDA cores:
//   1. nibble pairs -> f16 magic values 1024+q      (one LOP3 per pair)
//   2. HFMA2 (1024+q)*sc - 1024*sc = sc*q, exact   (one per pair)
//   3. mixed FMA d(f16)*(sc*q)(f16) - dmin*m (f32) = f32(d*sc*q - dmin*m), the
//      exact product rounded once, as the reference's f64 expression then
//      Float32Array store rounds it
//   4. cvt.rn.f16x2.f32 -> the f16 weight pair (round to nearest even)
// and feeds the f16 pairs to mma.sync m16n8k16 as the A operand.  The tensor
// core is only the multiply-accumulate engine: its B operand is x split
// exactly into f16 hi/lo parts (2 columns per token), so f16 x f16 products
// are exact and accumulate in f32; the two columns add up to the f32 dot
// product of the f16 weights with x to ~2^-22 relative per term.
#include <cuda_fp16.h>
#include <stdint.h>

#include "q4k_device.cuh"
#include "q4k_engine.cuh"

namespace q4k {
namespace {

constexpr float kFloorE = -1e30f;

// ---- small PTX helpers -------------------------------------------------------

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

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

// {hi, lo} f32 -> f16x2 (lo in the low half), round to nearest even.
__device__ __forceinline__ uint32_t cvt_f16x2(float hi, float lo) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ uint2 ldg_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint2 b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
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

// sel: prmt selector picking the (j0, j1) bytes of a packed scale word into
// bytes 0 and 2, zeros elsewhere (precomputed from c).
__device__ __forceinline__ RowConsts row_consts(const uint4& h, uint32_t c, uint32_t sel) {
  RowConsts r;
  const ScaleMin4 sm = unpack_scale_min(h.y, h.z, h.w);
  const uint32_t scw = c < 2 ? sm.sc_lo : sm.sc_hi;
  const uint32_t mw = c < 2 ? sm.m_lo : sm.m_hi;
  const uint32_t kMagic = 0x64006400u;  // f16x2 (1024, 1024)
  const uint32_t sc = hsub2(prmt(scw, 0u, sel) | kMagic, kMagic);  // (sc_j0, sc_j1) f16x2, exact
  const uint32_t mm = hsub2(prmt(mw, 0u, sel) | kMagic, kMagic);   // (m_j0, m_j1)
  r.sc0 = prmt(sc, sc, 0x1010u);
  r.nsc0 = hmul2(r.sc0, 0xE400E400u);                     // * (-1024)
  const uint32_t s1 = prmt(sc, sc, 0x3232u);
  r.sc1 = hmul2(s1, 0x2C002C00u);                         // * (1/16)
  r.nsc1 = hmul2(s1, 0xD400D400u);                        // * (-64)
  const uint16_t ndmin = (uint16_t)((h.x >> 16) ^ 0x8000u);  // -dmin
  r.ndm0 = fma_h_h_f(ndmin, (uint16_t)(mm & 0xffffu), 0.0f);
  r.ndm1 = fma_h_h_f(ndmin, (uint16_t)(mm >> 16), 0.0f);
  r.d = (uint16_t)(h.x & 0xffffu);
  return r;
}

// One 32-bit word of nibbles (bytes b0..b3 of one row) -> four f16x2 weight
// pairs: lo02 = (w[b0 lo], w[b2 lo]), lo13 = (w[b1 lo], w[b3 lo]), and the
// same for the high nibbles.  Low nibbles belong to sub-block j0, high to j1.
struct WordPairs {
  uint32_t lo02, lo13, hi02, hi13;
};

__device__ __forceinline__ WordPairs dequant_word(uint32_t v, const RowConsts& r) {
  const uint32_t kMagic = 0x64006400u;
  const uint32_t v8 = v >> 8;
  const uint32_t p_lo02 = hfma2((v & 0x000F000Fu) | kMagic, r.sc0, r.nsc0);   // sc*q, exact
  const uint32_t p_lo13 = hfma2((v8 & 0x000F000Fu) | kMagic, r.sc0, r.nsc0);
  const uint32_t p_hi02 = hfma2((v & 0x00F000F0u) | kMagic, r.sc1, r.nsc1);
  const uint32_t p_hi13 = hfma2((v8 & 0x00F000F0u) | kMagic, r.sc1, r.nsc1);
  WordPairs o;
  o.lo02 = cvt_f16x2(fma_h_h_f(r.d, (uint16_t)(p_lo02 >> 16), r.ndm0),
                     fma_h_h_f(r.d, (uint16_t)(p_lo02 & 0xffffu), r.ndm0));
  o.lo13 = cvt_f16x2(fma_h_h_f(r.d, (uint16_t)(p_lo13 >> 16), r.ndm0),
                     fma_h_h_f(r.d, (uint16_t)(p_lo13 & 0xffffu), r.ndm0));
  o.hi02 = cvt_f16x2(fma_h_h_f(r.d, (uint16_t)(p_hi02 >> 16), r.ndm1),
                     fma_h_h_f(r.d, (uint16_t)(p_hi02 & 0xffffu), r.ndm1));
  o.hi13 = cvt_f16x2(fma_h_h_f(r.d, (uint16_t)(p_hi13 >> 16), r.ndm1),
                     fma_h_h_f(r.d, (uint16_t)(p_hi13 & 0xffffu), r.ndm1));
  return o;
}

// The 96 bytes one lane reads per super-block: both rows' headers and qs groups.
struct BlockRegs {
  uint4 ha, hb, qa0, qa1, qb0, qb1;
};

__device__ __forceinline__ BlockRegs load_block(const uint8_t* pa, const uint8_t* pb, uint32_t c) {
  BlockRegs r;
  r.ha = ldg_v4(pa);
  r.hb = ldg_v4(pb);
  r.qa0 = ldg_v4(pa + 16 + 32 * c);
  r.qa1 = ldg_v4(pa + 32 + 32 * c);
  r.qb0 = ldg_v4(pb + 16 + 32 * c);
  r.qb1 = ldg_v4(pb + 32 + 32 * c);
  return r;
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

__device__ __forceinline__ EngineTask task_at(const TaskList& tl, uint32_t i) {
  return tl.dev ? tl.dev[i] : tl.inl;
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

// ---- TMA bulk copies and mbarriers ---------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after kSpinLimit polls (each poll may itself block
// for a short hardware-defined time), so a lost completion cannot hang the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// 1-D bulk copy global -> shared through the TMA unit, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_u32(p)));
  return r;
}

// ---- the engine kernel ----------------------------------------------------------

constexpr int kStages = 4;                                // blocks in flight per warp
constexpr uint32_t kStageBytes = kTileRows * kBlockBytes;  // 16 rows x one super-block
constexpr size_t kWarpSmem = kStages * (size_t)kStageBytes;

// Where a warp's copy engine stands: work item, super-block and its task.
struct Cursor {
  uint32_t item, b, ti;
  const uint8_t* w;
  uint32_t M, nb, item_begin, item_end;
};

__device__ __forceinline__ void cursor_task(Cursor& cu, const TaskList& tl) {
  const EngineTask T = task_at(tl, cu.ti);
  cu.w = T.w;
  cu.M = T.M;
  cu.nb = T.N >> 8;
  cu.item_begin = T.item_begin;
  cu.item_end = T.item_end;
}

__device__ __forceinline__ void cursor_seek(Cursor& cu, const TaskList& tl) {
  while (cu.item < tl.total_items && cu.item >= cu.item_end) {
    ++cu.ti;
    cursor_task(cu, tl);
  }
}

__device__ __forceinline__ void cursor_next(Cursor& cu, const TaskList& tl, uint32_t stride) {
  if (++cu.b == cu.nb) {
    cu.b = 0;
    cu.item += stride;
    cursor_seek(cu, tl);
  }
}

// Lanes 0..15 copy row (tile row = lane) of the cursor's super-block into the
// stage; lane 0 first arms the stage's barrier with the byte count.
__device__ __forceinline__ void issue_stage(const Cursor& cu, uint8_t* stage, uint64_t* bar, uint32_t lane) {
  if (lane == 0) mbar_arrive_expect_tx(bar, kStageBytes);
  __syncwarp();
  if (lane < (uint32_t)kTileRows) {
    uint32_t row = (cu.item - cu.item_begin) * kTileRows + lane;
    if (row >= cu.M) row = 0;  // past the last row: copy row 0, result discarded
    const uint8_t* src = cu.w + (uint64_t)row * cu.nb * kBlockBytes + (uint64_t)cu.b * kBlockBytes;
    bulk_g2s(stage + lane * kBlockBytes, src, kBlockBytes, bar);
  }
}

template <int NT>
__global__ void __launch_bounds__(kEngineWarps * 32, 2)
    engine_kernel(const TaskList tl, uint32_t batch, int has_select, SelectScratch sel) {
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  __shared__ uint64_t s_bar[kEngineWarps][kStages];
  __shared__ float s_bv[kEngineWarps][256];
  __shared__ uint32_t s_bi[kEngineWarps][256];

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t g = lane >> 2, c = lane & 3u;
  // bytes (2(c&1), 2(c&1)+1) of a packed scale word -> bytes 0 and 2
  const uint32_t bsel = (c & 1u) ? ((4u << 12) | (3u << 8) | (4u << 4) | 2u) : ((4u << 12) | (1u << 8) | (4u << 4) | 0u);
  uint8_t* wsm = smem_dyn + warp * kWarpSmem;
  uint64_t* bars = s_bar[warp];

  if (lane == 0)
    for (int st = 0; st < kStages; ++st) mbar_init(&bars[st], 1);
  if (has_select)
    for (uint32_t r = lane; r < 256; r += 32) {
      s_bv[warp][r] = kFloorE;
      s_bi[warp][r] = 0u;
    }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncwarp();

  const uint32_t total_warps = gridDim.x * kEngineWarps;
  const uint32_t first = blockIdx.x * kEngineWarps + warp;

  // copy cursor runs kStages super-blocks ahead of the math
  Cursor F;
  F.item = first;
  F.b = 0;
  F.ti = 0;
  cursor_task(F, tl);
  cursor_seek(F, tl);
  uint32_t issued = 0;
  for (int st = 0; st < kStages && F.item < tl.total_items; ++st) {
    issue_stage(F, wsm + st * kStageBytes, &bars[st], lane);
    cursor_next(F, tl, total_warps);
    ++issued;
  }

  uint32_t ti = 0;
  EngineTask T = task_at(tl, 0);
  uint32_t item = first;
  while (item < tl.total_items && item >= T.item_end) T = task_at(tl, ++ti);
  uint32_t b = 0, k = 0;
  bool timed_out = false;

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;

  while (item < tl.total_items) {
    const uint32_t slot = k % kStages;
    if (!mbar_wait(&bars[slot], (k / kStages) & 1u)) {
      timed_out = true;
      break;
    }
    const uint8_t* stg = wsm + slot * kStageBytes;
    const uint4 ha = lds128(stg + g * kBlockBytes);
    const uint4 hb = lds128(stg + (g + 8) * kBlockBytes);
    const uint4 qa0 = lds128(stg + g * kBlockBytes + 16 + 32 * c);
    const uint4 qa1 = lds128(stg + g * kBlockBytes + 32 + 32 * c);
    const uint4 qb0 = lds128(stg + (g + 8) * kBlockBytes + 16 + 32 * c);
    const uint4 qb1 = lds128(stg + (g + 8) * kBlockBytes + 32 + 32 * c);
    // the stage is in registers: hand it back to the copy engine
    fence_proxy_async_smem();
    __syncwarp();
    if (F.item < tl.total_items) {
      issue_stage(F, wsm + slot * kStageBytes, &bars[slot], lane);
      cursor_next(F, tl, total_warps);
      ++issued;
    }

    const uint32_t nb = T.N >> 8;
    const RowConsts ka = row_consts(ha, c, bsel);
    const RowConsts kb = row_consts(hb, c, bsel);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const WordPairs A = dequant_word(word_of(qa0, qa1, w), ka);
      const WordPairs B = dequant_word(word_of(qb0, qb1, w), kb);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        // only the 2 columns per token of the tile hold data; other lanes use 0
        const uint32_t cols = 2u * min(4u, batch - 4u * n);
        uint2 blo = make_uint2(0u, 0u), bhi = make_uint2(0u, 0u);
        if (g < cols) {
          const uint2* f = T.xfrag + ((size_t)(n * nb + b) * 16) * 32 + lane;
          blo = ldg_v2(f + w * 32);
          bhi = ldg_v2(f + (8 + w) * 32);
        }
        mma_16816(acc[n], A.lo02, B.lo02, A.lo13, B.lo13, blo);
        mma_16816(acc[n], A.hi02, B.hi02, A.hi13, B.hi13, bhi);
      }
    }
    ++k;
    if (++b < nb) continue;

    // item done: acc[n][0..1] = (hi, lo) parts of token 4n+c for row ra, [2..3] for rb
    const uint32_t ra = (item - T.item_begin) * kTileRows + g, rb = ra + 8;
    const bool va = ra < T.M, vb = rb < T.M;
    if (T.kind == kTaskPlain) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t t = 4 * n + c;
        if (t < batch) {
          const float inv = T.inv_scale[t];
          if (va) T.y[(uint64_t)t * T.M + ra] = (acc[n][0] + acc[n][1]) * inv;
          if (vb) T.y[(uint64_t)t * T.M + rb] = (acc[n][2] + acc[n][3]) * inv;
        }
      }
    } else {
      if (c == 0) {
        const float inv = T.inv_scale[0];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!(h ? vb : va)) continue;
          const uint32_t row = h ? rb : ra;
          float v = (h ? (acc[0][2] + acc[0][3]) : (acc[0][0] + acc[0][1])) * inv;
          if (T.cap > 0.0f) v = softcap(v, T.cap);
          if (T.logits) T.logits[row] = v;
          const uint32_t gi = T.row_offset + row;
          const uint32_t res = gi & 255u;
          if (better(v, gi, s_bv[warp][res], s_bi[warp][res])) {
            s_bv[warp][res] = v;
            s_bi[warp][res] = gi;
          }
        }
      }
      __syncwarp();
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    b = 0;
    item += total_warps;
    while (item < tl.total_items && item >= T.item_end) T = task_at(tl, ++ti);
  }

  if (timed_out) {
    // record the failure, then let every copy still in flight land (bounded)
    if (lane == 0) atomicOr(sel.status, 1u);
    for (uint32_t j = k; j < issued; ++j) mbar_wait(&bars[j % kStages], (j / kStages) & 1u);
  }

  if (!has_select) return;
  // Publish this warp's per-residue candidates; the last warp of the grid
  // turns the keys into the 256 candidates + argmax and resets the scratch.
  __syncwarp();
  for (uint32_t r = lane; r < 256; r += 32) {
    const float v = s_bv[warp][r];
    const uint32_t i = s_bi[warp][r];
    if (!(v == kFloorE && i == 0u)) atomicMax(&sel.slots[r], sel_key(v, i));
  }
  __threadfence();
  __syncwarp();
  uint32_t last = 0;
  if (lane == 0) last = (atomicAdd(sel.counter, 1u) == total_warps - 1) ? 1u : 0u;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  EngineTask S = task_at(tl, 0);
  for (uint32_t i = 0; i < tl.n; ++i) {
    S = task_at(tl, i);
    if (S.kind == kTaskSelect) break;
  }
  float* fv = s_bv[warp];
  uint32_t* fi = s_bi[warp];
  for (uint32_t r = lane; r < 256; r += 32) {
    const unsigned long long key = atomicExch(&sel.slots[r], sel_key(kFloorE, 0u));
    float v;
    uint32_t i;
    sel_unkey(key, v, i);
    S.cand_val[r] = v;
    S.cand_idx[r] = i;
    fv[r] = v;
    fi[r] = i;
  }
  __syncwarp();
  // the reference's argmax tree (shaders/argmax.wgsl:21-27), one warp
  for (uint32_t stride = 128; stride > 0; stride >>= 1) {
    for (uint32_t t = lane; t < stride; t += 32) {
      if (fv[t + stride] > fv[t]) {
        fv[t] = fv[t + stride];
        fi[t] = fi[t + stride];
      }
    }
    __syncwarp();
  }
  if (lane == 0) {
    *S.argmax = fi[0];
    *sel.counter = 0u;
  }
}

// ---- activation preparation --------------------------------------------------------

__device__ __forceinline__ float xjob_value(const XJob& J, uint64_t i) {
  return J.mode ? gelu_mul_value(J.gate[i], J.up[i]) : J.x[i];
}

// One CTA per (job, token): max|x| -> power-of-two scale -> hi/lo f16 split in
// B-fragment order (columns 2t%8, 2t%8+1 of n-tile t/4; the engine never reads
// the columns of tokens >= batch).
__global__ void __launch_bounds__(256) xprep_kernel(const JobList jl, uint32_t batch) {
  __shared__ float s_red[8];
  const uint32_t job = blockIdx.x / batch, t = blockIdx.x % batch;
  const XJob J = jl.dev ? jl.dev[job] : jl.inl;
  const uint32_t N = J.N, nb = N >> 8;
  const uint64_t base = (uint64_t)t * N;

  float mx = 0.0f;
  for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) {
    const float v = xjob_value(J, base + k);
    if (J.mode && J.act) J.act[base + k] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  int e = 0;
  int sexp = 0;
  if (mx > 0.0f && mx <= 3.402823466e38f) {
    frexpf(mx, &e);  // mx < 2^e
    sexp = 15 - e;
    sexp = sexp > 100 ? 100 : (sexp < -100 ? -100 : sexp);
  }
  const float s = ldexpf(1.0f, sexp);
  if (threadIdx.x == 0) J.inv_scale[t] = ldexpf(1.0f, -sexp);

  const uint32_t nt = t >> 2, col_hi = 2 * (t & 3u), col_lo = col_hi + 1;
  for (uint32_t idx = threadIdx.x; idx < nb * 64; idx += blockDim.x) {
    const uint32_t b = idx >> 6, i = (idx >> 2) & 15u, c = idx & 3u;
    const uint32_t off = i < 8 ? 4 * i : 32 + 4 * (i - 8);
    const uint64_t k0 = base + 256u * b + 64u * c + off;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = xjob_value(J, k0 + j) * s;
    __half hh[4], hl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hh[j] = __float2half_rn(v[j]);
      hl[j] = __float2half_rn(v[j] - __half2float(hh[j]));
    }
    uint2* dst = J.xfrag + ((size_t)(nt * nb + b) * 16 + i) * 32;
    // (b0, b1) = (x[k0], x[k0+2]), (b2, b3) = (x[k0+1], x[k0+3])
    dst[4 * col_hi + c] = make_uint2(__half_as_ushort(hh[0]) | ((uint32_t)__half_as_ushort(hh[2]) << 16),
                                     __half_as_ushort(hh[1]) | ((uint32_t)__half_as_ushort(hh[3]) << 16));
    dst[4 * col_lo + c] = make_uint2(__half_as_ushort(hl[0]) | ((uint32_t)__half_as_ushort(hl[2]) << 16),
                                     __half_as_ushort(hl[1]) | ((uint32_t)__half_as_ushort(hl[3]) << 16));
  }
}

__global__ void init_select_kernel(SelectScratch sc) {
  sc.slots[threadIdx.x] = sel_key(kFloorE, 0u);
  if (threadIdx.x == 0) {
    *sc.counter = 0u;
    *sc.status = 0u;
  }
}

}  // namespace

cudaError_t init_select_scratch(const SelectScratch& sc, cudaStream_t s) {
  init_select_kernel<<<1, 256, 0, s>>>(sc);
  return cudaGetLastError();
}

cudaError_t launch_xprep(const JobList& jobs, uint32_t batch, cudaStream_t s) {
  xprep_kernel<<<jobs.n * batch, 256, 0, s>>>(jobs, batch);
  return cudaGetLastError();
}

cudaError_t launch_engine(const TaskList& tasks, uint32_t batch, bool has_select, const SelectScratch& sel,
                          int sm_count, cudaStream_t s) {
  const uint32_t items = tasks.total_items;
  uint32_t grid = (items + kEngineWarps - 1) / kEngineWarps;
  const uint32_t cap = (uint32_t)sm_count * 2u;
  if (grid > cap) grid = cap;
  if (grid == 0) grid = 1;
  const int nt = (int)((batch + 3) / 4);
  const int hs = has_select ? 1 : 0;
  const size_t smem = kEngineWarps * kWarpSmem;
  static bool attr_done[4] = {false, false, false, false};
  cudaError_t e = cudaSuccess;
  switch (nt) {
    case 1:
      if (!attr_done[0]) e = cudaFuncSetAttribute(engine_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr_done[0] = e == cudaSuccess;
      if (e == cudaSuccess) engine_kernel<1><<<grid, kEngineWarps * 32, smem, s>>>(tasks, batch, hs, sel);
      break;
    case 2:
      if (!attr_done[1]) e = cudaFuncSetAttribute(engine_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr_done[1] = e == cudaSuccess;
      if (e == cudaSuccess) engine_kernel<2><<<grid, kEngineWarps * 32, smem, s>>>(tasks, batch, hs, sel);
      break;
    case 3:
      if (!attr_done[2]) e = cudaFuncSetAttribute(engine_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr_done[2] = e == cudaSuccess;
      if (e == cudaSuccess) engine_kernel<3><<<grid, kEngineWarps * 32, smem, s>>>(tasks, batch, hs, sel);
      break;
    default:
      if (!attr_done[3]) e = cudaFuncSetAttribute(engine_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr_done[3] = e == cudaSuccess;
      if (e == cudaSuccess) engine_kernel<4><<<grid, kEngineWarps * 32, smem, s>>>(tasks, batch, hs, sel);
      break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace q4k
