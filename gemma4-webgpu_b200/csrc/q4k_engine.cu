// Q4_K GEMV engine for sm_100a.
//
// y[t, m] = sum_k f32(w16[m, k]) * x[t, k], w16 = f16_rne(f32(d*sc*q - dmin*m))
// (the weight the reference GPU multiplies: src/gguf.ts:168-210 + 425-473,
// shaders/matmul_quant.wgsl:35), for t < batch <= 16.
//
// Work decomposition: one 16-warp CTA per SM walks a contiguous range of a
// shared work list; an item is a 16-row tile of one GEMV task (the tasks of a
// launch are a single call, or every GEMV of a plan stage).  The warps of a
// CTA take the range's items in turn, so a CTA touches few tasks and keeps
// their prepared activations in shared memory.  Each warp streams its tiles'
// 144-byte super-blocks HBM -> shared memory with the TMA bulk-copy engine,
// two super-blocks per stage, two stages in flight per warp.
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

#include "q4k_dequant.cuh"
#include "q4k_device.cuh"
#include "q4k_engine.cuh"
#include "q4k_engine_math.cuh"
#include "q4k_ptx.cuh"
#include "q6k_dequant.cuh"

namespace q4k {
namespace {

constexpr float kFloorE = -1e30f;

// ---- small PTX helpers -------------------------------------------------------

__device__ __forceinline__ EngineTask task_at(const TaskList& tl, uint32_t i) {
  return tl.dev ? tl.dev[i] : tl.inl;
}

// ---- programmatic dependent launch ----------------------------------------------------
// Engine launches are made with programmatic stream serialization: a launch
// may start while the previous kernel on the stream finishes, runs its
// prologue on static data only (schedule, task descriptors, the first weight
// stages), and waits for the previous kernel's completion and memory before
// it reads activations or writes outputs.  Each CTA signals its dependents
// once its work loop is done.

__device__ __forceinline__ void wait_prior_grids() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- activation preparation --------------------------------------------------------

__device__ __forceinline__ float xjob_value(const XJob& J, uint64_t i) {
  return J.mode ? gelu_mul_value(J.gate[i], J.up[i]) : J.x[i];
}

// Max |value| of token t of job J over a block of NW warps (stores the
// gelu_mul output on the way when `store_act`); every thread gets the max.
template <int NW>
__device__ float job_token_max(const XJob& J, uint32_t t, bool store_act, float* s_red) {
  const uint64_t base = (uint64_t)t * J.N;
  float mx = 0.0f;
  for (uint32_t k = threadIdx.x; k < J.N; k += NW * 32) {
    const float v = xjob_value(J, base + k);
    if (store_act) J.act[base + k] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) mx = fmaxf(mx, s_red[i]);
  __syncthreads();
  return mx;
}

// Token t of job J, scaled by s and split into f16 hi/lo, into the job's
// fragment array `frags` (global or shared memory; layout of
// q4k_engine.cuh), by a block of NW warps.
template <int NW>
__device__ void job_token_frags(const XJob& J, uint32_t t, uint32_t batch, float s, uint4* frags) {
  const uint32_t nb = J.N >> 8;
  const uint64_t base = (uint64_t)t * J.N;
  const uint32_t nt = t >> 2, cols = 2u * min(4u, batch - 4u * nt);
  const uint32_t col_hi = 2 * (t & 3u), col_lo = col_hi + 1;
  uint4* tile = frags + (size_t)nt * nb * 256u;
  for (uint32_t idx = threadIdx.x; idx < nb * 32; idx += NW * 32) {
    const uint32_t b = idx >> 5, w = (idx >> 2) & 7u, c = idx & 3u;
    // k-step w (low nibbles) starts at k0, k-step w+8 (high nibbles) at k0+32
    const uint64_t k0 = base + 256u * b + 64u * c + 4u * w;
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = xjob_value(J, k0 + j) * s;
      v[4 + j] = xjob_value(J, k0 + 32 + j) * s;
    }
    uint16_t hh[8], hl[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half h = __float2half_rn(v[j]);
      hh[j] = __half_as_ushort(h);
      hl[j] = __half_as_ushort(__float2half_rn(v[j] - __half2float(h)));
    }
    uint4* dst = tile + (size_t)(b * 8 + w) * cols * 4;
    // per k-step: (b0, b1) = (x[k], x[k+2]), (b2, b3) = (x[k+1], x[k+3])
    dst[4 * col_hi + c] = make_uint4(hh[0] | ((uint32_t)hh[2] << 16), hh[1] | ((uint32_t)hh[3] << 16),
                                     hh[4] | ((uint32_t)hh[6] << 16), hh[5] | ((uint32_t)hh[7] << 16));
    dst[4 * col_lo + c] = make_uint4(hl[0] | ((uint32_t)hl[2] << 16), hl[1] | ((uint32_t)hl[3] << 16),
                                     hl[4] | ((uint32_t)hl[6] << 16), hl[5] | ((uint32_t)hl[7] << 16));
  }
}

// Token t of job J in one pass when its 8-element groups fit kPrepGroups
// per thread: each thread evaluates its groups once (x, or gelu_mul of gate
// and up, stored to J.act when `store_act`), keeps them in registers for the
// block-wide max, then writes their scaled hi/lo fragments.  Returns 1/s.
// Falls back to two passes (values evaluated twice) for longer rows.
constexpr uint32_t kPrepGroups = 4;

template <int NW>
__device__ float job_token_prep(const XJob& J, uint32_t t, uint32_t batch, bool store_act, uint4* frags,
                                float* s_red) {
  const uint32_t nb = J.N >> 8, groups = nb * 32;
  if (groups > kPrepGroups * NW * 32) {
    const float2 sc = token_scale(job_token_max<NW>(J, t, store_act, s_red));
    job_token_frags<NW>(J, t, batch, sc.x, frags);
    return sc.y;
  }
  const uint64_t base = (uint64_t)t * J.N;
  float v[kPrepGroups][8];
  float mx = 0.0f;
#pragma unroll
  for (uint32_t i = 0; i < kPrepGroups; ++i) {
    const uint32_t idx = threadIdx.x + i * NW * 32;
    if (idx < groups) {
      const uint32_t b = idx >> 5, w = (idx >> 2) & 7u, c = idx & 3u;
      const uint64_t k0 = base + 256u * b + 64u * c + 4u * w;  // elements k0..k0+3 and k0+32..k0+35
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint64_t k = k0 + 32u * h;
        float4 q;
        if (J.mode) {
          const float4 g = *reinterpret_cast<const float4*>(J.gate + k);
          const float4 u = *reinterpret_cast<const float4*>(J.up + k);
          q = make_float4(gelu_mul_value(g.x, u.x), gelu_mul_value(g.y, u.y), gelu_mul_value(g.z, u.z),
                          gelu_mul_value(g.w, u.w));
          if (store_act) *reinterpret_cast<float4*>(J.act + k) = q;
        } else {
          q = *reinterpret_cast<const float4*>(J.x + k);
        }
        v[i][4 * h + 0] = q.x;
        v[i][4 * h + 1] = q.y;
        v[i][4 * h + 2] = q.z;
        v[i][4 * h + 3] = q.w;
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) mx = fmaxf(mx, s_red[i]);
  __syncthreads();
  const float2 sc = token_scale(mx);
  const uint32_t nt = t >> 2, cols = 2u * min(4u, batch - 4u * nt);
  const uint32_t col_hi = 2 * (t & 3u), col_lo = col_hi + 1;
  uint4* tile = frags + (size_t)nt * nb * 256u;
#pragma unroll
  for (uint32_t i = 0; i < kPrepGroups; ++i) {
    const uint32_t idx = threadIdx.x + i * NW * 32;
    if (idx < groups) {
      const uint32_t b = idx >> 5, w = (idx >> 2) & 7u, c = idx & 3u;
      uint16_t hh[8], hl[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float x = v[i][j] * sc.x;
        const __half h = __float2half_rn(x);
        hh[j] = __half_as_ushort(h);
        hl[j] = __half_as_ushort(__float2half_rn(x - __half2float(h)));
      }
      uint4* dst = tile + (size_t)(b * 8 + w) * cols * 4;
      // per k-step: (b0, b1) = (x[k], x[k+2]), (b2, b3) = (x[k+1], x[k+3])
      dst[4 * col_hi + c] = make_uint4(hh[0] | ((uint32_t)hh[2] << 16), hh[1] | ((uint32_t)hh[3] << 16),
                                       hh[4] | ((uint32_t)hh[6] << 16), hh[5] | ((uint32_t)hh[7] << 16));
      dst[4 * col_lo + c] = make_uint4(hl[0] | ((uint32_t)hl[2] << 16), hl[1] | ((uint32_t)hl[3] << 16),
                                       hl[4] | ((uint32_t)hl[6] << 16), hl[5] | ((uint32_t)hl[7] << 16));
    }
  }
  return sc.y;
}

// One CTA per (job, token) for launches that do not prepare in the engine:
// max|x| -> power-of-two scale -> hi/lo f16 split into the job's global
// fragment array.
__global__ void __launch_bounds__(256) xprep_kernel(const JobList jl, uint32_t batch) {
  __shared__ float s_red[8];
  const uint32_t job = blockIdx.x / batch, t = blockIdx.x % batch;
  const XJob J = jl.dev ? jl.dev[job] : jl.inl;
  const float inv = job_token_prep<8>(J, t, batch, J.mode && J.act, reinterpret_cast<uint4*>(J.xfrag), s_red);
  if (threadIdx.x == 0) J.inv_scale[t] = inv;
}

// ---- the engine kernel ----------------------------------------------------------

// Per-warp weight pipeline of each format.
//
// Q4_K: a stage holds one weight-map box: 16 tile rows of 2 super-blocks
// plus 16 bytes (the box width; 144 bytes for one-block rows), so the 8 rows
// a quarter-warp reads land in distinct banks; 2 stages in flight.
// Q6_K: a stage holds one 208-byte body of each of the 16 rows (rows 52
// words apart: conflict-free) and the rows' 16 f16 d values behind them; 3
// stages in flight (about the same bytes as Q4_K's 2 x 2 super-blocks).
constexpr uint32_t kBoxWords2 = 2 * kBlockBytes / 4 + 4;  // 76 words = 304 bytes
constexpr uint32_t kBoxWords1 = kBlockBytes / 4;          // 36 words = 144 bytes

template <int FMT>
struct Pipe;
template <>
struct Pipe<kFmtQ4K> {
  static constexpr int kStages = 2;
  static constexpr uint32_t kBlocks = 2;  // super-blocks per stage (per tile row)
  static constexpr uint32_t kStageBytes = kTileRows * kBoxWords2 * 4;
};
template <>
struct Pipe<kFmtQ6K> {
  static constexpr int kStages = 3;
  static constexpr uint32_t kBlocks = 1;
  static constexpr uint32_t kDOff = kTileRows * kQ6BodyBytes;  // 3328: the d values (128-byte aligned)
  static constexpr uint32_t kTxBytes = kDOff + kTileRows * 2;   // bytes the two copies deliver
  static constexpr uint32_t kStageBytes = (kTxBytes + 127u) & ~127u;  // stages stay 128-byte aligned
};
constexpr int kMaxStages = 3;

template <int FMT>
constexpr size_t weight_smem() {
  return (size_t)kEngineWarps * Pipe<FMT>::kStages * Pipe<FMT>::kStageBytes;
}
constexpr size_t kSelectSmem = (size_t)kEngineWarps * 256 * 8;
constexpr size_t kTaskSmem = (size_t)kMaxCtaTasks * sizeof(EngineTask);
constexpr size_t kSmemLimit = 227 * 1024;
constexpr size_t kStaticSmemHeadroom = 4096;

// Where a CTA reads task descriptors: its shared-memory copy of tasks
// [t0, t0+nt), the global table, or (table = null) the inline task.
struct TaskSrc {
  const EngineTask* table;
  uint32_t t0;
  const CUtensorMap* pmap;   // the launch's own weight map (inline task)
  const CUtensorMap* pdmap;  // and its Q6_K d-plane map
};

__device__ __forceinline__ EngineTask task_get(const TaskList& tl, const TaskSrc& ts, uint32_t i) {
  return ts.table ? ts.table[i - ts.t0] : tl.inl;
}

// Where a warp's copy engine stands: work item, super-block and its task.
struct Cursor {
  uint32_t item, b, b_hi, ti;
  uint32_t claims, issued;  // items claimed, stages issued
  const CUtensorMap* map;
  const CUtensorMap* dmap;  // Q6_K: the d-plane map
  uint32_t tile_bytes, nb, item_begin, item_end;
};

// The item's super-block range for this warp: all of the row, or quarter q
// of it when the launch splits each tile's K range over KS warps.
__device__ __forceinline__ void cursor_range(Cursor& cu, uint32_t q, uint32_t ks) {
  const uint32_t part = cu.nb / ks;
  cu.b = q * part;
  cu.b_hi = cu.b + part;
}

__device__ __forceinline__ void cursor_task(Cursor& cu, const TaskList& tl, const TaskSrc& ts) {
  const EngineTask T = task_get(tl, ts, cu.ti);
  cu.map = T.tmap ? T.tmap : ts.pmap;
  cu.dmap = T.tmap ? T.tmap + 1 : ts.pdmap;
  cu.tile_bytes = T.tile_bytes;
  cu.nb = T.N >> 8;
  cu.item_begin = T.item_begin;
  cu.item_end = T.item_end;
}

__device__ __forceinline__ void cursor_seek(Cursor& cu, const TaskList& tl, const TaskSrc& ts, uint32_t end) {
  while (cu.item < end && cu.item >= cu.item_end) {
    ++cu.ti;
    cursor_task(cu, tl, ts);
  }
}

// Super-blocks of the cursor's stage: up to the format's per-stage count,
// not past the range.
template <int FMT>
__device__ __forceinline__ uint32_t cursor_blocks(const Cursor& cu) {
  return min(Pipe<FMT>::kBlocks, cu.b_hi - cu.b);
}

// Lane 0 copies the stage's tile data and arms the stage's barrier with its
// size.  Q4_K: super-blocks b, b+1 of the tile's 16 rows (one map box, rows
// tile_bytes apart).  Q6_K: body b of the 16 rows (one box) and their 16 d
// values (one box of the d plane).  Rows past M and words past the row end
// arrive as zeros.
template <int FMT>
__device__ __forceinline__ void issue_stage(const Cursor& cu, uint8_t* stage, uint64_t* bar, uint32_t lane) {
  if (lane == 0) {
    const uint32_t row0 = (cu.item - cu.item_begin) * kTileRows;
    if constexpr (FMT == kFmtQ6K) {
      mbar_arrive_expect_tx(bar, Pipe<kFmtQ6K>::kTxBytes);
      tma_tile_g2s(stage, cu.map, cu.b * kQ6BodyWords, row0, bar);
      tma_tile_g2s(stage + Pipe<kFmtQ6K>::kDOff, cu.dmap, row0, cu.b, bar);
    } else {
      mbar_arrive_expect_tx(bar, kTileRows * cu.tile_bytes);
      tma_tile_g2s(stage, cu.map, cu.b * (kBlockBytes / 4), row0, bar);
    }
  }
}


// One Q6_K super-block of the lane's two rows in a stage: the rows' bodies,
// the lane's scale words and the rows' d values (the ql / qh words are read
// per 16-column half inside the math, so they never all sit in registers).
struct Q6Rows {
  const uint8_t* ra;
  const uint8_t* rb;
  uint32_t sa, sb;
  uint16_t da, db;
};

__device__ __forceinline__ Q6Rows q6_rows(const uint8_t* stg, uint32_t g, uint32_t c) {
  Q6Rows r;
  r.ra = stg + g * kQ6BodyBytes;
  r.rb = stg + (g + 8) * kQ6BodyBytes;
  r.sa = *reinterpret_cast<const uint32_t*>(r.ra + 192 + 4 * c);
  r.sb = *reinterpret_cast<const uint32_t*>(r.rb + 192 + 4 * c);
  const uint16_t* dv = reinterpret_cast<const uint16_t*>(stg + kTileRows * kQ6BodyBytes);
  r.da = dv[g];
  r.db = dv[g + 8];
  return r;
}

__device__ __forceinline__ uint32_t u4_word(const uint4& a, int w) {
  return w == 0 ? a.x : (w == 1 ? a.y : (w == 2 ? a.z : a.w));
}

// The math of one Q6_K super-block: 2 rows x 64 weights per lane, words in
// the Q4_K order (word w = 4*is + j of the lane's half), same B fragments.
template <int NT, int COLS, bool SX, bool EXACT>
__device__ __forceinline__ void q6_block_math(float (&acc)[NT][2][4], const Q6Rows& R, uint32_t c,
                                              const uint8_t* const (&base)[NT], const uint32_t (&wstep)[NT]) {
  const uint32_t sh = (c & 1u) * 4u, h = c >> 1;
  const float d4a = 4.0f * __half2float(__ushort_as_half(R.da));
  const float d4b = 4.0f * __half2float(__ushort_as_half(R.db));
#pragma unroll
  for (int is = 0; is < 2; ++is) {
    const uint4 la0 = sld128(R.ra + 64 * h + 16 * is), la1 = sld128(R.ra + 64 * h + 32 + 16 * is);
    const uint4 ha = sld128(R.ra + 128 + 32 * h + 16 * is);
    const uint4 lb0 = sld128(R.rb + 64 * h + 16 * is), lb1 = sld128(R.rb + 64 * h + 32 + 16 * is);
    const uint4 hb = sld128(R.rb + 128 + 32 * h + 16 * is);
    const Q6Consts ka = q6_consts(R.sa, is, d4a);
    const Q6Consts kb = q6_consts(R.sb, is, d4b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int w = 4 * is + j;
      const WordPairs A = dequant6_word<EXACT>(u4_word(la0, j), u4_word(la1, j), u4_word(ha, j), sh, ka);
      const WordPairs B = dequant6_word<EXACT>(u4_word(lb0, j), u4_word(lb1, j), u4_word(hb, j), sh, kb);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t ws = COLS > 0 ? (uint32_t)COLS * 64u : wstep[n];
        const uint4 f = load_frag<SX>(base[n] + w * ws);
        mma_16816(acc[n][0], A.lo02, B.lo02, A.lo13, B.lo13, make_uint2(f.x, f.y));
        mma_16816(acc[n][1], A.hi02, B.hi02, A.hi13, B.hi13, make_uint2(f.z, f.w));
      }
    }
  }
}

// The task fields the math loop keeps in registers.
template <int NT>
struct Hot {
  uint32_t M, nb, item_begin, item_end, kind, tile_bytes;
  const uint2* xfrag;
  float* y;
  uint32_t xs;      // shared-memory byte offset of the prepared activations, or ~0
  float inv[NT];    // 1/scale of this lane's token in each n-tile
};

template <int NT>
__device__ __forceinline__ Hot<NT> hot_of(const TaskList& tl, const TaskSrc& ts, uint32_t ti, const CtaSched& xc,
                                          uint32_t c, uint32_t batch, const float (*s_inv)[kMaxTokens]) {
  const EngineTask T = task_get(tl, ts, ti);
  Hot<NT> h;
  h.M = T.M;
  h.nb = T.N >> 8;
  h.item_begin = T.item_begin;
  h.item_end = T.item_end;
  h.kind = T.kind;
  h.tile_bytes = T.tile_bytes;
  h.xfrag = T.xfrag;
  h.y = T.y;
  h.xs = 0xffffffffu;
  uint32_t slot = 0;
  for (uint32_t j = 0; j < xc.nx; ++j)
    if (xc.xptr[j] == T.xfrag) {
      h.xs = xc.xoff[j];
      slot = j;
    }
#pragma unroll
  for (int n = 0; n < NT; ++n)
    h.inv[n] = tl.prep ? s_inv[slot][min(4u * n + c, batch - 1)] : T.inv_scale[min(4u * n + c, batch - 1)];
  return h;
}

// XS = 1: a launch that prepares its activations in the engine (tl.prep), so
// every task's activation sits in the CTA's shared-memory cache and the math
// loop has only the shared-memory path.
template <int NT, int COLS, int KS, int FMT, int XS, int PR>
__global__ void __launch_bounds__(kEngineWarps * 32, 1)
    engine_kernel(const TaskList tl, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap dmap, uint32_t batch, int has_select, SelectScratch sel,
                  uint32_t xcache_cap) {
  constexpr int kSt = Pipe<FMT>::kStages;
  constexpr uint32_t kSB = Pipe<FMT>::kStageBytes;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // tile copies land on 128-byte boundaries
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  __shared__ uint64_t s_bar[kEngineWarps][kMaxStages];
  __shared__ uint64_t s_xbar;
  __shared__ CtaSched s_sched;
  __shared__ uint32_t s_next;                    // next unclaimed item of this CTA's range
  __shared__ uint32_t s_ring[kEngineWarps][4];   // items claimed by each warp, in order
  __shared__ Cursor s_cur[kEngineWarps];          // each warp's copy cursor (lane 0's)
  __shared__ float s_inv[kMaxCachedX][kMaxTokens];  // prep: 1/scale of each cached activation and token
  __shared__ float s_red[kEngineWarps];
  __shared__ uint64_t s_gbar[kEngineWarps];          // K-split launches: one per tile group

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t g = lane >> 2, c = lane & 3u;
  const uint32_t spin = spin_or_default(sel.spin_limit);  // polls per bounded wait
  // bytes (2(c&1), 2(c&1)+1) of a packed scale word -> bytes 0 and 2
  const uint32_t bsel = scale_sel(c);
  uint8_t* wsm = smem + warp * (kSt * kSB);
  EngineTask* s_tasks = reinterpret_cast<EngineTask*>(smem + weight_smem<FMT>());
  uint8_t* xsm = smem + weight_smem<FMT>() + kTaskSmem;
  float* s_bv = reinterpret_cast<float*>(xsm + xcache_cap) + warp * 512;
  uint32_t* s_bi = reinterpret_cast<uint32_t*>(s_bv + 256);
  uint64_t* bars = s_bar[warp];
  uint32_t* ring = s_ring[warp];

  // launches that copy prepared activations from global memory read data a
  // previous kernel wrote: wait for it before anything else
  if (!tl.prep) wait_prior_grids();
  if (lane == 0)
    for (int st = 0; st < kSt; ++st) mbar_init(&bars[st], 1);
  if (threadIdx.x == 0) mbar_init(&s_xbar, 1);
  // K-split launches (tl.ksplit = KS > 1): the KS warps of a group take the
  // same tiles, each a 1/KS slice of the row's super-blocks, and add their
  // partial sums through shared memory; tiles go to groups in turn.
  constexpr uint32_t ks_n = KS;  // == tl.ksplit (1: no split)
  const uint32_t gq = warp % ks_n, grp = warp / ks_n, ngrp = kEngineWarps / ks_n;
  if (threadIdx.x == 0 && ks_n > 1)
    for (uint32_t i = 0; i < ngrp; ++i) mbar_init(&s_gbar[i], ks_n);
  if (has_select)
    for (uint32_t r = lane; r < 256; r += 32) {
      s_bv[r] = kFloorE;
      s_bi[r] = 0u;
    }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();

  // This CTA's share: from the host-made schedule (device task lists), or an
  // equal share of the single inline task's tiles.  Its task descriptors and
  // prepared activations are bulk-copied into shared memory.
  if (threadIdx.x == 0) {
    if (tl.sched) {
      s_sched = tl.sched[blockIdx.x];
    } else {
      const uint32_t per = (tl.total_items + gridDim.x - 1) / gridDim.x;
      s_sched.c0 = min(tl.total_items, blockIdx.x * per);
      s_sched.c1 = min(tl.total_items, s_sched.c0 + per);
      s_sched.t0 = 0;
      s_sched.nt = 0;
      const uint32_t xb = (uint32_t)xfrag_bytes(tl.inl.N, batch);
      s_sched.nx = (s_sched.c0 < s_sched.c1 && xb <= xcache_cap) ? 1u : 0u;
      s_sched.xoff[0] = 0;
      s_sched.xbytes[0] = xb;
      s_sched.xptr[0] = tl.inl.xfrag;
      s_sched.xjob[0] = 0;
      // an inline job's gelu_mul output is stored by CTA 0
      s_sched.act_mask = (blockIdx.x == 0) ? 1u : 0u;
    }
    s_next = s_sched.c0;
    uint32_t bytes = s_sched.nt * (uint32_t)sizeof(EngineTask);
    if (!tl.prep)
      for (uint32_t j = 0; j < s_sched.nx; ++j) bytes += s_sched.xbytes[j];
    mbar_arrive_expect_tx(&s_xbar, bytes);
    if (s_sched.nt) bulk_g2s(s_tasks, tl.dev + s_sched.t0, s_sched.nt * (uint32_t)sizeof(EngineTask), &s_xbar);
    if (!tl.prep)
      for (uint32_t j = 0; j < s_sched.nx; ++j)
        for (uint32_t o = 0; o < s_sched.xbytes[j]; o += 32768u)
          bulk_g2s(xsm + s_sched.xoff[j] + o, reinterpret_cast<const uint8_t*>(s_sched.xptr[j]) + o,
                   min(32768u, s_sched.xbytes[j] - o), &s_xbar);
  }
  __syncthreads();
  const uint32_t c0 = s_sched.c0, c1 = s_sched.c1;
  bool timed_out = false;
  if (!mbar_wait(&s_xbar, 0, spin)) timed_out = true;
  TaskSrc ts;
  ts.table = !tl.dev ? nullptr : (s_sched.nt ? s_tasks : tl.dev);
  ts.t0 = s_sched.nt ? s_sched.t0 : 0u;
  ts.pmap = &wmap;
  ts.pdmap = &dmap;
  const uint32_t t_first = s_sched.nt ? s_sched.t0 : 0u;

  // Items are claimed from the CTA's range by the copy cursor (a shared
  // counter, so warps that finish early take more) and recorded in the
  // warp's ring, which the math follows in the same order.
  // (K-split launches: a group's tiles are fixed, c0 + grp + ngrp*i.)
  // The copy cursor lives in shared memory and only lane 0 touches it (at
  // the start and when a stage is handed back), so it holds no registers
  // across the math.
  auto claim = [&](Cursor& F) -> uint32_t {  // lane 0
    const uint32_t it = ks_n > 1 ? c0 + grp + ngrp * F.claims : atomicAdd(&s_next, 1u);
    ring[F.claims & 3u] = it;
    ++F.claims;
    return it;
  };
  // Lane 0: issue the cursor's stage into `slot` and advance the cursor.
  auto issue_next = [&](Cursor& F, uint32_t slot) {
    issue_stage<FMT>(F, wsm + slot * kSB, &bars[slot], 0u);
    F.b += cursor_blocks<FMT>(F);
    if (F.b == F.b_hi) {
      F.item = claim(F);
      cursor_seek(F, tl, ts, c1);
      cursor_range(F, gq, ks_n);
    }
    ++F.issued;
  };

  // Prepare-in-engine launches: with the first weight stages in flight, the
  // whole CTA turns each cached job's activation (x, or gelu_mul(gate, up))
  // into scaled hi/lo fragments in shared memory.
  if (tl.prep) {
    wait_prior_grids();  // the activations and outputs belong to the previous kernels until now
    for (uint32_t j = 0; j < s_sched.nx; ++j) {
      const XJob J = tl.dev ? tl.jobs[s_sched.xjob[j]] : tl.inl_job;
      const bool store_act = J.mode && J.act && ((s_sched.act_mask >> j) & 1u);
      for (uint32_t t = 0; t < batch; ++t) {
        const float inv = job_token_prep<kEngineWarps>(J, t, batch, store_act,
                                                       reinterpret_cast<uint4*>(xsm + s_sched.xoff[j]), s_red);
        if (threadIdx.x == 0) s_inv[j][t] = inv;
      }
    }
    __syncthreads();
  }
  // Each warp's copy engine starts after the activation preparation: the
  // preparation's reads then do not queue behind a full ring of weight
  // copies (measured: the first stage's math starts ~1.5 us sooner).
  if (lane == 0) {
    Cursor F;
    F.claims = 0;
    F.issued = 0;
    F.ti = t_first;
    F.item = timed_out ? c1 : claim(F);
    cursor_task(F, tl, ts);
    cursor_seek(F, tl, ts, c1);
    cursor_range(F, gq, ks_n);
    for (int st = 0; st < kSt && F.item < c1; ++st) issue_next(F, st);
    s_cur[warp] = F;
  }
  __syncwarp();

  // B-fragment column of this lane in each n-tile: any stored column serves,
  // results of columns past the batch are never read.
  const uint32_t cols_last = COLS > 0 ? (uint32_t)COLS : 2u * (batch - 4u * (NT - 1));
  uint32_t lane_off[NT], wstep[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const uint32_t cols = n + 1 < NT ? 8u : cols_last;
    lane_off[n] = ((g % cols) * 4u + c) * 16u;
    wstep[n] = cols * 64u;
  }

  uint32_t consumed = 0;
  uint32_t item = timed_out ? c1 : ring[0];
  uint32_t ti = t_first;
  Hot<NT> H = hot_of<NT>(tl, ts, ti, s_sched, c, batch, s_inv);
  while (item < c1 && item >= H.item_end) H = hot_of<NT>(tl, ts, ++ti, s_sched, c, batch, s_inv);
  uint32_t b = gq * (H.nb / ks_n), b_hi = b + H.nb / ks_n, k = 0, tiles = 0;
  float* s_part = reinterpret_cast<float*>(xsm + xcache_cap);  // K-split partial sums

  float acc[NT][2][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int h = 0; h < 2; ++h) acc[n][h][0] = acc[n][h][1] = acc[n][h][2] = acc[n][h][3] = 0.0f;

  while (item < c1 && !timed_out) {
    const uint32_t slot = k % kSt;
    if (!mbar_wait(&bars[slot], (k / kSt) & 1u, spin)) {
      timed_out = true;
      break;
    }
    const uint8_t* stg = wsm + slot * kSB;
    const bool sx = XS ? true : (H.xs != 0xffffffffu);
    if constexpr (FMT == kFmtQ6K) {
      // one super-block per stage: compute straight from the stage (the
      // other stages stay in flight meanwhile), then hand it back
      const Q6Rows R = q6_rows(stg, g, c);
      // (each branch forms its own fragment pointers, so shared-memory ones
      // stay recognisably shared and load with LDS)
      // a non-finite d anywhere in the warp's rows: the exact (slower) form
      const bool odd_d = ((R.da & 0x7C00u) == 0x7C00u) || ((R.db & 0x7C00u) == 0x7C00u);
      const bool exact = __any_sync(0xffffffffu, odd_d);
      if (sx) {
        const uint8_t* base[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) base[n] = xsm + H.xs + (n * H.nb * 4096u + b * 8u * wstep[n] + lane_off[n]);
        if (exact) q6_block_math<NT, COLS, true, true>(acc, R, c, base, wstep);
        else q6_block_math<NT, COLS, true, false>(acc, R, c, base, wstep);
      } else {
        const uint8_t* base[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n)
          base[n] = reinterpret_cast<const uint8_t*>(H.xfrag) + (n * H.nb * 4096u + b * 8u * wstep[n] + lane_off[n]);
        if (exact) q6_block_math<NT, COLS, false, true>(acc, R, c, base, wstep);
        else q6_block_math<NT, COLS, false, false>(acc, R, c, base, wstep);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && s_cur[warp].item < c1) {
        Cursor F = s_cur[warp];
        issue_next(F, slot);
        s_cur[warp] = F;
      }
      ++b;
    } else {
    // PR: both super-blocks of every stage, tile rows kPairTileBytes apart
    const uint32_t nblk = PR ? Pipe<FMT>::kBlocks : min(Pipe<FMT>::kBlocks, b_hi - b);
    const uint32_t rs = PR ? kPairTileBytes : H.tile_bytes;
    // both super-blocks of a stage in one unrolled body, so the second
    // block's shared-memory loads can be scheduled under the first one's math
#pragma unroll
    for (uint32_t sb = 0; sb < nblk; ++sb, ++b) {
      const BlockRegs R = read_block(stg + g * rs + sb * kBlockBytes, stg + (g + 8) * rs + sb * kBlockBytes, c);
      if (sb + 1 == nblk) {
        // the whole stage is in registers: hand it back to the copy engine
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && s_cur[warp].item < c1) {
          Cursor F = s_cur[warp];
          issue_next(F, slot);
          s_cur[warp] = F;
        }
      }
      // n-tiles before the last are full (8 columns): nb*4096 bytes each
      // (each branch forms its own fragment pointers, so shared-memory ones
      // stay recognisably shared and load with LDS)
      if (sx) {
        const uint8_t* base[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) base[n] = xsm + H.xs + (n * H.nb * 4096u + b * 8u * wstep[n] + lane_off[n]);
        block_math<NT, COLS, true>(acc, R, c, bsel, base, wstep);
      } else {
        const uint8_t* base[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n)
          base[n] = reinterpret_cast<const uint8_t*>(H.xfrag) + (n * H.nb * 4096u + b * 8u * wstep[n] + lane_off[n]);
        block_math<NT, COLS, false>(acc, R, c, bsel, base, wstep);
      }
    }
    }
    ++k;
    if (b < b_hi) continue;

    // item done: acc[n][*][0..1] = (hi, lo) parts of token 4n+c for row ra, [2..3] for rb
    const uint32_t ra = (item - H.item_begin) * kTileRows + g, rb = ra + 8;
    const bool va = ra < H.M, vb = rb < H.M;
    if constexpr (KS > 1) {
      // K-split: leave this warp's slice sums, wait for the group's other
      // warps (bounded), and warp 0 of the group adds the slices in order.
      const uint32_t par = tiles & 1u;
      float* mine = s_part + (((par * ngrp + grp) * ks_n + gq) * kTileRows) * 4;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t t = 4 * n + c;
        if (t < batch) {
          mine[g * 4 + t] = (acc[n][0][0] + acc[n][1][0]) + (acc[n][0][1] + acc[n][1][1]);
          mine[(g + 8) * 4 + t] = (acc[n][0][2] + acc[n][1][2]) + (acc[n][0][3] + acc[n][1][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_gbar[grp]);
      if (!mbar_wait(&s_gbar[grp], par, spin)) {
        timed_out = true;
        break;
      }
      if (gq == 0) {
        const float* all = s_part + (((par * ngrp + grp) * ks_n) * kTileRows) * 4;
        const uint32_t t = c;
        if (t < batch) {
          float sa = all[g * 4 + t], sb = all[(g + 8) * 4 + t];
          for (uint32_t q = 1; q < ks_n; ++q) {
            sa += all[(q * kTileRows + g) * 4 + t];
            sb += all[(q * kTileRows + g + 8) * 4 + t];
          }
          if (va) H.y[(uint64_t)t * H.M + ra] = sa * H.inv[0];
          if (vb) H.y[(uint64_t)t * H.M + rb] = sb * H.inv[0];
        }
      }
      ++tiles;
    }
    if (KS > 1) {
      // (the group combine above wrote y)
    } else if (H.kind == kTaskPlain) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t t = 4 * n + c;
        if (t < batch) {
          if (va) H.y[(uint64_t)t * H.M + ra] = ((acc[n][0][0] + acc[n][1][0]) + (acc[n][0][1] + acc[n][1][1])) * H.inv[n];
          if (vb) H.y[(uint64_t)t * H.M + rb] = ((acc[n][0][2] + acc[n][1][2]) + (acc[n][0][3] + acc[n][1][3])) * H.inv[n];
        }
      }
    } else {
      // The token's results sit in the c == 0 lanes (row ra in [0..1], rb in
      // [2..3]); lane c == 1 takes rb from its neighbour, so 16 lanes each
      // finish one row (softcap, logits, per-residue best) in parallel.
      const float v_a = ((acc[0][0][0] + acc[0][1][0]) + (acc[0][0][1] + acc[0][1][1])) * H.inv[0];
      const float v_b = __shfl_sync(0xffffffffu,
                                    ((acc[0][0][2] + acc[0][1][2]) + (acc[0][0][3] + acc[0][1][3])) * H.inv[0],
                                    lane & ~3u);
      if (c < 2 && (c ? vb : va)) {
        const EngineTask& T = ts.table ? ts.table[ti - ts.t0] : tl.inl;
        const uint32_t row = c ? rb : ra;
        float v = c ? v_b : v_a;
        if (T.cap > 0.0f) v = softcap(v, T.cap);
        if (T.logits) T.logits[row] = v;
        const uint32_t gi = T.row_offset + row;
        const uint32_t res = gi & 255u;  // the 16 rows of a tile have distinct residues
        if (better(v, gi, s_bv[res], s_bi[res])) {
          s_bv[res] = v;
          s_bi[res] = gi;
        }
      }
      __syncwarp();
    }
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int h = 0; h < 2; ++h) acc[n][h][0] = acc[n][h][1] = acc[n][h][2] = acc[n][h][3] = 0.0f;
    ++consumed;
    __syncwarp();
    item = ring[consumed & 3u];
    while (item < c1 && item >= H.item_end) H = hot_of<NT>(tl, ts, ++ti, s_sched, c, batch, s_inv);
    b = gq * (H.nb / ks_n);
    b_hi = b + H.nb / ks_n;
  }

  allow_dependents();
  if (timed_out) {
    // record the failure, then let every copy still in flight land (bounded)
    if (lane == 0) atomicOr(sel.status, 1u);
    if (lane == 0)
      for (uint32_t j = k; j < s_cur[warp].issued; ++j) mbar_wait(&bars[j % kSt], (j / kSt) & 1u, spin);
  }

  if (!has_select) return;
  // Merge the CTA's 16 per-warp candidate sets in shared memory (thread r
  // owns residue r) and publish one key per touched residue; the last CTA of
  // the grid turns the keys into the 256 candidates + argmax and resets the
  // scratch.  One publish per CTA keeps the same-address atomics few.
  __shared__ uint32_t s_last;
  __syncthreads();
  float* s_all = reinterpret_cast<float*>(xsm + xcache_cap);  // warp w: values at w*512, indices at w*512+256
  if (threadIdx.x < 256) {
    const uint32_t r = threadIdx.x;
    float v = s_all[r];
    uint32_t i = reinterpret_cast<const uint32_t*>(s_all)[256 + r];
#pragma unroll 1
    for (int w = 1; w < kEngineWarps; ++w) {
      const float wv = s_all[w * 512 + r];
      const uint32_t wi = reinterpret_cast<const uint32_t*>(s_all)[w * 512 + 256 + r];
      if (better(wv, wi, v, i)) {
        v = wv;
        i = wi;
      }
    }
    if (!(v == kFloorE && i == 0u)) atomicMax(&sel.slots[r], sel_key(v, i));
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(sel.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const EngineTask S = task_at(tl, tl.select_task);
  float* f_v = s_all;
  uint32_t* f_i = reinterpret_cast<uint32_t*>(s_all) + 256;
  if (threadIdx.x < 256) {
    const uint32_t r = threadIdx.x;
    const unsigned long long key = atomicExch(&sel.slots[r], sel_key(kFloorE, 0u));
    float v;
    uint32_t i;
    sel_unkey(key, v, i);
    if (tl.xc.world == 0) {
      S.cand_val[r] = v;
      S.cand_idx[r] = i;
    }
    f_v[r] = v;
    f_i[r] = i;
  }
  __syncthreads();
  if (tl.xc.world > 0) {
    // Sharded head: push this rank's candidates to every rank's mailbox,
    // wait for every rank's, merge (per residue: larger value, then lower
    // index) into the outputs; the argmax tree below runs on the merge.
    // Each sender has two slots per mailbox, used by calls of alternating
    // epoch parity: a rank reaches call e+2's stores only after every rank
    // raised its call-(e+1) flag, which each does after finishing its call-e
    // merge, so a slot is never overwritten while its reader still needs it.
    const Exchange& X = tl.xc;
    __shared__ uint32_t s_epoch;
    if (threadIdx.x == 0) {
      s_epoch = *X.epoch + 1u;
      *X.epoch = s_epoch;
    }
    __syncthreads();
    const uint32_t ep = s_epoch;
    const uint32_t par = ep & 1u;
    for (uint32_t p = 0; p < X.world; ++p) {
      uint32_t* slot = X.peer[p] + mailbox_slot(X.rank, par);
      if (threadIdx.x < 256) {
        slot[threadIdx.x] = __float_as_uint(f_v[threadIdx.x]);
        slot[256 + threadIdx.x] = f_i[threadIdx.x];
      }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < X.world)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(X.peer[threadIdx.x] + mailbox_slot(X.rank, par) + kSlotFlag),
                   "r"(ep)
                   : "memory");
    // every rank's slot in this rank's mailbox (bounded wait)
    if (threadIdx.x < X.world) {
      const uint32_t* flag = X.peer[X.rank] + mailbox_slot(threadIdx.x, par) + kSlotFlag;
      bool ok = false;
      for (uint32_t i = 0; i < spin && !ok; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        ok = (v == ep);
      }
      if (!ok) atomicOr(sel.status, 1u);
      __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x < 256) {
      const uint32_t r = threadIdx.x;
      const uint32_t* mb = X.peer[X.rank];
      float bv = __uint_as_float(__ldcv(mb + mailbox_slot(0, par) + r));
      uint32_t bi = __ldcv(mb + mailbox_slot(0, par) + 256 + r);
      for (uint32_t q = 1; q < X.world; ++q) {
        const float v = __uint_as_float(__ldcv(mb + mailbox_slot(q, par) + r));
        const uint32_t i = __ldcv(mb + mailbox_slot(q, par) + 256 + r);
        if (better(v, i, bv, bi)) {
          bv = v;
          bi = i;
        }
      }
      S.cand_val[r] = bv;
      S.cand_idx[r] = bi;
      f_v[r] = bv;
      f_i[r] = bi;
    }
    __syncthreads();
  }
  // the reference's argmax tree (shaders/argmax.wgsl:21-27): the partner wins
  // only when strictly greater
  for (uint32_t st = 128; st > 0; st >>= 1) {
    const uint32_t t = threadIdx.x;
    if (t < st && f_v[t + st] > f_v[t]) {
      f_v[t] = f_v[t + st];
      f_i[t] = f_i[t + st];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *S.argmax = f_i[0];
    *sel.counter = 0u;
  }
}

__global__ void init_select_kernel(SelectScratch sc, int clear_status) {
  sc.slots[threadIdx.x] = sel_key(kFloorE, 0u);
  if (threadIdx.x == 0) {
    *sc.counter = 0u;
    if (clear_status) *sc.status = 0u;
  }
}

constexpr size_t kAlignSlack = 128;  // room to align the dynamic shared memory base

// K-split partial sums: 2 tile parities x kEngineWarps slices x 16 rows x 4 tokens.
constexpr size_t kPartSmem = (size_t)2 * kEngineWarps * kTileRows * 4 * sizeof(float);

// hs: the launch has an LM head (per-warp candidate tables); else the same
// space holds K-split partial sums.
template <int FMT>
size_t xcache_bytes(int hs) {
  return kSmemLimit - kStaticSmemHeadroom - kAlignSlack - weight_smem<FMT>() - kTaskSmem -
         (hs ? kSelectSmem : kPartSmem);
}

template <int NT, int COLS, int KS, int FMT, int XS, int PR>
cudaError_t launch_xs(const TaskList& tasks, const CUtensorMap& map, const CUtensorMap& dmap, uint32_t batch,
                           int hs, const SelectScratch& sel, uint32_t grid, cudaStream_t s) {
  const size_t xcap = xcache_bytes<FMT>(hs);
  const size_t smem = kAlignSlack + weight_smem<FMT>() + kTaskSmem + xcap + (hs ? kSelectSmem : kPartSmem);
  static std::atomic<uint8_t> attr_set[kAttrDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = smem_attr_once(attr_set, dev, engine_kernel<NT, COLS, KS, FMT, XS, PR>, (int)(kSmemLimit - kStaticSmemHeadroom));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kEngineWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, engine_kernel<NT, COLS, KS, FMT, XS, PR>, tasks, map, dmap, batch, hs, sel,
                            (uint32_t)xcap);
}

template <int NT, int COLS, int KS = 1, int FMT = kFmtQ4K>
cudaError_t launch_variant(const TaskList& tasks, const CUtensorMap& map, const CUtensorMap& dmap, uint32_t batch,
                           int hs, const SelectScratch& sel, uint32_t grid, cudaStream_t s) {
  if constexpr (FMT == kFmtQ4K) {
    if (tasks.pairs)
      return tasks.prep ? launch_xs<NT, COLS, KS, FMT, 1, 1>(tasks, map, dmap, batch, hs, sel, grid, s)
                        : launch_xs<NT, COLS, KS, FMT, 0, 1>(tasks, map, dmap, batch, hs, sel, grid, s);
  }
  return tasks.prep ? launch_xs<NT, COLS, KS, FMT, 1, 0>(tasks, map, dmap, batch, hs, sel, grid, s)
                    : launch_xs<NT, COLS, KS, FMT, 0, 0>(tasks, map, dmap, batch, hs, sel, grid, s);
}

}  // namespace

cudaError_t init_select_scratch(const SelectScratch& sc, cudaStream_t s, bool clear_status) {
  init_select_kernel<<<1, 256, 0, s>>>(sc, clear_status ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_xprep(const JobList& jobs, uint32_t batch, cudaStream_t s) {
  xprep_kernel<<<jobs.n * batch, 256, 0, s>>>(jobs, batch);
  return cudaGetLastError();
}

// One CTA per SM up to the item count: a launch with fewer items than SMs
// gives each item an SM of its own (the math of an item then runs with the
// whole SM to itself instead of sharing it with 15 other warps).
uint32_t engine_grid(uint32_t total_items, int sm_count) {
  uint32_t grid = total_items;
  if (grid > (uint32_t)sm_count) grid = (uint32_t)sm_count;
  return grid == 0 ? 1 : grid;
}

uint32_t engine_xcache_bytes(bool has_select, uint32_t fmt) {
  return (uint32_t)(fmt == kFmtQ6K ? xcache_bytes<kFmtQ6K>(has_select ? 1 : 0)
                                   : xcache_bytes<kFmtQ4K>(has_select ? 1 : 0));
}

namespace {
using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

// The driver's tensor-map encoder, looked up once through the runtime (the
// library does not link libcuda directly).
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

cudaError_t encode_weight_map(CUtensorMap* map, const void* w, uint32_t M, uint32_t N, uint32_t* tile_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const uint64_t nb = N / kQK;
  const cuuint64_t dims[2] = {nb * (kBlockBytes / 4), M};
  const cuuint64_t strides[1] = {nb * kBlockBytes};
  const cuuint32_t estr[2] = {1, 1};
  // Two-block boxes are 76 words wide; if the encoder refuses a box wider
  // than a 2-block row, fall back to the exact 72-word row.
  const cuuint32_t widths[2] = {nb >= 2 ? kBoxWords2 : kBoxWords1, nb >= 2 ? 2 * kBoxWords1 : kBoxWords1};
  for (cuuint32_t box_w : widths) {
    const cuuint32_t box[2] = {box_w, (cuuint32_t)kTileRows};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS) {
      *tile_bytes = box_w * 4;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t encode_q6k_maps(CUtensorMap* maps, const void* w, uint32_t M, uint32_t N, uint32_t* tile_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const uint64_t nb = N / kQK;
  const cuuint32_t estr[2] = {1, 1};
  {
    const cuuint64_t dims[2] = {nb * kQ6BodyWords, M};
    const cuuint64_t strides[1] = {nb * kQ6BodyBytes};
    const cuuint32_t box[2] = {kQ6BodyWords, (cuuint32_t)kTileRows};
    if (fn(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const uint32_t mp = q6k_dpitch(M);
    void* dp = static_cast<uint8_t*>(const_cast<void*>(w)) + (uint64_t)M * nb * kQ6BodyBytes;
    const cuuint64_t dims[2] = {mp, nb};
    const cuuint64_t strides[1] = {(cuuint64_t)mp * 2u};
    const cuuint32_t box[2] = {(cuuint32_t)kTileRows, 1};
    if (fn(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, dp, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  *tile_bytes = kQ6BodyBytes;
  return cudaSuccess;
}

// First work item whose super-blocks start at or after cost position p.
static uint32_t host_item_at_cost(const EngineTask* t, uint32_t n, uint32_t total_cost, uint32_t total_items,
                                  uint64_t p) {
  if (p >= total_cost) return total_items;
  uint32_t lo = 0, hi = n - 1;  // last task with cost_begin <= p
  while (lo < hi) {
    const uint32_t mid = (lo + hi + 1) / 2;
    if (t[mid].cost_begin <= p) lo = mid; else hi = mid - 1;
  }
  const uint32_t ic = item_cost(t[lo].N, t[lo].kind);
  const uint64_t item = t[lo].item_begin + (p - t[lo].cost_begin + ic - 1) / ic;
  return item < t[lo].item_end ? (uint32_t)item : t[lo].item_end;
}

void engine_schedule(const EngineTask* tasks, uint32_t n, uint32_t total_cost, uint32_t total_items,
                     uint32_t batch, uint32_t grid, uint32_t xcache_cap, CtaSched* out) {
  for (uint32_t b = 0; b < grid; ++b) {
    CtaSched& S = out[b];
    S = CtaSched{};
    S.c0 = host_item_at_cost(tasks, n, total_cost, total_items, (uint64_t)total_cost * b / grid);
    S.c1 = host_item_at_cost(tasks, n, total_cost, total_items, (uint64_t)total_cost * (b + 1) / grid);
    if (S.c0 >= S.c1) continue;
    uint32_t t0 = 0;
    while (t0 < n && tasks[t0].item_end <= S.c0) ++t0;
    uint32_t t1 = t0;
    while (t1 + 1 < n && tasks[t1 + 1].item_begin < S.c1) ++t1;
    S.t0 = t0;
    S.nt = (t1 - t0 + 1 <= (uint32_t)kMaxCtaTasks) ? t1 - t0 + 1 : 0u;
    uint32_t used = 0;
    for (uint32_t i = t0; i <= t1; ++i) {
      bool seen = false;
      for (uint32_t j = 0; j < S.nx; ++j) seen |= (S.xptr[j] == tasks[i].xfrag);
      const uint32_t bytes = (uint32_t)xfrag_bytes(tasks[i].N, batch);
      if (seen || S.nx == (uint32_t)kMaxCachedX || used + bytes > xcache_cap) continue;
      S.xptr[S.nx] = tasks[i].xfrag;
      S.xjob[S.nx] = tasks[i].aux;  // the task's preparation job
      S.xoff[S.nx] = used;
      S.xbytes[S.nx] = bytes;
      used += bytes;
      ++S.nx;
    }
  }
}

bool schedule_covers_tasks(const EngineTask* tasks, uint32_t n, const CtaSched* sched, uint32_t grid) {
  for (uint32_t b = 0; b < grid; ++b) {
    const CtaSched& S = sched[b];
    for (uint32_t i = 0; i < n; ++i) {
      if (tasks[i].item_end <= S.c0 || tasks[i].item_begin >= S.c1) continue;
      bool found = false;
      for (uint32_t j = 0; j < S.nx; ++j) found |= (S.xptr[j] == tasks[i].xfrag);
      if (!found) return false;
    }
  }
  return true;
}

template <int FMT>
cudaError_t launch_fmt(const TaskList& tasks, const CUtensorMap& map, const CUtensorMap& dmap, uint32_t batch,
                       int hs, const SelectScratch& sel, uint32_t grid, cudaStream_t s) {
  switch (batch) {
    case 1: return launch_variant<1, 2, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
    case 2: return launch_variant<1, 4, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
    case 3: return launch_variant<1, 6, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
    case 4: return launch_variant<1, 8, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
    default:
      switch ((batch + 3) / 4) {
        case 2: return launch_variant<2, 0, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
        case 3: return launch_variant<3, 0, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
        default: return launch_variant<4, 0, 1, FMT>(tasks, map, dmap, batch, hs, sel, grid, s);
      }
  }
}

cudaError_t launch_engine(const TaskList& tasks, const CUtensorMap& map, uint32_t batch, bool has_select,
                          const SelectScratch& sel, int sm_count, cudaStream_t s, const CUtensorMap* dmap) {
  const uint32_t grid = tasks.sched ? tasks.grid : engine_grid(tasks.total_items, sm_count);
  const int hs = has_select ? 1 : 0;
  const CUtensorMap& dm = dmap ? *dmap : map;
  if (tasks.fmt == kFmtQ6K) {
    if (tasks.ksplit > 1) return cudaErrorInvalidValue;
    return launch_fmt<kFmtQ6K>(tasks, map, dm, batch, hs, sel, grid, s);
  }
  if (tasks.fmt != kFmtQ4K) return cudaErrorInvalidValue;
  if (tasks.ksplit == 4) {
    switch (batch) {
      case 1: return launch_variant<1, 2, 4>(tasks, map, dm, batch, hs, sel, grid, s);
      case 2: return launch_variant<1, 4, 4>(tasks, map, dm, batch, hs, sel, grid, s);
      case 3: return launch_variant<1, 6, 4>(tasks, map, dm, batch, hs, sel, grid, s);
      case 4: return launch_variant<1, 8, 4>(tasks, map, dm, batch, hs, sel, grid, s);
      default: return cudaErrorInvalidValue;
    }
  }
  return launch_fmt<kFmtQ4K>(tasks, map, dm, batch, hs, sel, grid, s);
}

}  // namespace q4k
