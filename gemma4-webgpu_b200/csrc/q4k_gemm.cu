// Batched Q4_K GEMM for sm_100a: Y[t][m] = sum_k w16[m][k] * x[t][k] for T
// activation rows at once (prefill, or many independent sequences sharing
// the weights).  The reference has only the one-row matmul_quant
// (shaders/matmul_quant.wgsl:21-54); this is that operation for T >= 64 rows,
// with the same weights w16 = f16_rne(f32(d*sc*q - dmin*m)) (src/gguf.ts:
// 168-210 + 425-473).
//
// Here the work is a dense contraction, so it runs on the 5th-generation
// tensor cores.  A tile of Y is 256 weight rows x up to 256 operand rows (one
// operand row per activation row in the f16 form, two -- the exact f16 hi
// and lo parts, scaled per row by a power of two -- in the exact form),
// computed as two 128-row blocks, each with tcgen05.mma (M = 128, N = the
// tile's operand rows, K = 16 per instruction) into its own fp32
// accumulator in tensor memory; both blocks read the same B tile, so the
// activation operand is fetched once per 256 weight rows.  The launch is
// persistent: one CTA per SM walks its tiles, every role keeping its ring
// counters from tile to tile.  Per 64-wide K step:
//   * the B operand arrives by TMA tensor copies in a swizzled K-major
//     layout;
//   * the A operand, the 256 x 64 f16 weights, is dequantized by 16 warps
//     (two groups of 8, one per K-step parity), computed before its stage is
//     free and stored once it is; the raw Q4_K super-blocks reach shared
//     memory by TMA, one 144-byte box per tile row per super-block column
//     (four K steps), from a copy warp of its own;
//   * one thread issues the MMAs and commits them to the stage's "empty"
//     barrier, which frees the stage for the producers; it waits on one
//     barrier per step, the producers' plus a relay arrival once B landed.
// Two forms (GemmForm below): SS, A in shared memory, four K = 32 stages;
// TS, for tiles of at most 128 operand rows (a batch of up to 128 f16 or 64
// exact activation rows), A stored straight into tensor memory, four K = 64
// stages.  The epilogue (the 16 producer warps: per accumulator one per
// 32-lane quarter of tensor memory and column half) reads the accumulators,
// adds each activation row's hi and lo columns, undoes the scale and stores
// Y (or adds into it, for the two K halves of a split matrix).  f16 x f16
// products are exact and the hi/lo split carries x to ~2^-22, so the result
// is the f32 dot product of the reference's f16 weights with x, up to fp32
// accumulation order.
//
// Every mbarrier wait is bounded; on expiry the CTA records the failure in
// the status word, lets its copies land and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_ctx.cuh"
#include "q4k_dequant.cuh"
#include "q4k_device.cuh"
#include "q4k_ptx.cuh"

namespace q4k {
namespace {

constexpr uint32_t kGMmaM = 128;                        // MMA M = TMEM lanes
constexpr uint32_t kGHalves = 2;                        // MMA row blocks per CTA (one accumulator each)
constexpr uint32_t kGRows = kGMmaM * kGHalves;          // weight rows per CTA tile
constexpr uint32_t kGTokens = 128;                      // max activation rows per tile (MMA N = 2 per row)
constexpr uint32_t kGK = 64;                            // K per producer step (one 32-byte qs group per row)
constexpr uint32_t kGDqGroups = 2;                      // producer groups: group p takes the K steps = p (mod 2)
constexpr uint32_t kGDqWarps = 8 * kGDqGroups;          // dequantizing warps (8 per group), also the epilogue
constexpr uint32_t kGRawWarp = 2 + kGDqWarps;            // the raw-weight copy warp
constexpr uint32_t kGThreads = (3 + kGDqWarps) * 32;    // + B-copy warp + MMA warp + raw-copy warp
constexpr uint32_t kGRawStages = 2;                     // raw super-block columns in flight (SS form)
constexpr uint32_t kGRawBytes = kGRows * kBlockBytes;   // 36 KB: one super-block of each of the 256 rows
constexpr uint32_t kGAccCols = 2 * kGTokens;            // fp32 columns of one accumulator
constexpr uint32_t kGTmemCols = kGHalves * kGAccCols;   // 512: all of tensor memory

// The two forms of the kernel.  SS: both operands in shared memory, tiles of
// up to 256 operand rows (MMA N <= 256), four stages of K = 32 in the 64-byte
// swizzled layout (two 64-wide K steps in flight, but a stage's B copy is
// issued half a step sooner than with two stages of K = 64: the B copy
// from L2 took ~0.65 us against ~0.5 us of MMAs per K step).  TS (tiles of at most
// 128 operand rows): the producers store the weights straight into tensor
// memory (tcgen05.st) and the MMA reads A from there.  A single-thread
// stream of M = 128 kind::f16 MMAs measured on B200 costs ~89 cycles per
// instruction for any N <= 128 with A in shared memory (N = 256: 128 cycles,
// the full rate), but 54 cycles at N = 64 and 64 cycles at N = 128 (the full
// rate) with A in tensor memory; the A stores, their proxy fence and the
// tensor core's A reads also leave shared memory.  Tensor memory then holds
// the two 128-column accumulators and four A stages of 2 x 32 columns (a
// row's 64 weights of a K step, two f16 per column, lane = row); the freed
// shared memory holds four B stages and four raw super-block columns.
template <bool kTA>
struct GemmForm {
  static constexpr uint32_t kStages = 4;
  static constexpr uint32_t kStageK = kTA ? kGK : kGK / 2;              // K per operand stage
  static constexpr uint32_t kRowBytes = kStageK * 2;                    // operand row: 128 (TS B) or 64 bytes
  static constexpr uint32_t kSbo = 8 * kRowBytes;                       // bytes between 8-row groups
  static constexpr uint32_t kLayout = kTA ? 2 : 4;                      // descriptor swizzle: 128 B / 64 B
  static constexpr uint32_t kASub = kGMmaM * kRowBytes;                 // smem A block (SS)
  static constexpr uint32_t kABytes = kTA ? 0 : kGHalves * kASub;       // smem A stage
  static constexpr uint32_t kBBytes = (kTA ? 128 : 2 * kGTokens) * kRowBytes;  // smem B stage (largest box)
  static constexpr uint32_t kAccCols = kTA ? 128 : kGAccCols;          // tensor-memory columns per accumulator
  static constexpr uint32_t kACol = kGHalves * kAccCols;               // first A column (TS)
  static constexpr uint32_t kAStageCols = kGHalves * (kGK / 2);        // A columns per stage (TS)
  static constexpr uint32_t kRawStages = kTA ? 4 : kGRawStages;        // raw super-block columns in flight
  static constexpr uint32_t kStepsPerBlock = 256 / kStageK;            // operand stages per super-block column
  static constexpr size_t kSmem = 1024 + (size_t)kStages * (kABytes + kBBytes) + (size_t)kRawStages * kGRawBytes;
  static_assert(!kTA || kACol + kStages * kAStageCols <= kGTmemCols, "TS tensor-memory layout");
  static_assert(kStages % (2 * kGK / kStageK) == 0, "a 64-wide K step's stages are filled by one producer group");
};
constexpr uint32_t kGMaxTsRows = 128;  // operand rows per tile up to which the TS form runs

// UMMA shared-memory descriptor of a K-major tile in a swizzled layout:
// rows of 128 (layout 2, 128-byte swizzle) or 64 bytes (layout 4, 64-byte
// swizzle), 8-row groups `sbo` bytes apart (stride offset), the leading
// offset unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor, kind::f16: D fp32, A and B f16 and K-major, M = 128.
__device__ __forceinline__ uint32_t idesc_f16(uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((kGMmaM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// The same with A in tensor memory: `a_tmem` addresses the 128 lanes x 8
// columns (two f16 per column, the lower K index in the low half) of one
// 16-wide k slice.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 tensor-memory lanes from
// the 8 chunks of each lane's row (chunk c -> columns 4c..4c+3), then waits
// until the stores are complete.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint4 (&c)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(c[0].x), "r"(c[0].y), "r"(c[0].z), "r"(c[0].w), "r"(c[1].x), "r"(c[1].y), "r"(c[1].z), "r"(c[1].w),
      "r"(c[2].x), "r"(c[2].y), "r"(c[2].z), "r"(c[2].w), "r"(c[3].x), "r"(c[3].y), "r"(c[3].z), "r"(c[3].w),
      "r"(c[4].x), "r"(c[4].y), "r"(c[4].z), "r"(c[4].w), "r"(c[5].x), "r"(c[5].y), "r"(c[5].z), "r"(c[5].w),
      "r"(c[6].x), "r"(c[6].y), "r"(c[6].z), "r"(c[6].w), "r"(c[7].x), "r"(c[7].y), "r"(c[7].z), "r"(c[7].w)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// K order inside the operand tiles.  The A producers write each 16-byte
// chunk of 8 weights in the order dequant_word yields them, elements
// (0, 2, 1, 3, 4, 6, 5, 7) of the chunk; the B operand (x) is stored in the
// same order, so the contraction over K is unchanged.  Position p of a chunk
// holds element chunk_elem(p) (bits 0 and 1 swapped).
__host__ __device__ constexpr uint32_t chunk_elem(uint32_t p) {
  return (p & ~3u) | ((p & 1u) << 1) | ((p >> 1) & 1u);
}

struct GemmArgs {
  const uint8_t* w;        // Q4_K [M][N/256*144]
  float* y;                // [T][M]
  const float* inv_scale;  // [T]: 1/scale of each activation row
  uint32_t M, N, T;
  uint32_t tile_tokens;    // activation rows per CTA tile (parts x tile_tokens = 128 or 256 operand rows,
                           // the B map's box)
  uint32_t parts;          // operand rows per activation row: 2 (exact f16 hi + lo) or 1 (f16 only)
  uint32_t* status;        // bit 0: a bounded wait expired
  uint32_t spin;           // polls per bounded wait (0: kSpinLimit)
  const GemmTask* tasks;   // multi-matrix launch: task table (null: the single matrix above)
  const uint2* tiles;      // multi-matrix launch: tile i = (task, row tile | token tile << 16)
  uint32_t n_tiles;        // tiles of the launch; CTA b takes tiles b, b + gridDim.x, ...
};

// The raw Q4_K bytes one A-producer thread (one row) needs for one K step:
// the super-block header and the step's 32-byte qs group, read from the
// row's 144 bytes in a raw stage (rows 144 bytes apart: the 8 lanes of each
// 16-byte load phase hit distinct banks).
struct RawGroup {
  uint4 hd, q0, q1;
};

__device__ __forceinline__ RawGroup raw_group(const uint8_t* srow, uint32_t j) {
  RawGroup g;
  g.hd = *reinterpret_cast<const uint4*>(srow);
  g.q0 = *reinterpret_cast<const uint4*>(srow + 16 + 32 * j);
  g.q1 = *reinterpret_cast<const uint4*>(srow + 32 + 32 * j);
  return g;
}

// One tile row's 64 weights of a K step as the 8 swizzle chunks they occupy
// (chunks 0-3: low nibbles, local k 0..31; chunks 4-7: high, k 32..63).
struct RowChunks {
  uint4 c[8];
};

__device__ __forceinline__ RowChunks dequant_group(const RawGroup& g, uint32_t j) {
  RowChunks o;
  const RowConsts rc = row_consts(g.hd, j, scale_sel(j));
  const uint32_t wd[8] = {g.q0.x, g.q0.y, g.q0.z, g.q0.w, g.q1.x, g.q1.y, g.q1.z, g.q1.w};
#pragma unroll
  for (uint32_t c = 0; c < 4; ++c) {
    const WordPairs p0 = dequant_word(wd[2 * c], rc), p1 = dequant_word(wd[2 * c + 1], rc);
    o.c[c] = make_uint4(p0.lo02, p0.lo13, p1.lo02, p1.lo13);
    o.c[4 + c] = make_uint4(p0.hi02, p0.hi13, p1.hi02, p1.hi13);
  }
  return o;
}

// Tile i of a launch: an entry of the multi-matrix tile table, or of the
// single matrix's (row tile, token tile) grid, row tiles fastest.
struct GemmTile {
  const CUtensorMap* amap;
  const CUtensorMap* bmap;
  float* y;
  const float* inv_scale;
  uint32_t M, N, T, tile_tokens, row0, tok0, n_mma;
  uint32_t k0, acc;  // K range start; 1: add into y (K split)
};

__device__ __forceinline__ GemmTile gemm_tile(const GemmArgs& a, const CUtensorMap* amap, const CUtensorMap* bmap,
                                              uint32_t i) {
  GemmTile t;
  if (a.tiles) {
    const uint2 tl = a.tiles[i];
    const GemmTask& tk = a.tasks[tl.x];
    t.amap = tk.amap;
    t.bmap = tk.bmap;
    t.y = tk.y;
    t.inv_scale = tk.inv_scale;
    t.M = tk.M;
    t.N = tk.N;
    t.T = tk.T;
    t.tile_tokens = tk.tile_tokens;
    t.row0 = (tl.y & 0xffffu) * kGRows;
    t.tok0 = (tl.y >> 16) * t.tile_tokens;
    t.k0 = tk.k0;
    t.acc = tk.accumulate;
  } else {
    const uint32_t row_tiles = (a.M + kGRows - 1) / kGRows;
    t.amap = amap;
    t.bmap = bmap;
    t.y = a.y;
    t.inv_scale = a.inv_scale;
    t.M = a.M;
    t.N = a.N;
    t.T = a.T;
    t.tile_tokens = a.tile_tokens;
    t.row0 = (i % row_tiles) * kGRows;
    t.tok0 = (i / row_tiles) * a.tile_tokens;
    t.k0 = 0;
    t.acc = 0;
  }
  // MMA N: the tile's operand rows, a multiple of 16
  const uint32_t ntok = min(t.tile_tokens, t.T - t.tok0);
  t.n_mma = a.parts == 2 ? 2u * ((ntok + 7u) & ~7u) : ((ntok + 15u) & ~15u);
  return t;
}

template <bool kTA>
__global__ void __launch_bounds__(kGThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap bmap,
                                                            const __grid_constant__ CUtensorMap amap, const GemmArgs a) {
  using F = GemmForm<kTA>;
  const uint32_t spin = spin_or_default(a.spin);  // polls per bounded wait
  extern __shared__ uint8_t g_smem_raw[];
  // swizzled operand tiles start on 1024-byte boundaries
  uint8_t* smem = g_smem_raw + ((1024u - (smem_u32(g_smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + F::kStages * F::kABytes;
  uint8_t* sRaw = sB + F::kStages * F::kBBytes;
  __shared__ uint64_t full_a[F::kStages], full_b[F::kStages], empty_bar[F::kStages], done_bar, acc_empty, drain_bar;
  __shared__ uint64_t raw_full[F::kRawStages], raw_empty[F::kRawStages];
  __shared__ uint32_t s_tmem;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t n_tiles = a.n_tiles;
  bool failed = false;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < F::kStages; ++s) {
      mbar_init(&full_a[s], kGDqWarps / kGDqGroups + 1);  // one producer group + the B-landed relay
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    mbar_init(&acc_empty, kGDqWarps);
    mbar_init(&drain_bar, 1);
    for (uint32_t s = 0; s < F::kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kGDqWarps);  // every producer warp takes some K steps of each column
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kGTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  // Every role walks the same tiles (blockIdx.x, + gridDim.x, ...) and keeps
  // its ring counters across them: gk counts K steps, gsb raw columns, so the
  // stage phases continue from tile to tile and the copies of the next tile
  // start while this one finishes.  A tile's K steps are a multiple of 4, so
  // every tile starts at stage 0 of both rings' unrolled walks.
  if (warp == 0) {
    // B producer: one TMA box (parts x tile_tokens operand rows x 64 halves) per stage
    if (lane == 0) {
      uint32_t gk = 0;
      for (uint32_t i = blockIdx.x; i < n_tiles && !failed; i += gridDim.x) {
        const GemmTile t = gemm_tile(a, &amap, &bmap, i);
        const uint32_t b_bytes = a.parts * t.tile_tokens * F::kRowBytes;  // one B box
        for (uint32_t ks = 0; ks < t.N / F::kStageK; ++ks, ++gk) {
          const uint32_t s = gk % F::kStages, use = gk / F::kStages;
          if (use > 0 && !mbar_wait(&empty_bar[s], (use - 1) & 1u, spin)) {
            failed = true;
            break;
          }
          mbar_arrive_expect_tx(&full_b[s], b_bytes);
          tma_tile_g2s(sB + s * F::kBBytes, t.bmap, t.k0 + ks * F::kStageK, a.parts * t.tok0, &full_b[s]);
        }
      }
      // every issued copy has landed before the CTA can exit
      for (uint32_t g = (gk > F::kStages ? gk - F::kStages : 0); g < gk; ++g)
        if (!mbar_wait(&full_b[g % F::kStages], (g / F::kStages) & 1u, spin)) failed = true;
    } else if (lane == 1) {
      // relay: once a step's B copy has landed, one more arrival on the
      // stage's A barrier, so the MMA thread waits on one barrier per step.
      // A wait issued right after MMAs costs that thread about as much as
      // waiting for those MMAs to complete (measured on B200), so it waits
      // as rarely as it can.  The relay cannot fall two phases behind: the
      // copy of step gk + kStages needs the MMAs of step gk, which need this
      // arrival.
      uint32_t gk = 0;
      for (uint32_t i = blockIdx.x; i < n_tiles && !failed; i += gridDim.x) {
        const uint32_t ksteps = gemm_tile(a, &amap, &bmap, i).N / F::kStageK;
        for (uint32_t ks = 0; ks < ksteps; ++ks, ++gk) {
          const uint32_t s = gk % F::kStages;
          if (!mbar_wait(&full_b[s], (gk / F::kStages) & 1u, spin)) {
            failed = true;
            break;
          }
          mbar_arrive(&full_a[s]);
        }
      }
    }
  } else if (warp == 1) {
    // MMA issuer: per stage and 16-wide k slice, one 128 x n_mma x 16 MMA per
    // row block, both reading the same B tile
    if (lane == 0) {
      // The ring is unrolled, so each stage's operand addresses are a base
      // plus constants (descriptor address fields count 16-byte units): the
      // single issuing thread paces the pipeline at small N, and per-MMA
      // address arithmetic on its dependency chain cost ~9% at T = 64.
      const uint64_t db = smem_desc(smem_u32(sB), F::kSbo, F::kLayout);
      const uint64_t da = smem_desc(smem_u32(sA), F::kSbo, F::kLayout);
      uint32_t gk0 = 0, tcount = 0;
      for (uint32_t i = blockIdx.x; i < n_tiles && !failed; i += gridDim.x, ++tcount) {
        const GemmTile t = gemm_tile(a, &amap, &bmap, i);
        const uint32_t idesc = idesc_f16(t.n_mma), ksteps = t.N / F::kStageK;  // operand stages of the tile
        // the epilogue has read the previous tile's accumulators
        if (tcount > 0) {
          if (!mbar_wait(&acc_empty, (tcount - 1) & 1u, spin)) {
            failed = true;
            break;
          }
          tc_fence_after();
        }
        for (uint32_t ks0 = 0; ks0 < ksteps && !failed; ks0 += F::kStages) {  // ksteps % kStages == 0
          const uint32_t ph = ((gk0 + ks0) / F::kStages) & 1u;
#pragma unroll
          for (uint32_t s = 0; s < F::kStages; ++s) {
            if (!mbar_wait(&full_a[s], ph, spin)) {
              failed = true;
              break;
            }
            tc_fence_after();
            const uint32_t first = ks0 + s == 0;
#pragma unroll
            for (uint32_t kk = 0; kk < F::kStageK / 16; ++kk) {
              const uint64_t bd = db + (s * F::kBBytes + 32 * kk) / 16;
              const uint32_t acc = kk != 0 || !first;
#pragma unroll
              for (uint32_t hb = 0; hb < kGHalves; ++hb) {
                if constexpr (kTA)
                  umma_f16_ts(tmem + hb * F::kAccCols,
                              tmem + F::kACol + s * F::kAStageCols + hb * (kGK / 2) + kk * 8, bd, idesc, acc);
                else
                  umma_f16(tmem + hb * F::kAccCols, da + (s * F::kABytes + hb * F::kASub + 32 * kk) / 16, bd, idesc,
                           acc);
              }
            }
            umma_commit(&empty_bar[s]);
          }
        }
        if (!failed) umma_commit(&done_bar);  // the accumulators are final once every MMA above completes
        gk0 += ksteps;
      }
      // no MMA may still run when tensor memory is freed
      umma_commit(&drain_bar);
      if (!mbar_wait(&drain_bar, 0, spin)) failed = true;
    }
  } else if (warp < kGRawWarp) {
    // A producers, two groups of 8 warps: group p dequantizes the K steps
    // = p (mod 2), thread (warp w, lane l) tile row r = 128 b + 32 (w % 4) + l
    // with b = ((w - 2) / 4) % 2 (so that the row's lane of tensor memory is
    // in the warp's lane quarter), its 64 weights of the step (its 32-byte qs
    // group, both nibbles: low -> local k 0..31 of sub-block 2j, high -> local
    // k 32..63 of sub-block 2j+1) into row r % 128 of A block b of the
    // step's stage.  The raw super-blocks arrive by TMA, one column of the
    // tile's 256 rows per raw stage (four K steps, two per group); a step's
    // weights are computed before waiting for its A stage to be free, so only
    // the stores sit between the tensor core releasing a stage and refilling
    // it.  A warp covers 32 consecutive rows: the 8 lanes of each 16-byte
    // shared-memory store phase hit 8 different swizzled chunks.  Rows past M
    // arrive as zeros; their accumulator rows are never stored.  Waits are
    // warp-uniform (a vote), as the tensor-memory accesses are warp-wide.
    const uint32_t e = warp - 2, grp = e >> 3, q = warp & 3u, blk = (e >> 2) & 1u;
    const uint32_t rb = 32 * q + lane, r = blk * kGMmaM + rb;
    uint32_t gk0 = 0, gsb0 = 0, tcount = 0;
    for (uint32_t i = blockIdx.x; i < n_tiles && !failed; i += gridDim.x, ++tcount) {
      const GemmTile t = gemm_tile(a, &amap, &bmap, i);
      const uint32_t ksteps = t.N / kGK;
      for (uint32_t ks = grp; ks < ksteps; ks += kGDqGroups) {
        const uint32_t gsb = gsb0 + (ks >> 2), j = ks & 3u, rs = gsb % F::kRawStages;
        // the group's first K step of this column waits for the column
        if (j == grp && !__all_sync(0xffffffffu, mbar_wait(&raw_full[rs], (gsb / F::kRawStages) & 1u, spin))) {
          failed = true;
          break;
        }
        const RawGroup g = raw_group(sRaw + rs * kGRawBytes + r * kBlockBytes, j);
        if (j + kGDqGroups >= 4) {
          // the group's last K step of this column is in registers: hand it back
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
        const RowChunks ch = dequant_group(g, j);
        if constexpr (kTA) {
          const uint32_t gk = gk0 + ks, s = gk % F::kStages, use = gk / F::kStages;
          if (use > 0 && !__all_sync(0xffffffffu, mbar_wait(&empty_bar[s], (use - 1) & 1u, spin))) {
            failed = true;
            break;
          }
          tc_fence_after();  // the MMAs that read this stage have completed
          tmem_st32(tmem + ((32u * q) << 16) + F::kACol + s * F::kAStageCols + blk * (kGK / 2), ch.c);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_a[s]);
        } else {
          // the step's two K = 32 stages: low nibbles (chunks 0-3) and high
          // (chunks 4-7), 64-byte rows, 16-byte chunk c at c ^ ((row / 2) % 4)
          const uint32_t h = 2 * (gk0 + ks), s = h % F::kStages, use = h / F::kStages;
          if (use > 0 && !__all_sync(0xffffffffu, mbar_wait(&empty_bar[s], (use - 1) & 1u, spin) &&
                                                      mbar_wait(&empty_bar[s + 1], (use - 1) & 1u, spin))) {
            failed = true;
            break;
          }
          const uint32_t sw64 = (rb >> 1) & 3u;
#pragma unroll
          for (uint32_t hh = 0; hh < 2; ++hh) {
            uint8_t* dst = sA + (s + hh) * F::kABytes + blk * F::kASub + rb * F::kRowBytes;
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(dst + ((c ^ sw64) << 4)) = ch.c[4 * hh + c];
          }
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&full_a[s]);
            mbar_arrive(&full_a[s + 1]);
          }
        }
      }
      if (failed) break;
      gk0 += ksteps;  // 64-wide K steps
      gsb0 += ksteps >> 2;
      // epilogue: producer warp e reads accumulator blk (rows 128 blk ..) in
      // its tensor-memory lane quarter w % 4, the 32-column chunks of parity
      // e/8, then hands the accumulators back to the MMA thread
      if (!__all_sync(0xffffffffu, mbar_wait(&done_bar, tcount & 1u, spin))) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t half = e >> 3, ntok = min(t.tile_tokens, t.T - t.tok0);
      const uint32_t erow = t.row0 + blk * kGMmaM + 32 * q + lane;
      for (uint32_t c0 = 32 * half; c0 < t.n_mma; c0 += 32 * (kGDqWarps / 8)) {
        float v[32];
        tmem_ld32(tmem + ((32u * q) << 16) + blk * F::kAccCols + c0, v);
        if (c0 + 32 * (kGDqWarps / 8) >= t.n_mma) {
          // this warp's last accumulator chunk is in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty);
        }
        // the chunk's per-token scales: one load per lane before any store
        // (y and the scales could alias, which would order every scale load
        // after the previous store), then broadcast
        const uint32_t tl0 = a.parts == 2 ? c0 / 2 : c0;
        const float my_scale = tl0 + lane < ntok ? t.inv_scale[t.tok0 + tl0 + lane] : 0.0f;
        float* ycol = t.y + (size_t)(t.tok0 + tl0) * t.M + erow;
        if (a.parts == 2) {
#pragma unroll
          for (uint32_t u = 0; u < 16; ++u) {
            const float sc = __shfl_sync(0xffffffffu, my_scale, u);
            if (tl0 + u < ntok && erow < t.M) {
              const float r = (v[2 * u] + v[2 * u + 1]) * sc;
              if (t.acc) atomicAdd(ycol + (size_t)u * t.M, r);
              else ycol[(size_t)u * t.M] = r;
            }
          }
        } else {
#pragma unroll
          for (uint32_t u = 0; u < 32; ++u) {
            const float sc = __shfl_sync(0xffffffffu, my_scale, u);
            if (tl0 + u < ntok && erow < t.M) {
              if (t.acc) atomicAdd(ycol + (size_t)u * t.M, v[u] * sc);
              else ycol[(size_t)u * t.M] = v[u] * sc;
            }
          }
        }
      }
      if (32 * half >= t.n_mma) {
        // no chunk for this warp (n_mma <= 32): nothing held
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty);
      }
    }
  } else if (lane == 0) {
    // raw-weight copy warp: super-block column sb of the tile's 256 rows (one
    // 144-byte box per row) into raw stage gsb % (raw stages), once the
    // producers have taken the column that stage held
    uint32_t gsb = 0;
    for (uint32_t i = blockIdx.x; i < n_tiles && !failed; i += gridDim.x) {
      const GemmTile t = gemm_tile(a, &amap, &bmap, i);
      for (uint32_t sb = 0; sb < (t.N >> 8); ++sb, ++gsb) {
        const uint32_t rs = gsb % F::kRawStages, use = gsb / F::kRawStages;
        if (use > 0 && !mbar_wait(&raw_empty[rs], (use - 1) & 1u, spin)) {
          failed = true;
          break;
        }
        mbar_arrive_expect_tx(&raw_full[rs], kGRawBytes);
        tma_tile_g2s(sRaw + rs * kGRawBytes, t.amap, (t.k0 / 256 + sb) * (kBlockBytes / 4), t.row0, &raw_full[rs]);
      }
    }
    // every issued copy has landed before the CTA can exit
    for (uint32_t g = (gsb > F::kRawStages ? gsb - F::kRawStages : 0); g < gsb; ++g)
      if (!mbar_wait(&raw_full[g % F::kRawStages], (g / F::kRawStages) & 1u, spin)) failed = true;
  }
  if (failed) atomicOr(a.status, 1u);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGTmemCols) : "memory");
  }
}

// x [T][N] f32 -> B operand [parts*T][N] f16: row parts*t = hi(x_t * s_t)
// and, for parts = 2, row 2t+1 = lo = x_t*s_t - hi; s_t a power of two with
// max|x_t| * s_t < 2^15, each 8-element chunk in the A tiles' K order
// (chunk_elem).
__global__ void __launch_bounds__(256) gemm_xprep_kernel(const float* x, __half* b, float* inv_scale, uint32_t N,
                                                         uint32_t parts) {
  __shared__ float s_red[8];
  const uint32_t t = blockIdx.x;
  const float* xr = x + (size_t)t * N;
  float mx = 0.0f;
  for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) mx = fmaxf(mx, fabsf(xr[k]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  int e = 0, sexp = 0;
  if (mx > 0.0f && mx <= 3.402823466e38f) {
    frexpf(mx, &e);
    sexp = 15 - e;
    sexp = sexp > 100 ? 100 : (sexp < -100 ? -100 : sexp);
  }
  const float s = ldexpf(1.0f, sexp);
  if (threadIdx.x == 0) inv_scale[t] = ldexpf(1.0f, -sexp);
  __half* hi = b + (size_t)(parts * t) * N;
  __half* lo = hi + N;
  for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) {
    const float v = xr[(k & ~7u) | chunk_elem(k & 7u)] * s;  // the A tiles' K order
    const __half hv = __float2half_rn(v);
    hi[k] = hv;
    if (parts == 2) lo[k] = __float2half_rn(v - __half2float(hv));
  }
}

// The same for the jobs of a multi-matrix launch: CTA j*T + t prepares
// token t of job j (x, or gelu_mul of gate and up, stored to act on the way).
__global__ void __launch_bounds__(256) gemm_prep_kernel(const GemmJob* jobs, uint32_t T, uint32_t parts) {
  __shared__ float s_red[8];
  const GemmJob J = jobs[blockIdx.x / T];
  const uint32_t t = blockIdx.x % T, N = J.N;
  if (J.mode == 2) {  // a K-split output row, to be accumulated into
    for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) J.act[(size_t)t * N + k] = 0.0f;
    return;
  }
  const size_t base = (size_t)t * N;
  auto value = [&](size_t i) { return J.mode ? gelu_mul_value(J.gate[i], J.up[i]) : J.x[i]; };  // modes 0, 1
  float mx = 0.0f;
  for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) {
    const float v = value(base + k);
    if (J.mode && J.act) J.act[base + k] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  int e = 0, sexp = 0;
  if (mx > 0.0f && mx <= 3.402823466e38f) {
    frexpf(mx, &e);
    sexp = 15 - e;
    sexp = sexp > 100 ? 100 : (sexp < -100 ? -100 : sexp);
  }
  const float sc = ldexpf(1.0f, sexp);
  if (threadIdx.x == 0) J.inv_scale[t] = ldexpf(1.0f, -sexp);
  __half* hi = static_cast<__half*>(J.operand) + (size_t)(parts * t) * N;
  __half* lo = hi + N;
  for (uint32_t k = threadIdx.x; k < N; k += blockDim.x) {
    const float v = value(base + ((k & ~7u) | chunk_elem(k & 7u))) * sc;  // the A tiles' K order
    const __half hv = __float2half_rn(v);
    hi[k] = hv;
    if (parts == 2) lo[k] = __float2half_rn(v - __half2float(hv));
  }
}

// The same with the token's row staged in shared memory (N floats), so the
// inputs are read once: 16-byte loads of x, or of gate and up (gelu_mul
// computed once and stored to act on the way), the row's max |value|, then
// each 8-element chunk scaled and written as one 16-byte store per operand
// row.  Every pointer of every job is 16-byte aligned (checked by the host).
__global__ void __launch_bounds__(256) gemm_prep_row_kernel(const GemmJob* jobs, uint32_t T, uint32_t parts) {
  extern __shared__ float4 s_row4[];
  __shared__ float s_red[8];
  const GemmJob J = jobs[blockIdx.x / T];
  const uint32_t t = blockIdx.x % T, n4 = J.N / 4;
  const size_t base4 = (size_t)t * n4;
  if (J.mode == 2) {  // a K-split output row, to be accumulated into
    for (uint32_t k = threadIdx.x; k < J.N; k += blockDim.x) J.act[(size_t)t * J.N + k] = 0.0f;
    return;
  }
  float mx = 0.0f;
  for (uint32_t k = threadIdx.x; k < n4; k += blockDim.x) {
    float4 v;
    if (J.mode) {
      const float4 g = reinterpret_cast<const float4*>(J.gate)[base4 + k];
      const float4 u = reinterpret_cast<const float4*>(J.up)[base4 + k];
      v = make_float4(gelu_mul_value(g.x, u.x), gelu_mul_value(g.y, u.y), gelu_mul_value(g.z, u.z),
                      gelu_mul_value(g.w, u.w));
      if (J.act) reinterpret_cast<float4*>(J.act)[base4 + k] = v;
    } else {
      v = reinterpret_cast<const float4*>(J.x)[base4 + k];
    }
    s_row4[k] = v;
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = s_red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, s_red[i]);
  int e = 0, sexp = 0;
  if (mx > 0.0f && mx <= 3.402823466e38f) {
    frexpf(mx, &e);
    sexp = 15 - e;
    sexp = sexp > 100 ? 100 : (sexp < -100 ? -100 : sexp);
  }
  const float sc = ldexpf(1.0f, sexp);
  if (threadIdx.x == 0) J.inv_scale[t] = ldexpf(1.0f, -sexp);
  const float* s_row = reinterpret_cast<const float*>(s_row4);
  __half* const op = static_cast<__half*>(J.operand) + (size_t)(parts * t) * J.N;
  for (uint32_t c = threadIdx.x; c < J.N / 8; c += blockDim.x) {
    uint32_t h[4], l[4];
#pragma unroll
    for (uint32_t q = 0; q < 4; ++q) {
      // positions 2q, 2q+1 of the chunk in the A tiles' K order
      const float v0 = s_row[8 * c + chunk_elem(2 * q)] * sc, v1 = s_row[8 * c + chunk_elem(2 * q + 1)] * sc;
      const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      h[q] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
      l[q] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    reinterpret_cast<uint4*>(op)[c] = make_uint4(h[0], h[1], h[2], h[3]);
    if (parts == 2) reinterpret_cast<uint4*>(op + J.N)[c] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

constexpr size_t kGemmPrepRowMax = 96 * 1024;  // widest row the single-read preparation stages in shared memory

EncodeTiledFn gemm_encode_fn() {
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

// One launch of the form that a tile of parts x tile_tokens operand rows uses.
template <bool kTA>
cudaError_t launch_form(uint32_t grid, const CUtensorMap& bmap, const CUtensorMap& amap, const GemmArgs& ga,
                        int device, cudaStream_t s) {
  static std::atomic<uint8_t> attr_set[kAttrDevices];
  const cudaError_t e = smem_attr_once(attr_set, device, gemm_kernel<kTA>, (int)GemmForm<kTA>::kSmem);
  if (e != cudaSuccess) return e;
  gemm_kernel<kTA><<<grid, kGThreads, GemmForm<kTA>::kSmem, s>>>(bmap, amap, ga);
  return cudaGetLastError();
}

// Persistent: one CTA per SM (at most one per tile), each walking its tiles.
cudaError_t launch_gemm_kernel(const CUtensorMap& bmap, const CUtensorMap& amap, const GemmArgs& ga, uint32_t sms,
                               int device, cudaStream_t s) {
  const uint32_t grid = ga.n_tiles < sms ? ga.n_tiles : sms;
  return ga.parts * ga.tile_tokens <= kGMaxTsRows ? launch_form<true>(grid, bmap, amap, ga, device, s)
                                                  : launch_form<false>(grid, bmap, amap, ga, device, s);
}

// The B operand's tensor map for tiles of `box_rows` operand rows: K = 64
// boxes in the 128-byte swizzle (TS form) or K = 32 in the 64-byte swizzle
// (SS form), matching the form's shared-memory stages.
CUresult encode_operand_map(EncodeTiledFn enc, CUtensorMap* map, const void* operand, uint32_t N, uint32_t rows,
                            uint32_t box_rows) {
  const bool ts = box_rows <= kGMaxTsRows;
  const cuuint64_t dims[2] = {N, rows};
  const cuuint64_t strides[1] = {2ull * N};
  const cuuint32_t box[2] = {ts ? GemmForm<true>::kStageK : GemmForm<false>::kStageK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(operand), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, ts ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace

int run_gemm(q4k_ctx* ctx, const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
             cudaStream_t s, uint32_t parts) {
  if (parts != 1 && parts != 2) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "parts=%u must be 1 or 2", parts);
  EncodeTiledFn enc = gemm_encode_fn();
  if (!enc) return ctx_fail(ctx, Q4K_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  // activation rows per pass: the B operand (4 bytes per element per row)
  // and the per-row scales fit the context scratch
  uint32_t cap = (uint32_t)(ctx->xfrag_cap / (4ull * N));
  cap = cap > kCtxScaleSlots ? kCtxScaleSlots : cap;
  cap -= cap % kGTokens;
  if (cap == 0) return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "N=%u too large for the GEMM scratch", N);
  __half* bbuf = reinterpret_cast<__half*>(ctx->xfrag);
  // the raw Q4_K matrix as [M rows][N/256*36 words], read in boxes of one
  // super-block (36 words) x 256 rows; rows past M read as zeros
  CUtensorMap amap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(N / 256) * (kBlockBytes / 4), M};
    const cuuint64_t strides[1] = {(cuuint64_t)(N / 256) * kBlockBytes};
    const cuuint32_t box[2] = {kBlockBytes / 4, kGRows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&amap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return ctx_fail(ctx, Q4K_ERR_CUDA, "q4k_gemm weight tensor map");
  }
  for (uint32_t done = 0; done < T;) {
    const uint32_t tc = (T - done) < cap ? (T - done) : cap;
    gemm_xprep_kernel<<<tc, 256, 0, s>>>(x + (size_t)done * N, bbuf, ctx->inv_scale, N, parts);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemm activation prep launch");
    // tiles of 256 operand rows (kGTokens x 2 / parts activation rows), or
    // half that when the full ones would fill at most a quarter of the SMs
    // and the smaller tiles still fit in one wave.  Every activation tile
    // reconstructs its rows' weights again, so larger tiles do less work in
    // total; with several matrices in flight on other streams (config 4)
    // that outweighs the idle SMs of a single call.
    const uint32_t row_tiles = (M + kGRows - 1) / kGRows;
    const uint32_t sms = (uint32_t)ctx->sm_count;
    const uint32_t full = 2 * kGTokens / parts, half = full / 2;
    uint32_t tile =
        (row_tiles * ((tc + full - 1) / full) * 4 <= sms && row_tiles * ((tc + half - 1) / half) <= sms) ? half
                                                                                                        : full;
    // a batch that fits one TS tile runs as one
    if (tile == full && gemm_tile_tokens(parts, tc) * parts <= kGMaxTsRows) tile = gemm_tile_tokens(parts, tc);
    CUtensorMap bmap;
    if (encode_operand_map(enc, &bmap, bbuf, N, parts * tc, parts * tile) != CUDA_SUCCESS)
      return ctx_fail(ctx, Q4K_ERR_CUDA, "q4k_gemm activation tensor map");
    GemmArgs ga;
    ga.w = w;
    ga.y = y + (size_t)done * M;
    ga.inv_scale = ctx->inv_scale;
    ga.M = M;
    ga.N = N;
    ga.T = tc;
    ga.tile_tokens = tile;
    ga.parts = parts;
    ga.status = ctx->select.status;
    ga.spin = ctx->select.spin_limit;
    ga.tasks = nullptr;
    ga.tiles = nullptr;
    ga.n_tiles = row_tiles * ((tc + ga.tile_tokens - 1) / ga.tile_tokens);
    e = launch_gemm_kernel(bmap, amap, ga, sms, ctx->device, s);
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_gemm launch");
    done += tc;
  }
  ctx->err[0] = 0;
  return Q4K_OK;
}

uint32_t gemm_tile_tokens(uint32_t parts, uint32_t T) {
  // the MMA's N (parts x activation rows) is a multiple of 16
  const uint32_t t = parts == 2 ? (T + 7u) & ~7u : (T + 15u) & ~15u;
  return parts * t <= kGMaxTsRows ? t : 2 * kGTokens / parts;
}

uint32_t gemm_tile_rows() { return kGRows; }

size_t gemm_operand_bytes(uint32_t N, uint32_t T, uint32_t parts) { return (size_t)2 * parts * T * N; }

cudaError_t gemm_weight_map(CUtensorMap* map, const void* w, uint32_t M, uint32_t N) {
  EncodeTiledFn enc = gemm_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {(cuuint64_t)(N / 256) * (kBlockBytes / 4), M};
  const cuuint64_t strides[1] = {(cuuint64_t)(N / 256) * kBlockBytes};
  const cuuint32_t box[2] = {kBlockBytes / 4, kGRows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

cudaError_t gemm_operand_map(CUtensorMap* map, const void* operand, uint32_t N, uint32_t T, uint32_t parts) {
  EncodeTiledFn enc = gemm_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  return encode_operand_map(enc, map, operand, N, parts * T, parts * gemm_tile_tokens(parts, T)) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

cudaError_t launch_gemm_prep(const GemmJob* jobs, uint32_t n_jobs, uint32_t T, uint32_t parts, uint32_t max_n,
                             bool aligned, int device, cudaStream_t s) {
  if (n_jobs == 0) return cudaSuccess;
  const size_t row_bytes = 4ull * max_n;
  if (aligned && row_bytes <= kGemmPrepRowMax) {
    static std::atomic<uint8_t> attr_set[kAttrDevices];
    const cudaError_t e = smem_attr_once(attr_set, device, gemm_prep_row_kernel, (int)kGemmPrepRowMax);
    if (e != cudaSuccess) return e;
    gemm_prep_row_kernel<<<n_jobs * T, 256, row_bytes, s>>>(jobs, T, parts);
  } else {
    gemm_prep_kernel<<<n_jobs * T, 256, 0, s>>>(jobs, T, parts);
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_tasks(const GemmTask* tasks, const uint2* tiles, uint32_t n_tiles, uint32_t parts,
                              uint32_t tile_tokens, uint32_t sms, int device, uint32_t* status, uint32_t spin,
                              cudaStream_t s) {
  if (n_tiles == 0) return cudaSuccess;
  GemmArgs ga{};
  ga.parts = parts;
  ga.tile_tokens = tile_tokens;  // selects the form; each task carries its own
  ga.status = status;
  ga.spin = spin;
  ga.tasks = tasks;
  ga.tiles = tiles;
  ga.n_tiles = n_tiles;
  const CUtensorMap unused{};
  return launch_gemm_kernel(unused, unused, ga, sms, device, s);
}

}  // namespace q4k
