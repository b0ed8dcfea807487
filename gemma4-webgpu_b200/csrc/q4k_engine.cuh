// The Q4_K GEMV engine: task and activation-preparation descriptors shared by
// the engine kernels (q4k_engine.cu), the single-call entry points and plans.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_kernels.cuh"

namespace q4k {

constexpr int kTileRows = 16;       // output rows per work item (one m16 MMA tile)
constexpr int kEngineWarps = 16;    // warps per engine CTA (one CTA per SM)
constexpr int kMaxTokens = 16;      // activation rows per GEMV (4 per n-tile, 4 n-tiles)

// Prepared activation ("x fragments"): x of each token, scaled by a power of
// two so max|x| < 2^15 and split exactly into f16 hi + f16 lo
// (x*s = hi + lo + O(2^-22 |x*s|)), stored in the per-lane order of the
// m16n8k16 B operand: n-tile nt holds tokens 4nt..4nt+3, column
// 2*(token%4) + part (part 0 = hi, 1 = lo).  Only the columns of existing
// tokens are stored: n-tile nt with cols_nt = 2*min(4, batch-4nt) columns is
// uint4 [N/256 blocks][8 words][cols_nt][4], each uint4 holding the lane's
// fragments of k-steps w and w+8 (low- and high-nibble MMAs of word w),
// n-tiles back to back.  4 bytes per element per token in total.
__host__ __device__ inline size_t xfrag_bytes(uint32_t N, uint32_t batch) { return (size_t)4 * N * batch; }

enum TaskKind : uint32_t { kTaskPlain = 0, kTaskSelect = 1 };

// Weight format of every task of an engine launch: Q4_K as GGUF stores it,
// or Q6_K in the device layout of q6k_dequant.cuh.
enum WeightFormat : uint32_t { kFmtQ4K = 0, kFmtQ6K = 1 };

// One GEMV of an engine launch: y[t*M + m] = sum_k w16[m,k] * x[t,k].
struct alignas(16) EngineTask {
  const uint8_t* w;         // Q4_K [M][N/256*144]
  const uint2* xfrag;       // prepared activations (see above)
  const float* inv_scale;   // [batch]: 1/s per token
  float* y;                 // kTaskPlain: [batch][M]
  float* logits;            // kTaskSelect: optional softcapped logits [M]
  float* cand_val;          // kTaskSelect: [256]
  uint32_t* cand_idx;       // kTaskSelect: [256]
  uint32_t* argmax;         // kTaskSelect: [1]
  uint32_t M, N;
  uint32_t item_begin, item_end;  // work items [begin, end) = 16-row tiles
  uint32_t cost_begin;            // sum of items * (N/256) over earlier tasks
  uint32_t kind;
  uint32_t row_offset;      // kTaskSelect: global index of row 0
  float cap;                // kTaskSelect: softcap (<= 0: none)
  const CUtensorMap* tmap;  // TMA map of w (device memory; Q6_K: the body map, the d-plane map
                            // follows it); null: the launch's own map(s)
  uint32_t tile_bytes;      // bytes per tile row in a weight stage (the map's box width)
  uint32_t aux;             // host-side bookkeeping while a plan is laid out
};
static_assert(sizeof(EngineTask) == 112, "EngineTask must stay a multiple of 16 bytes");

constexpr int kMaxCachedX = 8;     // distinct prepared activations one CTA keeps in shared memory
constexpr int kMaxCtaTasks = 64;   // task descriptors one CTA keeps in shared memory

// One CTA's share of an engine launch, computed on the host when a plan is
// committed: its item range, the tasks that range touches, and the prepared
// activations it stages in shared memory (offsets into its activation cache).
struct CtaSched {
  uint32_t c0, c1;   // work items [c0, c1)
  uint32_t t0, nt;   // tasks [t0, t0+nt) (nt = 0: read tasks from global memory)
  uint32_t nx;       // activations to stage
  uint32_t xoff[kMaxCachedX];
  uint32_t xbytes[kMaxCachedX];
  const uint2* xptr[kMaxCachedX];  // the tasks' xfrag pointer each slot stands for
  uint32_t xjob[kMaxCachedX];      // prepare-in-engine launches: the job of each slot
  uint32_t act_mask;               // bit j: this CTA stores slot j's gelu_mul output
};

// One activation to prepare: mode 0 reads x, mode 1 computes
// gelu_tanh(gate) * up (shaders/gelu_mul.wgsl) and optionally stores it.
struct XJob {
  const float* x;
  const float* gate;
  const float* up;
  float* act;
  uint2* xfrag;
  float* inv_scale;
  uint32_t N;
  uint32_t mode;
};

// Tasks / jobs either live in device memory (plans) or are passed inline as
// kernel parameters (single calls).
// Candidate exchange of a vocabulary-sharded LM head (q4k_exchange): every
// rank owns a mailbox of 2 x kMaxRanks slots in its own device memory; the
// last CTA of a rank's LM-head launch for call epoch e writes its 256
// candidates into slot (rank, e & 1) of every rank's mailbox (peer stores
// over NVLink), raises that slot's flag to e, waits (bounded) until the
// (q, e & 1) slots of all `world` senders q in its own mailbox carry e, and
// merges them.  Two slots per sender, alternating by epoch parity, keep a
// fast rank's next call from overwriting candidates a slower rank is still
// merging.
constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kSlotWords = 576;      // 256 values, 256 indices, flag at word 512; 2304 bytes
constexpr uint32_t kSlotFlag = 512;
constexpr uint32_t kMailboxSlots = 2 * kMaxRanks;
constexpr uint32_t kMailboxEpochWord = kMailboxSlots * kSlotWords;  // this rank's call counter

// Word offset of sender q's slot for epoch parity `par` in a mailbox.
__host__ __device__ inline uint32_t mailbox_slot(uint32_t q, uint32_t par) { return (2u * q + par) * kSlotWords; }

struct Exchange {
  uint32_t* peer[kMaxRanks];  // mailbox of each rank as mapped on this device (peer[rank] = own)
  uint32_t* epoch;            // this rank's call counter (own device memory)
  uint32_t rank, world;       // world = 0: no exchange
};

// prep != 0: every CTA prepares the activations of its task range itself,
// straight into its shared-memory cache (from `jobs`, or `inl_job` for an
// inline task), so no preparation launch precedes the engine; the host
// chooses this only when every task's activation fits each CTA's cache.
struct TaskList {
  const EngineTask* dev;
  const CtaSched* sched;  // per-CTA schedule of a device task list (grid entries)
  const XJob* jobs;       // device job table (prep with a device task list)
  EngineTask inl;
  XJob inl_job;
  uint32_t prep;
  uint32_t n;
  uint32_t total_items;
  uint32_t total_cost;  // sum of item_cost over the work items of the launch
  uint32_t grid;        // CTAs the schedule was made for
  uint32_t select_task; // index of the kTaskSelect task, if the launch has one
  uint32_t ksplit;      // > 1: KS warps share each tile, one K slice each (plain tasks, batch <= 4,
                        // every task's N/256 a multiple of KS; Q4_K only)
  uint32_t fmt;         // WeightFormat of every task
  uint32_t pairs;       // 1: every warp's super-block range has an even length and every tile row
                        // is kPairTileBytes (Q4_K only; see pairs_of)
  Exchange xc;          // LM-head candidate exchange across ranks (xc.world > 0)
};

// Bytes per tile row of a two-super-block Q4_K stage (the box of
// encode_weight_map: 2 x 144 bytes + 16).
constexpr uint32_t kPairTileBytes = 304;

// Whether a Q4_K task of N columns, split over ks warps (0 or 1: no split),
// always fills both super-blocks of its stages from tile rows of
// kPairTileBytes: launches whose tasks all do run a kernel with the
// per-stage block count and row pitch fixed at compile time.
__host__ __device__ inline bool pairs_of(uint32_t N, uint32_t ks, uint32_t tile_bytes) {
  const uint32_t nb = N >> 8, k = ks > 1 ? ks : 1u;
  return nb % k == 0 && (nb / k) % 2 == 0 && tile_bytes == kPairTileBytes;
}

struct JobList {
  const XJob* dev;
  XJob inl;
  uint32_t n;
};

// The weight matrix as a 2-D TMA tensor of 32-bit words, [M rows][N/256*36
// words], read in boxes of 16 rows x 2 super-blocks (+16 bytes, so tile rows
// sit 304 bytes apart in shared memory and the lanes' 16-byte reads of 8
// rows fall in distinct banks).  Rows past M and words past the row end
// read as zeros.  *tile_bytes = the box width in bytes.
cudaError_t encode_weight_map(CUtensorMap* map, const void* w, uint32_t M, uint32_t N, uint32_t* tile_bytes);

// A Q6_K matrix in the device layout as two TMA tensors: maps[0] the bodies
// as 32-bit words [M rows][N/256*52 words], read in boxes of 16 rows x one
// 208-byte body; maps[1] the d plane as f16 [N/256][Mp], read in boxes of
// 16 rows of one super-block column.  *tile_bytes = 208.
cudaError_t encode_q6k_maps(CUtensorMap* maps, const void* w, uint32_t M, uint32_t N, uint32_t* tile_bytes);

// Schedule cost of one work item (16 rows) of a task: its super-blocks per
// row.  LM-head items (softcap + per-residue selection in the epilogue) cost
// the same: with them weighted 5 % above plain items, a per-CTA trace of
// the decode step's first launch showed the CTAs holding LM-head items
// finishing ~5 % before the others.
__host__ __device__ inline uint32_t item_cost(uint32_t N, uint32_t kind) {
  (void)kind;
  return N >> 8;
}

// Engine launch geometry: CTAs for a work list, and the shared-memory
// activation cache each CTA has (depends on whether an LM head is present).
uint32_t engine_grid(uint32_t total_items, int sm_count);
uint32_t engine_xcache_bytes(bool has_select, uint32_t fmt = kFmtQ4K);

// Host-side schedule of a device task list (tasks sorted by item_begin):
// equal shares of super-blocks per CTA, and what each CTA stages.
void engine_schedule(const EngineTask* tasks, uint32_t n, uint32_t total_cost, uint32_t total_items,
                     uint32_t batch, uint32_t grid, uint32_t xcache_bytes, CtaSched* out);

// Whether every CTA of a schedule caches the activation of every task in its
// range (the condition for preparing activations in the engine).
bool schedule_covers_tasks(const EngineTask* tasks, uint32_t n, const CtaSched* sched, uint32_t grid);

cudaError_t launch_xprep(const JobList& jobs, uint32_t batch, cudaStream_t s);
// `map` (and for Q6_K `dmap`, the d-plane map): the weight maps of an inline
// task (tasks.dev == null); ignored for device task lists, whose tasks carry
// their own maps.
cudaError_t launch_engine(const TaskList& tasks, const CUtensorMap& map, uint32_t batch, bool has_select,
                          const SelectScratch& sel, int sm_count, cudaStream_t s, const CUtensorMap* dmap = nullptr);

}  // namespace q4k
