// The Q4_K GEMV engine: task and activation-preparation descriptors shared by
// the engine kernels (q4k_engine.cu), the single-call entry points and plans.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_kernels.cuh"

namespace q4k {

constexpr int kTileRows = 16;       // output rows per work item (one m16 MMA tile)
constexpr int kEngineWarps = 8;     // warps per engine CTA
constexpr int kMaxTokens = 16;      // activation rows per GEMV (4 per n-tile, 4 n-tiles)

// Prepared activation ("x fragments"): x of each token, scaled by a power of
// two so max|x| < 2^15 and split exactly into f16 hi + f16 lo
// (x*s = hi + lo + O(2^-22 |x*s|)), stored in the per-lane order of the
// m16n8k16 B operand.  Column n = 2*(token%4) + part of n-tile token/4.
// Layout: uint2 [n_tiles][N/256 blocks][16 k-steps][32 lanes].
inline size_t xfrag_bytes(uint32_t N, uint32_t batch) {
  const uint32_t nt = (batch + 3) / 4;
  return (size_t)nt * N * 16;
}

enum TaskKind : uint32_t { kTaskPlain = 0, kTaskSelect = 1 };

// One GEMV of an engine launch: y[t*M + m] = sum_k w16[m,k] * x[t,k].
struct EngineTask {
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
  uint32_t kind;
  uint32_t row_offset;      // kTaskSelect: global index of row 0
  float cap;                // kTaskSelect: softcap (<= 0: none)
  uint32_t pad_;
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
struct TaskList {
  const EngineTask* dev;
  EngineTask inl;
  uint32_t n;
  uint32_t total_items;
};

struct JobList {
  const XJob* dev;
  XJob inl;
  uint32_t n;
};

cudaError_t launch_xprep(const JobList& jobs, uint32_t batch, cudaStream_t s);
cudaError_t launch_engine(const TaskList& tasks, uint32_t batch, bool has_select, const SelectScratch& sel,
                          int sm_count, cudaStream_t s);

}  // namespace q4k
