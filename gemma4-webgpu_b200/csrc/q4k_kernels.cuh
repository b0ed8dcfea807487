// Host-side launchers of the Q4_K kernels (internal to libq4k.so).  Each
// returns the cudaError_t of its launch; argument validation happens in the
// C-ABI layer (q4k_abi.cu) before these are called.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace q4k {

// Raises a kernel's dynamic shared-memory limit once per device.  `done` is
// the kernel's own per-device flag table; a flag is set only after the call
// succeeded, and two host threads that both see it unset both make the
// (idempotent) call, so threads driving different devices never skip it.
constexpr int kAttrDevices = 64;

// Default polls per bounded wait in the kernels (mbarrier and peer-flag
// waits); a context may set its own (q4k_set_wait_limit).
constexpr uint32_t kSpinLimit = 1u << 22;

template <typename K>
inline cudaError_t smem_attr_once(std::atomic<uint8_t> (&done)[kAttrDevices], int dev, K* kernel, int bytes) {
  if (dev >= 0 && dev < kAttrDevices && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < kAttrDevices) done[dev].store(1, std::memory_order_release);
  return e;
}

// Scratch of the fused LM head: 256 64-bit order keys (one per residue) and a
// completion counter.  Between calls the keys hold the empty candidate
// (-1e30, 0) and the counter is 0; the last CTA of every call restores that.
struct SelectScratch {
  unsigned long long* slots = nullptr;  // [256]
  uint32_t* counter = nullptr;          // [1]
  uint32_t* status = nullptr;           // [1] nonzero: a kernel gave up a bounded wait
  uint32_t spin_limit = 0;              // polls per bounded wait (0: kSpinLimit, q4k_ptx.cuh)
};

constexpr size_t kSelectScratchBytes = 256 * sizeof(unsigned long long) + 256;

// Writes the between-calls state (empty keys, counter 0) into the scratch;
// clear_status also zeroes the status word (a fresh scratch).
cudaError_t init_select_scratch(const SelectScratch& sc, cudaStream_t s, bool clear_status = true);

// y[b*ldy + m] = sum_k w16(m,k) * x[b*ldx + k] for b < batch, m < M.
// The scratch-free CUDA-core kernel (one warp per row); the engine
// (q4k_engine.cuh) is the fast path.
cudaError_t launch_gemv(const uint8_t* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
                        uint32_t ldx, uint32_t ldy, int variant, cudaStream_t s);

// Q4_K blocks -> f16 bit patterns of the reference weights.
cudaError_t launch_dequant_f16(const uint8_t* w, uint16_t* out, uint64_t n_blocks, cudaStream_t s);

cudaError_t launch_softcap(float* logits, uint32_t n, float cap, cudaStream_t s);
cudaError_t launch_argmax(const float* logits, uint32_t n, uint32_t* result, cudaStream_t s);
cudaError_t launch_topk256(const float* logits, uint32_t n, float* result512, cudaStream_t s);
cudaError_t launch_gelu_mul(const float* gate, const float* up, float* out, uint32_t n, cudaStream_t s);

// Softcap (cap > 0) + per-residue candidates + argmax of B <= kMaxSelectRows
// rows of n logits in one launch, over the row scratch (slots [rows][256],
// counters [rows]) that init_row_slots prepares.
constexpr uint32_t kMaxSelectRows = 16;
cudaError_t init_row_slots(unsigned long long* slots, uint32_t* counters, uint32_t rows, cudaStream_t s);
cudaError_t launch_select_rows(float* logits, uint32_t B, uint32_t n, float cap, unsigned long long* slots,
                               uint32_t* counters, float* cand_val, uint32_t* cand_idx, uint32_t* argmax, int sms,
                               cudaStream_t s);

// Merge G ranks' candidate sets ([G][256] each, rank-major) into one.
cudaError_t launch_merge_candidates(const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                                    uint32_t* out_idx, uint32_t* argmax, cudaStream_t s);

}  // namespace q4k
