// q4k_lmhead_select_static: the fused LM head without any allocation.
//
// Some callers cannot call cudaMalloc (or anything that does): real-time
// decode loops that must never enter the driver's allocator (an allocation
// can block on device-wide synchronization), and embedders whose device
// memory is owned and budgeted by another runtime and who therefore cannot
// create a q4k_ctx (q4k_create allocates the context's scratch).  For them
// this file keeps the LM head's scratch -- the prepared activation, its
// scale, the 256 per-residue selection keys, the completion counter and the
// status word -- in one file-scope device array of fixed size, present on
// every GPU that loads libq4k.so until the process exits.  The caller still
// passes and owns the weights, the input and every output buffer.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "q4k_ctx.cuh"

using namespace q4k;

namespace {

// Largest reduction dimension (row length) the static scratch serves.
constexpr uint32_t kStaticMaxN = 16384;
constexpr size_t kSelBytes = 256 * sizeof(unsigned long long);  // selection keys
constexpr size_t kWordsBytes = 256;                              // counter, status
constexpr size_t kScaleBytes = 256;                              // 1/scale of the activation
constexpr size_t kXfragOff = kSelBytes + kWordsBytes + kScaleBytes;
constexpr size_t kStaticScratchBytes = kXfragOff + 4 * (size_t)kStaticMaxN;  // 67,328 bytes

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the array on the current device (host code only sees a
// stand-in symbol, never a device address).  Looked up once per device.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int q4k_lmhead_select_static(const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                                        uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx,
                                        uint32_t* argmax, void* stream) {
  if (!w || !x || !cand_val || !cand_idx || !argmax) return Q4K_ERR_INVALID_ARG;
  if (N == 0 || N % Q4K_QK != 0 || V == 0) return Q4K_ERR_INVALID_ARG;
  if (N > kStaticMaxN) return Q4K_ERR_SCRATCH_LIMIT;
  if ((uint64_t)row_offset + V >= (1ull << 31)) return Q4K_ERR_INVALID_ARG;
  if (!aligned16(w) || !aligned16(x) || (logits && !aligned16(logits))) return Q4K_ERR_INVALID_ARG;

  void* base = nullptr;
  if (scratch_address(&base) != cudaSuccess) return Q4K_ERR_CUDA;
  char* b = static_cast<char*>(base);
  SelectScratch sel;
  sel.slots = reinterpret_cast<unsigned long long*>(b);
  sel.counter = reinterpret_cast<uint32_t*>(b + kSelBytes);
  sel.status = reinterpret_cast<uint32_t*>(b + kSelBytes + 4);
  float* inv_scale = reinterpret_cast<float*>(b + kSelBytes + kWordsBytes);
  uint2* xfrag = reinterpret_cast<uint2*>(b + kXfragOff);

  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return Q4K_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap map;
  uint32_t tile_bytes = 0;
  if (encode_weight_map(&map, w, V, N, &tile_bytes) != cudaSuccess) return Q4K_ERR_CUDA;

  // The array keeps the previous call's contents: put the selection keys
  // and the counter back to their starting values before this call.  The
  // status word is left alone: a bounded wait that expired in an earlier
  // call stays recorded until q4k_check_static reads and clears it.
  if (init_select_scratch(sel, s, false) != cudaSuccess) return Q4K_ERR_CUDA;
  JobList jl{};
  jl.n = 1;
  jl.inl.x = x;
  jl.inl.xfrag = xfrag;
  jl.inl.inv_scale = inv_scale;
  jl.inl.N = N;
  const bool prep = xfrag_bytes(N, 1) <= engine_xcache_bytes(true);
  if (!prep && launch_xprep(jl, 1, s) != cudaSuccess) return Q4K_ERR_CUDA;
  TaskList tl{};
  tl.prep = prep ? 1u : 0u;
  tl.inl_job = jl.inl;
  tl.n = 1;
  tl.inl.w = static_cast<const uint8_t*>(w);
  tl.inl.xfrag = xfrag;
  tl.inl.inv_scale = inv_scale;
  tl.inl.logits = logits;
  tl.inl.cand_val = cand_val;
  tl.inl.cand_idx = cand_idx;
  tl.inl.argmax = argmax;
  tl.inl.M = V;
  tl.inl.N = N;
  tl.inl.item_begin = 0;
  tl.inl.item_end = tiles_of(V);
  tl.inl.kind = kTaskSelect;
  tl.inl.row_offset = row_offset;
  tl.inl.cap = cap;
  tl.inl.tile_bytes = tile_bytes;
  tl.total_items = tiles_of(V);
  tl.total_cost = tiles_of(V) * (N / Q4K_QK);
  tl.pairs = pairs_of(N, 0, tile_bytes) ? 1u : 0u;
  if (launch_engine(tl, map, 1, true, sel, sms, s) != cudaSuccess) return Q4K_ERR_CUDA;
  return Q4K_OK;
}

extern "C" int q4k_check_static(void) {
  // The status word sits at a fixed offset of the array; it is read and
  // cleared by symbol, so no device address or allocation is involved.
  constexpr size_t kStatusOff = kSelBytes + 4;
  if (cudaDeviceSynchronize() != cudaSuccess) return Q4K_ERR_CUDA;
  uint32_t status = 0;
  if (cudaMemcpyFromSymbol(&status, g_static_scratch, sizeof(status), kStatusOff) != cudaSuccess)
    return Q4K_ERR_CUDA;
  if (status == 0) return Q4K_OK;
  const uint32_t zero = 0;
  if (cudaMemcpyToSymbol(g_static_scratch, &zero, sizeof(zero), kStatusOff) != cudaSuccess) return Q4K_ERR_CUDA;
  return Q4K_ERR_TIMEOUT;
}
