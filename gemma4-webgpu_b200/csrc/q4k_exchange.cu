// Vocabulary-sharded LM head with the candidate exchange fused into the
// head's launch (no collective library call): the mailboxes of
// q4k_engine.cuh's Exchange, mapped across the ranks' GPUs with CUDA IPC,
// and the entry point that runs a rank's shard.
//
// The reference runs its LM head on one device (src/engine.ts:1686-1741);
// this is its vocabulary-parallel form, equal in outputs to the unsharded
// head (rows are independent; the topk256/argmax selection reduces per
// residue class, shaders/topk256.wgsl:5-21, argmax.wgsl:7-34).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "q4k_ctx.cuh"

using namespace q4k;

struct q4k_exchange {
  q4k_ctx* ctx = nullptr;
  uint32_t rank = 0, world = 0;
  uint32_t* mailbox = nullptr;          // own: kMailboxSlots slots + the epoch word
  uint32_t* peer[kMaxRanks] = {nullptr};  // mapped peer mailboxes (peer[rank] = mailbox)
  bool opened[kMaxRanks] = {false};
  bool ipc[kMaxRanks] = {false};        // peer mapped through CUDA IPC (closed on destroy)
};

namespace {
constexpr size_t kMailboxBytes = (size_t)kMailboxEpochWord * 4 + 256;
}

extern "C" {

int q4k_exchange_create(q4k_ctx* ctx, uint32_t rank, uint32_t world, q4k_exchange** out, void* handle_out) {
  if (!ctx || !out || !handle_out) return Q4K_ERR_INVALID_ARG;
  *out = nullptr;
  if (world == 0 || world > kMaxRanks || rank >= world)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "rank %u / world %u outside 1..%u ranks", rank, world, kMaxRanks);
  if (cudaSetDevice(ctx->device) != cudaSuccess) return ctx_fail(ctx, Q4K_ERR_CUDA, "cudaSetDevice failed");
  q4k_exchange* ex = new q4k_exchange();
  ex->ctx = ctx;
  ex->rank = rank;
  ex->world = world;
  cudaError_t e = cudaMalloc(&ex->mailbox, kMailboxBytes);
  if (e == cudaSuccess) e = cudaMemset(ex->mailbox, 0, kMailboxBytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ex->mailbox);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (ex->mailbox) cudaFree(ex->mailbox);
    delete ex;
    return ctx_cuda(ctx, e, "q4k_exchange_create");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == Q4K_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  ex->peer[rank] = ex->mailbox;
  ex->opened[rank] = true;
  *out = ex;
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_exchange_open(q4k_exchange* ex, uint32_t peer, const void* handle) {
  if (!ex || !handle) return Q4K_ERR_INVALID_ARG;
  q4k_ctx* ctx = ex->ctx;
  if (peer >= ex->world) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "peer %u outside world %u", peer, ex->world);
  if (peer == ex->rank || ex->opened[peer]) return Q4K_OK;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return ctx_fail(ctx, Q4K_ERR_CUDA, "cudaSetDevice failed");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_exchange_open");
  ex->peer[peer] = static_cast<uint32_t*>(p);
  ex->opened[peer] = true;
  ex->ipc[peer] = true;
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_exchange_open_local(q4k_exchange* ex, uint32_t peer, const q4k_exchange* other) {
  if (!ex || !other) return Q4K_ERR_INVALID_ARG;
  q4k_ctx* ctx = ex->ctx;
  if (peer >= ex->world) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "peer %u outside world %u", peer, ex->world);
  if (other->world != ex->world || other->rank != peer)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "the other mailbox is rank %u of %u, expected rank %u of %u",
                    other->rank, other->world, peer, ex->world);
  if (peer == ex->rank || ex->opened[peer]) return Q4K_OK;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return ctx_fail(ctx, Q4K_ERR_CUDA, "cudaSetDevice failed");
  const int pdev = other->ctx->device;
  if (pdev != ctx->device) {
    int can = 0;
    cudaError_t e = cudaDeviceCanAccessPeer(&can, ctx->device, pdev);
    if (e != cudaSuccess || !can)
      return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "device %d cannot access device %d's memory", ctx->device, pdev);
    e = cudaDeviceEnablePeerAccess(pdev, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    else if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_exchange_open_local peer access");
  }
  ex->peer[peer] = other->mailbox;
  ex->opened[peer] = true;
  ex->ipc[peer] = false;
  ctx->err[0] = 0;
  return Q4K_OK;
}

void q4k_exchange_destroy(q4k_exchange* ex) {
  if (!ex) return;
  cudaSetDevice(ex->ctx->device);
  for (uint32_t p = 0; p < ex->world; ++p)
    if (p != ex->rank && ex->opened[p] && ex->ipc[p]) cudaIpcCloseMemHandle(ex->peer[p]);
  if (ex->mailbox) cudaFree(ex->mailbox);
  delete ex;
}

int q4k_lmhead_select_sharded(q4k_ctx* ctx, q4k_exchange* ex, const void* w, const float* x, uint32_t V, uint32_t N,
                              float cap, uint32_t row_offset, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                              void* stream) {
  if (!ctx || !ex) return Q4K_ERR_INVALID_ARG;
  if (!w || !x || !cand_val || !cand_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (N == 0 || N % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "N=%u is not a positive multiple of %d", N, Q4K_QK);
  if (V == 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "V must be >= 1");
  if ((uint64_t)row_offset + V >= (1ull << 31))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "row_offset + V must be < 2^31");
  if (!aligned16(w) || !aligned16(x)) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "w and x must be 16-byte aligned");
  for (uint32_t p = 0; p < ex->world; ++p)
    if (!ex->opened[p]) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "peer %u's mailbox is not open", p);
  if (xfrag_bytes(N, 1) > engine_xcache_bytes(true))
    return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "N=%u exceeds the engine's activation cache", N);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap map;
  uint32_t tile_bytes = 0;
  cudaError_t e = encode_weight_map(&map, w, V, N, &tile_bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_lmhead_select_sharded weight tensor map");
  TaskList tl{};
  tl.n = 1;
  tl.prep = 1;
  tl.inl_job.x = x;
  tl.inl_job.xfrag = ctx->xfrag;
  tl.inl_job.inv_scale = ctx->inv_scale;
  tl.inl_job.N = N;
  tl.inl.w = static_cast<const uint8_t*>(w);
  tl.inl.xfrag = ctx->xfrag;
  tl.inl.inv_scale = ctx->inv_scale;
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
  tl.total_cost = tiles_of(V) * item_cost(N, kTaskSelect);
  tl.pairs = pairs_of(N, 0, tile_bytes) ? 1u : 0u;
  for (uint32_t p = 0; p < ex->world; ++p) tl.xc.peer[p] = ex->peer[p];
  tl.xc.epoch = ex->mailbox + kMailboxEpochWord;
  tl.xc.rank = ex->rank;
  tl.xc.world = ex->world;
  return ctx_cuda(ctx, launch_engine(tl, map, 1, true, ctx->select, ctx->sm_count, s),
                  "q4k_lmhead_select_sharded launch");
}

}  // extern "C"
