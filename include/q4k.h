/*
 * q4k.h -- C ABI of libq4k.so, the B200 (sm_100a) Q4_K matmul path of
 * gemma4-webgpu (tylerstraub/gemma4-webgpu).
 *
 * Every entry point is a drop-in for one WebGPU pipeline dispatch that
 * src/engine.ts records on the decode hot path; the comment of each names the
 * reference interface it replaces.  Conventions shared by all calls:
 *
 *   - All array arguments are DEVICE pointers owned by the caller.  The
 *     library never allocates per call (the context allocates its small
 *     scratch once, in q4k_create).  Outputs are overwritten.
 *   - Weights are GGUF Q4_K bytes exactly as the file stores them: rows of
 *     N/256 super-blocks of 144 bytes (f16 d, f16 dmin, 12 bytes of packed
 *     6-bit scales/mins, 128 bytes of nibbles; src/gguf.ts:157-210), row-major
 *     (ne0 = N fastest, src/gguf.ts:89-97).  N must be a multiple of 256.
 *   - The weight each output sees is the reference's: the Q4_K value rounded
 *     once to f32 and then to f16 (round to nearest even), multiplied in f32
 *     (src/gguf.ts:168-210 + 425-473, shaders/matmul_quant.wgsl:35).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous on that stream; none synchronizes the host, none allocates,
 *     so they can be captured in a CUDA graph.
 *   - Pointers must be 16-byte aligned (weights, activations, outputs).
 *   - Return value: Q4K_OK (0) or a negative Q4K_ERR_* code; the reason is in
 *     q4k_last_error(ctx).  Launch errors are reported at the call; faults
 *     inside a kernel surface at the caller's next synchronization, as CUDA
 *     errors do.  Nothing throws across the ABI.
 *   - A context belongs to one device and one host thread; calls on one
 *     context must be ordered on one stream (the fused LM head shares the
 *     context's selection scratch between calls).
 */
#ifndef Q4K_H_
#define Q4K_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q4K_API __attribute__((visibility("default")))
#else
#define Q4K_API
#endif

#define Q4K_OK 0
#define Q4K_ERR_INVALID_ARG (-1) /* shape, alignment or null pointer rejected */
#define Q4K_ERR_CUDA (-2)        /* CUDA runtime error (launch, device) */
#define Q4K_ERR_UNSUPPORTED (-3) /* valid request this build cannot serve */
#define Q4K_ERR_TIMEOUT (-4)     /* a kernel gave up a bounded wait; outputs invalid */
#define Q4K_ERR_SCRATCH_LIMIT (-5) /* request larger than q4k_lmhead_select_static's fixed scratch */

#define Q4K_QK 256          /* weights per Q4_K super-block */
#define Q4K_BLOCK_BYTES 144 /* bytes per Q4_K super-block */

typedef struct q4k_ctx q4k_ctx;

/* ABI version (major * 100 + minor). */
Q4K_API int q4k_version(void);

/* Create a context on `device` (makes it current on the calling thread) and
 * allocate its scratch.  Replaces the engine's device/pipeline set-up for this
 * path: initWebGPU + createPipelines (src/engine.ts:354-430). */
Q4K_API int q4k_create(int device, q4k_ctx** out);

/* Free the context and its scratch.  NULL is ignored. */
Q4K_API void q4k_destroy(q4k_ctx* ctx);

/* Message of the last failed call on `ctx` ("" if none); never NULL. */
Q4K_API const char* q4k_last_error(const q4k_ctx* ctx);

/* Synchronize the device and report whether any kernel launched through
 * `ctx` gave up one of its bounded waits since the last check (every wait
 * on an asynchronous copy has an iteration limit; on expiry the kernel
 * records it, drains its copies and returns instead of hanging), or met an
 * invalid device-side input (a token id past the vocabulary in
 * q4k_ple_stage1).  Returns Q4K_OK, Q4K_ERR_TIMEOUT or Q4K_ERR_INVALID_ARG,
 * and clears the record.  The reference's
 * counterpart is the device-lost flag checked before public calls
 * (src/engine.ts:385-388, 1677). */
Q4K_API int q4k_check(q4k_ctx* ctx);

/* Polls each bounded wait of this context's kernels makes before giving up
 * (the wait on a weight copy, a K-split partner or a peer rank's candidates;
 * expiry is what q4k_check reports as Q4K_ERR_TIMEOUT).  polls = 0 restores
 * the built-in default (2^22 polls, seconds).  A smaller limit makes a lost
 * peer or copy surface sooner; it must stay well above the longest legitimate
 * wait (microseconds for copies, a peer's whole shard for the sharded head).
 * Applies to launches made after the call.  No reference counterpart (WebGPU
 * exposes no timeout; the engine's only failure signal is device loss,
 * src/engine.ts:385-388). */
Q4K_API int q4k_set_wait_limit(q4k_ctx* ctx, uint32_t polls);

/* matmul_quant: output[m] = sum_k f32(w[m,k]) * input[k], m < M.
 * Argument order and meaning follow the pipeline's bind group 0
 * {0: input f32[N], 1: weight, 2: output f32[M], 3: {M, N}}
 * (shaders/matmul_quant.wgsl:12-16, shaders/matmul_quant_mr4.wgsl:73-76,
 * dispatched by dispatchMatmul, src/engine.ts:332-341); the weight binding
 * holds Q4_K bytes instead of the pre-dequantized f16 buffer. */
Q4K_API int q4k_matmul_quant(q4k_ctx* ctx, const float* input, const void* weight, float* output, uint32_t M, uint32_t N,
                     void* stream);

/* Batched form: y[b*M + m] = sum_k f32(w[m,k]) * x[b*N + k] for b < batch.
 * One weight stream serves all `batch` activation rows (the MR4 pipeline's
 * shared input read, shaders/matmul_quant_mr4.wgsl:107-115, turned around:
 * several inputs share one weight read).  batch >= 1; batch >= 64 runs as
 * q4k_gemm. */
Q4K_API int q4k_gemv(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t batch,
             void* stream);

/* Batched form for many activation rows (prefill, or T independent sequences
 * sharing the weights): y[t*M + m] = sum_k f32(w[m,k]) * x[t*N + k], t < T,
 * on the tensor cores (tcgen05).  The reference has only the one-row
 * matmul_quant (shaders/matmul_quant.wgsl:21-54), run once per row; q4k_gemv
 * hands batch >= 64 to this path.  Any T >= 1. */
Q4K_API int q4k_gemm(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
                     void* stream);

/* q4k_gemm with each activation row rounded once to f16 (after a
 * power-of-two row scale that keeps it in range) instead of entering as
 * exact f16 hi + lo parts: half the tensor-core work and operand traffic,
 * for prefill and batched sequences where the relative tolerance of 2e-3
 * applies (the weights are still the reference's f16 values exactly; the
 * product error is that of an f16 activation, ~2e-4 relative in L2).
 * Replaces the same per-row matmul_quant passes as q4k_gemm
 * (shaders/matmul_quant.wgsl:21-54, run per prompt token by
 * src/engine.ts:1932-1934).  Any T >= 1. */
Q4K_API int q4k_gemm_f16x(q4k_ctx* ctx, const void* w, const float* x, float* y, uint32_t M, uint32_t N, uint32_t T,
                          void* stream);

/* The f16 weights the reference uploads for a Q4_K tensor (its
 * dequantizeQ4_K + f32ToF16Array + createF16Buffer, src/gguf.ts:168-210,
 * 425-473, src/engine.ts:553-578, 828-841): n_blocks super-blocks ->
 * n_blocks*256 f16 bit patterns.  The weight-probe comparison
 * (src/diagnostics/weight-probe.ts:60-162) reads these. */
Q4K_API int q4k_dequant_f16(q4k_ctx* ctx, const void* w, uint16_t* out, uint64_t n_blocks, void* stream);

/* logit_softcap in place: logits[i] = tanh(clamp(logits[i]/cap, -15, 15))*cap
 * (shaders/logit_softcap.wgsl:9-16; cap from src/engine.ts:447). */
Q4K_API int q4k_logit_softcap(q4k_ctx* ctx, float* logits, uint32_t n, float cap, void* stream);

/* argmax: *result = index of the maximum with the reference's tie rule
 * (shaders/argmax.wgsl:7-34; result buffer src/engine.ts:1037). */
Q4K_API int q4k_argmax(q4k_ctx* ctx, const float* logits, uint32_t n, uint32_t* result, void* stream);

/* topk256: result f32[512] = 256 (max, bitcast<f32>(index)) pairs, pair t
 * being the first strict maximum over indices = t (mod 256)
 * (shaders/topk256.wgsl:5-21; buffer src/engine.ts:1042). */
Q4K_API int q4k_topk256(q4k_ctx* ctx, const float* logits, uint32_t n, float* result, void* stream);

/* logitSoftcap + topk256 + argmax for B (1..16) rows of n logits (row b at
 * logits + b*n) in one launch: the per-token tail of sampleNextTokenSubmit
 * (src/engine.ts:1686-1741) when several sequences decode together.  cap > 0
 * softcaps the logits in place first (shaders/logit_softcap.wgsl:9-16);
 * cap <= 0 leaves them.  cand_val [B][256] / cand_idx [B][256] are each
 * row's topk256 pairs (shaders/topk256.wgsl:5-21), argmax [B] its argmax
 * (shaders/argmax.wgsl:7-34), bit-identical to q4k_logit_softcap then
 * q4k_topk256 and q4k_argmax per row.  Uses the context's row scratch: order
 * the calls of one context on one stream. */
Q4K_API int q4k_select_rows(q4k_ctx* ctx, float* logits, uint32_t B, uint32_t n, float cap, float* cand_val,
                            uint32_t* cand_idx, uint32_t* argmax, void* stream);

/* gelu_mul: out[i] = GELU_tanh(gate[i]) * up[i] (shaders/gelu_mul.wgsl:1-17). */
Q4K_API int q4k_gelu_mul(q4k_ctx* ctx, const float* gate, const float* up, float* out, uint32_t n, void* stream);

/* Fused LM head on a vocabulary shard: the lmHead matmul + logitSoftcap +
 * argmax/topk256 passes of sampleNextTokenSubmit (src/engine.ts:1686-1741)
 * in one launch.  Rows [0, V) of `w` are global vocabulary indices
 * row_offset + i (row_offset = 0 for an unsharded head).  cap <= 0 skips
 * the softcap (src/engine.ts:1695).  Outputs: cand_val/cand_idx [256] =
 * the topk256 pairs of this shard in global indices, *argmax = the argmax of
 * this shard, logits [V] = the softcapped logits (may be NULL: not stored).
 * row_offset + V must be < 2^31. */
Q4K_API int q4k_lmhead_select(q4k_ctx* ctx, const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                      uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                      void* stream);

/* Merge G shards' candidate sets (vals/idx [G][256], e.g. after an
 * all-gather) into the candidates and argmax the unsharded head would give.
 * No reference counterpart: the reference is single-device. */
Q4K_API int q4k_merge_candidates(q4k_ctx* ctx, const float* vals, const uint32_t* idx, uint32_t G, float* out_val,
                         uint32_t* out_idx, uint32_t* argmax, void* stream);

/* The fused LM head of q4k_lmhead_select for callers that cannot allocate
 * device memory: no context, no cudaMalloc/cudaFree, no allocating library
 * call.  It exists for real-time decode loops that must never enter the
 * driver's allocator (an allocation can block on device-wide
 * synchronization), and for embedders whose device memory is owned and
 * budgeted by another runtime, so they cannot call q4k_create (which
 * allocates the context's scratch).  No counterpart in the reference.
 *
 * Its scratch is a fixed array inside libq4k.so (67,328 bytes on every GPU
 * that loads the library, held until the process exits), which limits the
 * row length to N <= 16384; larger N returns Q4K_ERR_SCRATCH_LIMIT.  The
 * first call on a device looks up that array's device address (with the
 * device current), so make the first call on each device before any stream
 * capture.  Every call shares the one array and resets its selection state
 * first: calls that overlap on the GPU (other streams, other host threads)
 * race and give wrong results; order them on one stream.  The cached
 * address does not survive cudaDeviceReset: do not reset a device between
 * calls.  Arguments and outputs as q4k_lmhead_select; errors are return
 * codes only: argument and launch errors at the call, and a bounded wait
 * that expired inside the kernel (outputs invalid) through
 * q4k_check_static. */
Q4K_API int q4k_lmhead_select_static(const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                                     uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx,
                                     uint32_t* argmax, void* stream);

/* The q4k_check of q4k_lmhead_select_static, which has no context: on the
 * current device, synchronize, then report whether any call since the last
 * check gave up a bounded wait (Q4K_ERR_TIMEOUT; those calls' outputs are
 * invalid) and clear the record, reading the fixed array's status word
 * without allocating.  Q4K_OK otherwise.  No counterpart in the reference. */
Q4K_API int q4k_check_static(void);

/* ---- vocabulary-sharded LM head, exchange fused into the launch -------
 * The reference's LM head runs on one device (sampleNextTokenSubmit,
 * src/engine.ts:1686-1741).  Split over G ranks (one process per GPU, rank r
 * owning rows [r*V/G, (r+1)*V/G), V/G a multiple of 256), each rank's launch
 * computes its shard, writes its 256 candidates straight into every rank's
 * mailbox over NVLink (peer stores, no collective library), waits for all
 * ranks' candidates (bounded) and merges them: the outputs on every rank
 * equal the unsharded head's.  Set-up: every rank creates its mailbox
 * (q4k_exchange_create returns a Q4K_EXCHANGE_HANDLE_BYTES handle), the
 * handles are exchanged out of band (e.g. a torch.distributed all-gather),
 * and every rank opens every peer's (q4k_exchange_open).  Calls must be made
 * by all ranks in the same order; a rank that never arrives makes the others
 * give up their bounded wait (Q4K_ERR_TIMEOUT from q4k_check). */
#define Q4K_EXCHANGE_HANDLE_BYTES 64
typedef struct q4k_exchange q4k_exchange;

Q4K_API int q4k_exchange_create(q4k_ctx* ctx, uint32_t rank, uint32_t world, q4k_exchange** out, void* handle_out);
Q4K_API int q4k_exchange_open(q4k_exchange* ex, uint32_t peer, const void* handle);
/* q4k_exchange_open for a peer mailbox created in this same process (ranks
 * driven as devices of one process, where a CUDA IPC handle cannot be
 * reopened): maps `other` (rank `peer` of the same world) directly, enabling
 * peer access when it lives on another device. */
Q4K_API int q4k_exchange_open_local(q4k_exchange* ex, uint32_t peer, const q4k_exchange* other);
Q4K_API void q4k_exchange_destroy(q4k_exchange* ex);

/* This rank's shard of the head (rows of `w` are global indices row_offset +
 * i, i < V) + the exchange + the merge, in one launch.  Outputs as
 * q4k_lmhead_select (without logits), for the whole vocabulary. */
Q4K_API int q4k_lmhead_select_sharded(q4k_ctx* ctx, q4k_exchange* ex, const void* w, const float* x, uint32_t V,
                                      uint32_t N, float cap, uint32_t row_offset, float* cand_val,
                                      uint32_t* cand_idx, uint32_t* argmax, void* stream);

/* ---- Q6_K matrices -----------------------------------------------------
 * Q4_K_M files store some matmul weights as Q6_K (docs/findings/why-q4km.md:33;
 * 210-byte super-blocks: ql[128], qh[64], int8 scales[16], f16 d).  The
 * reference decodes them on the CPU at load (dequantizeQ6_K,
 * src/gguf.ts:316-368, then f32ToF16Array + upload via tensorToF16,
 * src/engine.ts:570-578) and multiplies them with the same matmul_quant
 * pipelines.  Here they stay 6.56 bits per weight on the device: once at
 * load, q4k_q6k_repack rewrites the GGUF bytes into the "Q6_K device
 * layout" (every 208-byte body ql|qh|scales 16-byte aligned, row-major
 * [M][N/256]; then the f16 d values as a plane [N/256][M rounded up to 8]),
 * q4k_q6k_device_bytes(M, N) bytes, and the calls below read that layout.
 * Weights seen by each output: f16_rne(f32(d*sc*(q-32))), the reference's. */

/* Bytes of the device layout of an M x N Q6_K matrix (0 if N % 256 != 0). */
Q4K_API uint64_t q4k_q6k_device_bytes(uint32_t M, uint32_t N);

/* Load-time repack: GGUF Q6_K bytes (w_gguf: M rows of N/256 super-blocks,
 * 2-byte aligned) -> device layout (w_dev, 16-byte aligned,
 * q4k_q6k_device_bytes(M, N) bytes).  Replaces the reference's per-tensor
 * dequantizeQ6_K + f32ToF16Array + writeBuffer (src/engine.ts:570-578). */
Q4K_API int q4k_q6k_repack(q4k_ctx* ctx, const void* w_gguf, void* w_dev, uint32_t M, uint32_t N, void* stream);

/* Weight probe: out[M*N] = the f16 bit patterns the GEMV multiplies, in
 * row-major order -- the reference's uploaded f16 weight buffer, for the
 * weight-probe comparison (src/diagnostics/weight-probe.ts:60-162). */
Q4K_API int q4k_q6k_dequant_f16(q4k_ctx* ctx, const void* w_dev, uint32_t M, uint32_t N, uint16_t* out,
                                void* stream);

/* y[t*M + m] = sum_k w16[m,k] * x[t*N + k] for a Q6_K matrix in the device
 * layout: the matmul_quant dispatch (shaders/matmul_quant.wgsl:21-54) of a
 * Q6_K-sourced weight (src/engine.ts:1547-1605 call sites).  Same tolerance
 * and conventions as q4k_gemv; batch > 16 runs in chunks of 16 rows. */
Q4K_API int q4k_q6k_gemv(q4k_ctx* ctx, const void* w_dev, const float* x, float* y, uint32_t M, uint32_t N,
                         uint32_t batch, void* stream);

/* q4k_lmhead_select for a Q6_K LM head in the device layout (Q4_K_M files
 * commonly store the tied token_embd / output matrix as Q6_K): lmHead matmul
 * + logitSoftcap + argmax/topk256 candidates in one launch
 * (src/engine.ts:1686-1741). */
Q4K_API int q4k_q6k_lmhead_select(q4k_ctx* ctx, const void* w_dev, const float* x, uint32_t V, uint32_t N,
                                  float cap, uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx,
                                  uint32_t* argmax, void* stream);

/* ---- per-layer embeddings (Q5_K) ---------------------------------------
 * Gemma-4-E2B's per-layer embedding table per_layer_token_embd is Q5_K
 * (176-byte super-blocks: f16 d, f16 dmin, 12 packed 6-bit scale/min bytes,
 * qh[32], qs[128]); row v holds `layers` consecutive super-blocks, block L
 * being layer L's 256 values.  The reference decodes the whole 1.6 GB table
 * at load into one f16 buffer per layer (streamDecodePleQ5_K,
 * src/engine.ts:642-721; decodeQ5_KBlock, src/gguf.ts:218-256) and per
 * token runs ple_stage1_fuse once per layer (src/engine.ts:1528-1535).
 * Here the table stays Q5_K on the device and is read only for the tokens
 * being decoded. */

/* Weight probe: out[n_blocks*256] = the f16 bit patterns of the decoded
 * values, the reference's uploaded per-layer embedding entries
 * (decodeQ5_KBlock + f32ToF16Array, src/engine.ts:683-702).  w 16-byte
 * aligned. */
Q4K_API int q4k_q5k_dequant_f16(q4k_ctx* ctx, const void* w, uint16_t* out, uint64_t n_blocks, void* stream);

/* shaders/ple_stage1_fuse.wgsl (bind group {projected, norm_weight,
 * embed_slice, ple_inputs, {layer_idx, token_id, per_layer_dim, eps}}) for
 * every layer of T tokens in one launch, per_layer_dim = 256:
 *   out[t][L*256+i] = ((projected[t][L*256+i] / rms_tL) * f32(norm_w[i])
 *                      + embed_L[token_t][i] * 16) * inverseSqrt(2),
 *   rms_tL = sqrt(sum_i projected[t][L*256+i]^2 / 256 + eps),
 * embed_L[v][i] decoded from the Q5_K table (16-byte aligned, vocab rows of
 * layers*176 bytes) exactly as the reference uploads it.  token_ids [T] are
 * device memory (e.g. the previous step's argmax output, as
 * src/engine.ts:1719-1727 feeds it); an id >= vocab makes that token's
 * outputs NaN and q4k_check return Q4K_ERR_INVALID_ARG. */
Q4K_API int q4k_ple_stage1(q4k_ctx* ctx, const void* table_q5k, const uint32_t* token_ids, uint32_t T,
                           uint32_t vocab, uint32_t layers, const float* projected, const uint16_t* norm_w,
                           float eps, float* out, void* stream);

/* ---- the chained decode step -------------------------------------------
 * One token's layers as a true chain, each layer reading the previous
 * layer's output, in ONE persistent launch (plus the fused LM head): the
 * matmul_quant dispatches of encodeTransformerPass (src/engine.ts:1538-1619)
 * with the reference's elementwise passes between them restated so the data
 * flows as it does there (norm weights 1):
 *   n1 = rms_norm(h)                      attn.rmsNorm     (rms_norm.wgsl)
 *   q, k, v = Wq n1, Wk n1, Wv n1         linearQKV
 *   a = per-head rms_norm(v) for every    vNorm + attention at position 0
 *       query head (one cached key:       (per_head_rms_norm_no_weight.wgsl;
 *       softmax of one score is 1)         attn_score/softmax/attn_output)
 *   o = Wo a                              linearOut
 *   h_attn = h + rms_norm(o)              attn.postNormAdd (fused_norm_add.wgsl)
 *   n2 = rms_norm(h_attn)                 ffn.rmsNorm
 *   g, u = Wg n2, Wu n2; act = gelu(g)*u  linearGateUp, geluMul
 *   d = Wd act                            linearDown
 *   h_out = h_attn + rms_norm(d)          ffn.postNormAdd: the next layer's h
 * and after the last layer normed_out = rms_norm(h_out) (final.rmsNorm,
 * src/engine.ts:1620-1626), the LM head's input.  rms_norm(x) = x /
 * sqrt(sum(x^2)/n + eps).  One KV head of kv_dim elements (q_dim a multiple
 * of it).  Every dimension a multiple of 256, at most 8192.  All buffers are
 * the caller's device memory, 16-byte aligned; every per-layer output is
 * written each run.  q4k_chain_create allocates the step's descriptors once;
 * q4k_chain_run allocates nothing and is graph-capturable.  The launch waits
 * on grid-wide stage counters with bounded polls (q4k_set_wait_limit); an
 * expired wait is reported by q4k_check. */
typedef struct q4k_chain q4k_chain;

typedef struct {
  const void* wq;  /* Q4_K [q_dim][hidden] */
  const void* wk;  /* Q4_K [kv_dim][hidden] */
  const void* wv;  /* Q4_K [kv_dim][hidden] */
  const void* wo;  /* Q4_K [hidden][q_dim] */
  const void* wg;  /* Q4_K [ffn][hidden] */
  const void* wu;  /* Q4_K [ffn][hidden] */
  const void* wd;  /* Q4_K [hidden][ffn] */
  float* q;        /* [q_dim] */
  float* k;        /* [kv_dim] */
  float* v;        /* [kv_dim] (before its norm) */
  float* o;        /* [hidden] */
  float* g;        /* [ffn] */
  float* u;        /* [ffn] */
  float* act;      /* [ffn] gelu(g)*u */
  float* d;        /* [hidden] */
  float* h_attn;   /* [hidden] residual after the attention block */
  float* h_out;    /* [hidden] residual after the FFN block */
} q4k_chain_layer;

/* Record the chain over `layers` layers: per_layer[layers], h_in [hidden]
 * the first layer's input, normed_out [hidden] the final norm.  No
 * reference counterpart as one call: it is the per-token layer loop of
 * encodeTransformerPass, recorded once like the engine's bind groups. */
Q4K_API int q4k_chain_create(q4k_ctx* ctx, uint32_t layers, uint32_t hidden, uint32_t q_dim, uint32_t kv_dim,
                             uint32_t ffn, float eps, const q4k_chain_layer* per_layer, const float* h_in,
                             float* normed_out, q4k_chain** out);

/* Add the fused LM head (q4k_lmhead_select with softcap `cap`) on
 * normed_out to every run: sampleNextTokenSubmit's lmHead + logitSoftcap +
 * topk256/argmax (src/engine.ts:1686-1741).  w: Q4_K [V][hidden]. */
Q4K_API int q4k_chain_lmhead(q4k_chain* chain, const void* w, uint32_t V, float cap, float* cand_val,
                             uint32_t* cand_idx, uint32_t* argmax);

/* Run the step on `stream`: one persistent launch (+ the LM head launch). */
Q4K_API int q4k_chain_run(q4k_chain* chain, void* stream);

/* Kernel launches one q4k_chain_run issues. */
Q4K_API int q4k_chain_launches(const q4k_chain* chain);

/* Free the chain's descriptors.  NULL is ignored. */
Q4K_API void q4k_chain_destroy(q4k_chain* chain);

/* ---- plans ------------------------------------------------------------
 * A plan records a decode step's matmul-path operations once and replays
 * them with two launches per stage, the way the engine records a token's
 * passes into one command encoder with pre-built bind groups and submits it
 * (encodeTransformerPass + queue.submit, src/engine.ts:1466-1626, 1748).
 * Operations of one stage are independent of each other; stage s+1 runs
 * after stage s.  A gelu_mul whose `act` buffer is the `x` of a GEMV in the
 * same stage is evaluated while that GEMV's input is prepared (the
 * geluMul -> linearDown pair of src/engine.ts:1604-1605).  Buffers are
 * bound by pointer at record time, like bind groups.  q4k_plan_commit
 * allocates the plan's device memory once; q4k_plan_run allocates nothing. */
typedef struct q4k_plan q4k_plan;

/* New empty plan whose GEMVs all take `batch` activation rows: 1..16 on
 * the GEMV engine, or 64..8192 (prefill, or that many sequences sharing the
 * weights) on the tcgen05 GEMM, where each stage runs as one preparation
 * launch over its distinct activations plus ONE GEMM launch over every
 * matrix of the stage (no per-matrix launches).  GEMM plans take Q4_K
 * GEMVs and gelu_mul ops, no LM head; their activations are rounded once to
 * f16 after a power-of-two row scale (q4k_gemm_f16x's 2e-3 prefill
 * tolerance) unless q4k_plan_gemm_exact asks for the exact form. */
Q4K_API int q4k_plan_create(q4k_ctx* ctx, uint32_t batch, q4k_plan** out);

/* GEMM plans only, before commit: exact != 0 feeds each activation row as
 * exact f16 hi + lo parts (q4k_gemm's GEMV tolerance; twice the tensor-core
 * work), 0 restores the f16 default.  The reference runs every prompt token
 * through the one-row matmul_quant (src/engine.ts:1932-1934). */
Q4K_API int q4k_plan_gemm_exact(q4k_plan* plan, int exact);

/* Free a plan and its device memory.  NULL is ignored. */
Q4K_API void q4k_plan_destroy(q4k_plan* plan);

/* Record y = matmul_quant(w, x) (as q4k_gemv with the plan's batch). */
Q4K_API int q4k_plan_gemv(q4k_plan* plan, uint32_t stage, const void* w, const float* x, float* y, uint32_t M,
                          uint32_t N);

/* Record act = gelu_mul(gate, up) (shaders/gelu_mul.wgsl), n a multiple of 256. */
Q4K_API int q4k_plan_gelu_mul(q4k_plan* plan, uint32_t stage, const float* gate, const float* up, float* act,
                              uint32_t n);

/* Record the fused LM head of q4k_lmhead_select (batch-1 plans, one per stage). */
Q4K_API int q4k_plan_lmhead(q4k_plan* plan, uint32_t stage, const void* w, const float* x, uint32_t V, uint32_t N,
                            float cap, uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx,
                            uint32_t* argmax);

/* Q6_K variants of q4k_plan_gemv / q4k_plan_lmhead: the weight is a Q6_K
 * matrix in the device layout (q4k_q6k_repack).  A stage that mixes Q4_K and
 * Q6_K matrices runs as one engine launch per format. */
Q4K_API int q4k_plan_gemv_q6k(q4k_plan* plan, uint32_t stage, const void* w_dev, const float* x, float* y,
                              uint32_t M, uint32_t N);
Q4K_API int q4k_plan_lmhead_q6k(q4k_plan* plan, uint32_t stage, const void* w_dev, const float* x, uint32_t V,
                                uint32_t N, float cap, uint32_t row_offset, float* logits, float* cand_val,
                                uint32_t* cand_idx, uint32_t* argmax);

/* Finish recording: lay out and upload the launch descriptors. */
Q4K_API int q4k_plan_commit(q4k_plan* plan);

/* Launch every stage on `stream` (asynchronous, graph-capturable). */
Q4K_API int q4k_plan_run(q4k_plan* plan, void* stream);

/* Kernel launches one q4k_plan_run issues (-1 before commit). */
Q4K_API int q4k_plan_launches(const q4k_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* Q4K_H_ */
