/*
 * q4k_oracle.c -- CPU restatement of gemma4-webgpu's Q4_K matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * (libq4k.so) and the timed CPU baseline of bench.py.  Nothing in the product
 * path links, loads or calls it; only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs do.
 *
 * Parity status: the reference is TypeScript + WGSL and cannot execute in this
 * container (no Node, no WebGPU adapter), and it ships no golden vectors for
 * this path.  The Q4_K decode (a1-a3 below) is pinned against golden vectors
 * produced by the `gguf` Python package 0.19.0 (gguf-py, the published
 * llama.cpp dequantize_row_q4_K algorithm that src/gguf.ts:164-166 cites),
 * committed under tests/golden/.  The f32->f16 rounding is pinned against
 * numpy's IEEE round-to-nearest-even conversion.  The GEMV summation order,
 * softcap, argmax and topk256 follow the WGSL text and are otherwise
 * "parity unpinned": no executable reference or fixture exists for them.
 *
 * Build flags matter: -ffp-contract=off and no -ffast-math, so every f32 and
 * f64 operation rounds exactly once as written.
 *
 * Reference citations (paths inside tylerstraub/gemma4-webgpu):
 *   f16 decode          src/gguf.ts:103-113   (f16ToF32)
 *   Q4_K decode         src/gguf.ts:157-210   (dequantizeQ4_K, getScaleMin :175-182)
 *   f32 -> f16          src/gguf.ts:425-473   (f32ToF16Array: Float16Array RNE at
 *                                              :432-436, truncating fallback :443-471)
 *   Q6_K decode         src/gguf.ts:316-368   (dequantizeQ6_K)
 *   Q5_K decode         src/gguf.ts:212-256   (decodeQ5_KBlock; :262-314 dequantizeQ5_K)
 *   PLE stage 1         shaders/ple_stage1_fuse.wgsl:16-38, embedding slice upload
 *                       src/engine.ts:681-702 (row v, layer L = block v*layers + L)
 *   GEMV                shaders/matmul_quant.wgsl:21-54
 *   4-row GEMV          shaders/matmul_quant_mr4.wgsl:33-88 (same per-row order)
 *   softcap             shaders/logit_softcap.wgsl:9-16
 *   argmax              shaders/argmax.wgsl:7-34
 *   topk256             shaders/topk256.wgsl:5-21
 *   gelu_mul            shaders/gelu_mul.wgsl:1-17
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>
#ifdef __F16C__
#include <immintrin.h>
#endif

#define ORC_API __attribute__((visibility("default")))

enum { QK_K = 256, Q4K_BLOCK_BYTES = 144, Q6K_BLOCK_BYTES = 210, Q5K_BLOCK_BYTES = 176 };

/* ---- f16 <-> f32 ------------------------------------------------------- */

/* Exact IEEE half decode, as src/gguf.ts:103-113 computes it in f64. */
static double f16_to_f64(uint16_t h) {
  const int sign = (h >> 15) & 1;
  const int ex = (h >> 10) & 0x1f;
  const int mant = h & 0x3ff;
  const double s = sign ? -1.0 : 1.0;
  if (ex == 0) {
    if (mant == 0) return sign ? -0.0 : 0.0;
    return s * ldexp(1.0, -14) * ((double)mant / 1024.0);
  }
  if (ex == 31) return mant == 0 ? s * INFINITY : NAN;
  return s * ldexp(1.0, ex - 15) * (1.0 + (double)mant / 1024.0);
}

ORC_API float orc_f16_to_f32(uint16_t h) { return (float)f16_to_f64(h); }

/* IEEE-754 binary32 -> binary16, round to nearest, ties to even.  This is the
 * conversion `Float16Array.set` performs (src/gguf.ts:432-436), written from
 * the IEEE definition: NaN stays NaN (quiet), |v| >= 65520 overflows to inf,
 * values below 2^-14 round to the 2^-24 subnormal grid. */
ORC_API uint16_t orc_f32_to_f16_rne(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const uint32_t a = b & 0x7fffffffu;
  if (a > 0x7f800000u) return sign | 0x7e00u;          /* NaN */
  if (a >= 0x477ff000u) return sign | 0x7c00u;         /* >= 65520 (or inf) */
  if (a >= 0x38800000u) {                              /* f16 normal range */
    const uint32_t odd = (a >> 13) & 1u;
    const uint32_t r = a + 0x0fffu + odd;              /* RNE at bit 13 */
    return sign | (uint16_t)((r - 0x38000000u) >> 13); /* rebias 127 -> 15 */
  }
  /* f16 subnormal or zero: integer multiple of 2^-24, RNE by rint(). */
  float mag;
  memcpy(&mag, &a, 4);
  const float scaled = mag * 16777216.0f;              /* exact: power of two */
  return sign | (uint16_t)rintf(scaled);
}

/* The manual fallback of src/gguf.ts:443-471 (used only where Float16Array is
 * missing): truncates the mantissa, flushes f32 subnormals to zero.  Kept so
 * tests can show the two modes differ; the parity target is RNE. */
ORC_API uint16_t orc_f32_to_f16_trunc(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const uint32_t exp_raw = (b >> 23) & 0xffu;
  const uint32_t mant = b & 0x7fffffu;
  if (exp_raw == 0xffu) return sign | 0x7c00u | (mant ? 0x200u : 0u);
  if (exp_raw == 0u) return sign;
  const int new_exp = (int)exp_raw - 127 + 15;
  if (new_exp >= 0x1f) return sign | 0x7c00u;
  if (new_exp <= 0) {
    if (new_exp < -10) return sign;
    return sign | (uint16_t)((mant | 0x800000u) >> (1 - new_exp + 13));
  }
  return sign | (uint16_t)((uint32_t)new_exp << 10) | (uint16_t)(mant >> 13);
}

/* ---- Q4_K super-block decode ------------------------------------------- */

/* getScaleMin, src/gguf.ts:175-182: 12 packed bytes -> (scale, min) of
 * sub-block j (0..7), both 6-bit. */
static void get_scale_min(const uint8_t* s, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 0x3f;
    *m = s[j + 4] & 0x3f;
  } else {
    *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

ORC_API void orc_q4k_scale_min(const uint8_t* block, int j, int* sc, int* m) {
  get_scale_min(block + 4, j, sc, m);
}

/* One super-block -> 256 f32, exactly as src/gguf.ts:187-206 evaluates it:
 * d1 = d*sc, min1 = dmin*m and d1*q - min1 in f64, then one rounding to f32
 * when stored into the Float32Array. */
static void dequant_block_f32(const uint8_t* blk, float* out) {
  const double d = f16_to_f64((uint16_t)(blk[0] | (blk[1] << 8)));
  const double dmin = f16_to_f64((uint16_t)(blk[2] | (blk[3] << 8)));
  const uint8_t* scales = blk + 4;
  const uint8_t* qs = blk + 16;
  for (int g = 0; g < 4; ++g) {
    int sc1, m1, sc2, m2;
    get_scale_min(scales, 2 * g, &sc1, &m1);
    get_scale_min(scales, 2 * g + 1, &sc2, &m2);
    const double d1 = d * sc1, min1 = dmin * m1;
    const double d2 = d * sc2, min2 = dmin * m2;
    for (int l = 0; l < 32; ++l) out[64 * g + l] = (float)(d1 * (qs[32 * g + l] & 0x0f) - min1);
    for (int l = 0; l < 32; ++l) out[64 * g + 32 + l] = (float)(d2 * ((qs[32 * g + l] >> 4) & 0x0f) - min2);
  }
}

ORC_API void orc_q4k_dequant_f32(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; ++b) dequant_block_f32(blocks + b * Q4K_BLOCK_BYTES, out + b * QK_K);
}

/* Q4_K -> f16 bit patterns: the weight the reference GPU actually multiplies
 * (dequantizeQ4_K then f32ToF16Array).  round_mode 0 = RNE (Float16Array),
 * 1 = the truncating fallback. */
ORC_API void orc_q4k_dequant_f16(const uint8_t* blocks, int64_t n_blocks, uint16_t* out, int round_mode) {
  float tmp[QK_K];
  for (int64_t b = 0; b < n_blocks; ++b) {
    dequant_block_f32(blocks + b * Q4K_BLOCK_BYTES, tmp);
    for (int i = 0; i < QK_K; ++i)
      out[b * QK_K + i] = round_mode ? orc_f32_to_f16_trunc(tmp[i]) : orc_f32_to_f16_rne(tmp[i]);
  }
}

/* ---- Q6_K super-block decode ------------------------------------------- */

/* One Q6_K super-block (210 bytes: ql[128], qh[64], int8 scales[16], f16 d)
 * -> 256 f32, as src/gguf.ts:329-364 evaluates it: per half, element l of
 * the four 32-wide quarters is (4 bits of ql, 2 bits of qh) - 32, times the
 * quarter's int8 scale of sub-block l/16 and d, in f64, one rounding to f32
 * at the Float32Array store. */
static void dequant_q6k_block_f32(const uint8_t* blk, float* out) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const int8_t* sc = (const int8_t*)(blk + 192);
  const double d = f16_to_f64((uint16_t)(blk[208] | (blk[209] << 8)));
  for (int half = 0; half < 2; ++half) {
    const uint8_t* l0 = ql + 64 * half;
    const uint8_t* h0 = qh + 32 * half;
    const int8_t* s0 = sc + 8 * half;
    float* o = out + 128 * half;
    for (int l = 0; l < 32; ++l) {
      const int is = l >> 4;
      const int q1 = ((l0[l] & 0x0f) | (((h0[l] >> 0) & 3) << 4)) - 32;
      const int q2 = ((l0[l + 32] & 0x0f) | (((h0[l] >> 2) & 3) << 4)) - 32;
      const int q3 = ((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32;
      const int q4 = ((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32;
      o[l] = (float)(d * s0[is + 0] * q1);
      o[l + 32] = (float)(d * s0[is + 2] * q2);
      o[l + 64] = (float)(d * s0[is + 4] * q3);
      o[l + 96] = (float)(d * s0[is + 6] * q4);
    }
  }
}

ORC_API void orc_q6k_dequant_f32(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; ++b) dequant_q6k_block_f32(blocks + b * Q6K_BLOCK_BYTES, out + b * QK_K);
}

/* Q6_K -> f16 bit patterns (dequantizeQ6_K then f32ToF16Array, RNE). */
ORC_API void orc_q6k_dequant_f16(const uint8_t* blocks, int64_t n_blocks, uint16_t* out) {
  float tmp[QK_K];
  for (int64_t b = 0; b < n_blocks; ++b) {
    dequant_q6k_block_f32(blocks + b * Q6K_BLOCK_BYTES, tmp);
    for (int i = 0; i < QK_K; ++i) out[b * QK_K + i] = orc_f32_to_f16_rne(tmp[i]);
  }
}

/* ---- Q5_K super-block decode ------------------------------------------- */

/* One Q5_K super-block (176 bytes: f16 d, f16 dmin, 12 packed scale/min
 * bytes, qh[32], qs[128]) -> 256 f32, as src/gguf.ts:218-256 evaluates it:
 * group g (0..3) of 64 elements takes the low nibbles of qs[32g..32g+31]
 * plus bit 2g of qh[l] as the 5th bit (value 16), then the high nibbles plus
 * bit 2g+1; d1*(q) - min1 in f64, one rounding to f32 at the store. */
static void dequant_q5k_block_f32(const uint8_t* blk, float* out) {
  const double d = f16_to_f64((uint16_t)(blk[0] | (blk[1] << 8)));
  const double dmin = f16_to_f64((uint16_t)(blk[2] | (blk[3] << 8)));
  const uint8_t* scales = blk + 4;
  const uint8_t* qh = blk + 16;
  const uint8_t* qs = blk + 48;
  for (int g = 0; g < 4; ++g) {
    int sc1, m1, sc2, m2;
    get_scale_min(scales, 2 * g, &sc1, &m1);
    get_scale_min(scales, 2 * g + 1, &sc2, &m2);
    const double d1 = d * sc1, min1 = dmin * m1;
    const double d2 = d * sc2, min2 = dmin * m2;
    const int u1 = 1 << (2 * g), u2 = 2 << (2 * g);
    for (int l = 0; l < 32; ++l) {
      const int q = (qs[32 * g + l] & 0x0f) + ((qh[l] & u1) ? 16 : 0);
      out[64 * g + l] = (float)(d1 * q - min1);
    }
    for (int l = 0; l < 32; ++l) {
      const int q = ((qs[32 * g + l] >> 4) & 0x0f) + ((qh[l] & u2) ? 16 : 0);
      out[64 * g + 32 + l] = (float)(d2 * q - min2);
    }
  }
}

ORC_API void orc_q5k_dequant_f32(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; ++b) dequant_q5k_block_f32(blocks + b * Q5K_BLOCK_BYTES, out + b * QK_K);
}

/* Q5_K -> f16 bit patterns: the per-layer embedding values the reference
 * uploads (decodeQ5_KBlock then f32ToF16Array, RNE; src/engine.ts:683-702). */
ORC_API void orc_q5k_dequant_f16(const uint8_t* blocks, int64_t n_blocks, uint16_t* out) {
  float tmp[QK_K];
  for (int64_t b = 0; b < n_blocks; ++b) {
    dequant_q5k_block_f32(blocks + b * Q5K_BLOCK_BYTES, tmp);
    for (int i = 0; i < QK_K; ++i) out[b * QK_K + i] = orc_f32_to_f16_rne(tmp[i]);
  }
}

/* shaders/ple_stage1_fuse.wgsl:16-38 for T tokens and `layers` layers, with
 * D = 256 (one Q5_K super-block per layer per token):
 *   rms = sqrt(sum_i projected[L*D+i]^2 / D + eps)   (256-lane tree sum)
 *   out[L*D+i] = ((projected[L*D+i] / rms) * f32(norm_w[i])
 *                 + f32(embed_L[token*D+i]) * sqrt(D)) * inverseSqrt(2)
 * where embed_L[token*D+i] is element i of super-block token*layers + L of
 * the Q5_K table, decoded and rounded to f16 as the upload does.  The
 * per-lane squares, the tree order and the f32 operation order follow the
 * shader; inverseSqrt(2) is taken as 1/sqrt(2) rounded to f32. */
ORC_API void orc_ple_stage1(const uint8_t* table, const uint32_t* tokens, int64_t T, int64_t layers,
                            const float* projected, const uint16_t* norm_w, float eps, float* out) {
  enum { D = 256 };
  float emb[QK_K];
  float sq[D];
  const float sqrt_d = sqrtf((float)D);
  const float inv_sqrt2 = (float)(1.0 / sqrt(2.0));
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t L = 0; L < layers; ++L) {
      const float* pr = projected + (t * layers + L) * D;
      float* o = out + (t * layers + L) * D;
      dequant_q5k_block_f32(table + ((int64_t)tokens[t] * layers + L) * Q5K_BLOCK_BYTES, emb);
      for (int i = 0; i < D; ++i) sq[i] = pr[i] * pr[i];
      for (int stride = 128; stride > 0; stride >>= 1)
        for (int i = 0; i < stride; ++i) sq[i] = sq[i] + sq[i + stride];
      const float rms = sqrtf(sq[0] / (float)D + eps);
      for (int i = 0; i < D; ++i) {
        const float nw = orc_f16_to_f32(norm_w[i]);
        const float e16 = orc_f16_to_f32(orc_f32_to_f16_rne(emb[i]));
        const float proj_normed = (pr[i] / rms) * nw;
        const float embed_val = e16 * sqrt_d;
        o[i] = (proj_normed + embed_val) * inv_sqrt2;
      }
    }
  }
}

/* ---- matmul_quant ------------------------------------------------------ */

/* One output row in the order of shaders/matmul_quant.wgsl:31-53: thread t of
 * a 256-wide workgroup accumulates k = t, t+256, ... in f32 (multiply, then
 * add), then an 8-level tree halves the 256 partials. `w` is the row's f32
 * weights (already f16-rounded). */
static float row_dot_wgsl(const float* w, const float* x, int64_t N) {
  float part[256];
  for (int t = 0; t < 256; ++t) {
    float acc = 0.0f;
    for (int64_t k = t; k < N; k += 256) {
      const float p = w[k] * x[k];
      acc = acc + p;
    }
    part[t] = acc;
  }
  for (int stride = 128; stride > 0; stride >>= 1)
    for (int t = 0; t < stride; ++t) part[t] = part[t] + part[t + stride];
  return part[0];
}

/* Row-parallel driver: rows [0, M) are split into n_threads contiguous
 * ranges, one pthread each (n_threads <= 0 means every online core). */
typedef void (*row_fn)(void* arg, int64_t m0, int64_t m1);
typedef struct {
  row_fn fn;
  void* arg;
  int64_t m0, m1;
} row_job;

static void* row_job_main(void* p) {
  row_job* j = (row_job*)p;
  j->fn(j->arg, j->m0, j->m1);
  return NULL;
}

static int resolve_threads(int n_threads) {
  if (n_threads <= 0) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    n_threads = n > 0 ? (int)n : 1;
  }
  return n_threads > 256 ? 256 : n_threads;
}

static void parallel_rows(row_fn fn, void* arg, int64_t M, int n_threads) {
  n_threads = resolve_threads(n_threads);
  if (n_threads > M) n_threads = M > 0 ? (int)M : 1;
  if (n_threads <= 1) {
    fn(arg, 0, M);
    return;
  }
  pthread_t th[256];
  row_job jobs[256];
  for (int t = 0; t < n_threads; ++t) {
    jobs[t].fn = fn;
    jobs[t].arg = arg;
    jobs[t].m0 = M * t / n_threads;
    jobs[t].m1 = M * (t + 1) / n_threads;
    pthread_create(&th[t], NULL, row_job_main, &jobs[t]);
  }
  for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}

typedef struct {
  const void* w;
  const float* x;
  void* y;
  double* wnorm;
  int64_t M, N, batch;
  int fmt; /* weight format of `w` for the fused GEMVs: 0 = Q4_K, 1 = Q6_K */
} gemv_args;

static void rows_matmul_f16(void* p, int64_t m0, int64_t m1) {
  const gemv_args* a = (const gemv_args*)p;
  const uint16_t* w16 = (const uint16_t*)a->w;
  float* y = (float*)a->y;
  float* w = (float*)malloc(sizeof(float) * (size_t)a->N);
  for (int64_t m = m0; m < m1; ++m) {
    for (int64_t k = 0; k < a->N; ++k) w[k] = (float)f16_to_f64(w16[m * a->N + k]);
    for (int64_t b = 0; b < a->batch; ++b) y[b * a->M + m] = row_dot_wgsl(w, a->x + b * a->N, a->N);
  }
  free(w);
}

/* y[m] = matmul_quant(w16, x) for every m < M.  w16: f16 bit patterns [M*N]
 * (the reference's GPU weight buffer), x: f32 [N], y: f32 [M].  With
 * batch > 1, x is [batch*N] and y is [batch*M] (one reference dispatch per
 * activation row). */
ORC_API void orc_matmul_quant_f16(const uint16_t* w16, const float* x, float* y, int64_t M, int64_t N,
                                  int64_t batch, int n_threads) {
  gemv_args a = {w16, x, y, NULL, M, N, batch, 0};
  parallel_rows(rows_matmul_f16, &a, M, n_threads);
}

/* f32 -> nearest f16 value, returned as f32.  With F16C the hardware
 * conversion (round-to-nearest-even immediate) is used; it is bit-identical
 * to orc_f32_to_f16_rne, which the tests check on both builds. */
static inline float round_f16(float v) {
#ifdef __F16C__
  return _cvtsh_ss(_cvtss_sh(v, _MM_FROUND_TO_NEAREST_INT));
#else
  return (float)f16_to_f64(orc_f32_to_f16_rne(v));
#endif
}

/* Decode one row of Q4_K into f16-rounded f32 weights (the values the
 * reference GPU multiplies). */
static void decode_row_f16r(const uint8_t* row, int64_t N, int fmt, float* w) {
  const int64_t nb = N / QK_K;
  for (int64_t b = 0; b < nb; ++b) {
    if (fmt == 1)
      dequant_q6k_block_f32(row + b * Q6K_BLOCK_BYTES, w + b * QK_K);
    else
      dequant_block_f32(row + b * Q4K_BLOCK_BYTES, w + b * QK_K);
  }
  for (int64_t k = 0; k < N; ++k) w[k] = round_f16(w[k]);
}

static int64_t row_bytes_of(int64_t N, int fmt) {
  return N / QK_K * (fmt == 1 ? Q6K_BLOCK_BYTES : Q4K_BLOCK_BYTES);
}

static void rows_q4k_gemv(void* p, int64_t m0, int64_t m1) {
  const gemv_args* a = (const gemv_args*)p;
  const int64_t row_bytes = row_bytes_of(a->N, a->fmt);
  float* y = (float*)a->y;
  float* w = (float*)malloc(sizeof(float) * (size_t)a->N);
  for (int64_t m = m0; m < m1; ++m) {
    decode_row_f16r((const uint8_t*)a->w + m * row_bytes, a->N, a->fmt, w);
    for (int64_t b = 0; b < a->batch; ++b) y[b * a->M + m] = row_dot_wgsl(w, a->x + b * a->N, a->N);
  }
  free(w);
}

/* Fused variant: Q4_K bytes in, y out, per row: decode -> RNE f16 -> the WGSL
 * dot.  The same arithmetic as dequantizeQ4_K + f32ToF16Array + matmul_quant.
 * Also the timed CPU baseline ("port"). */
ORC_API void orc_q4k_gemv(const uint8_t* w_q4k, const float* x, float* y, int64_t M, int64_t N, int64_t batch,
                          int n_threads) {
  gemv_args a = {w_q4k, x, y, NULL, M, N, batch, 0};
  parallel_rows(rows_q4k_gemv, &a, M, n_threads);
}

/* The same for Q6_K bytes (GGUF layout, 210-byte super-blocks): decode
 * (dequantizeQ6_K) -> RNE f16 -> the WGSL dot. */
ORC_API void orc_q6k_gemv(const uint8_t* w_q6k, const float* x, float* y, int64_t M, int64_t N, int64_t batch,
                          int n_threads) {
  gemv_args a = {w_q6k, x, y, NULL, M, N, batch, 1};
  parallel_rows(rows_q4k_gemv, &a, M, n_threads);
}

static void rows_q4k_gemv_f64(void* p, int64_t m0, int64_t m1) {
  const gemv_args* a = (const gemv_args*)p;
  const int64_t row_bytes = row_bytes_of(a->N, a->fmt);
  double* y = (double*)a->y;
  float* w = (float*)malloc(sizeof(float) * (size_t)a->N);
  for (int64_t m = m0; m < m1; ++m) {
    decode_row_f16r((const uint8_t*)a->w + m * row_bytes, a->N, a->fmt, w);
    if (a->wnorm) {
      double nrm = 0.0;
      for (int64_t k = 0; k < a->N; ++k) nrm += (double)w[k] * (double)w[k];
      a->wnorm[m] = sqrt(nrm);
    }
    for (int64_t b = 0; b < a->batch; ++b) {
      const float* xb = a->x + b * a->N;
      double acc = 0.0;
      for (int64_t k = 0; k < a->N; ++k) acc += (double)w[k] * (double)xb[k];
      y[b * a->M + m] = acc;
    }
  }
  free(w);
}

/* Error-bound companion: the same f16-rounded weights, dot product in f64.
 * Also returns ||w_row||_2 per row (for the per-output tolerance term). */
ORC_API void orc_q4k_gemv_f64(const uint8_t* w_q4k, const float* x, double* y, double* wnorm, int64_t M,
                              int64_t N, int64_t batch, int n_threads) {
  gemv_args a = {w_q4k, x, y, wnorm, M, N, batch, 0};
  parallel_rows(rows_q4k_gemv_f64, &a, M, n_threads);
}

ORC_API void orc_q6k_gemv_f64(const uint8_t* w_q6k, const float* x, double* y, double* wnorm, int64_t M,
                              int64_t N, int64_t batch, int n_threads) {
  gemv_args a = {w_q6k, x, y, wnorm, M, N, batch, 1};
  parallel_rows(rows_q4k_gemv_f64, &a, M, n_threads);
}

/* ---- LM-head consumers -------------------------------------------------- */

/* shaders/logit_softcap.wgsl:13-15: x/cap, clamp to [-15, 15], tanh, *cap. */
ORC_API void orc_logit_softcap(float* logits, int64_t n, float cap) {
  for (int64_t i = 0; i < n; ++i) {
    float v = logits[i] / cap;
    if (v < -15.0f) v = -15.0f;
    if (v > 15.0f) v = 15.0f;
    logits[i] = tanhf(v) * cap;
  }
}

/* shaders/argmax.wgsl:12-33: 256 lanes, lane t scans i = t, t+256, ... keeping
 * the first strict maximum (start -1e30, index 0); then a tree where the
 * partner only wins if strictly greater, so ties keep the lower lane. */
ORC_API uint32_t orc_argmax(const float* logits, int64_t n) {
  float mx[256];
  uint32_t ix[256];
  for (int t = 0; t < 256; ++t) {
    float lm = -1e30f;
    uint32_t li = 0;
    for (int64_t i = t; i < n; i += 256)
      if (logits[i] > lm) {
        lm = logits[i];
        li = (uint32_t)i;
      }
    mx[t] = lm;
    ix[t] = li;
  }
  for (int stride = 128; stride > 0; stride >>= 1)
    for (int t = 0; t < stride; ++t)
      if (mx[t + stride] > mx[t]) {
        mx[t] = mx[t + stride];
        ix[t] = ix[t + stride];
      }
  return ix[0];
}

/* shaders/topk256.wgsl:10-20: for each residue class t = i mod 256, the first
 * strict maximum and its index (lanes start at -1e30 / 0). */
ORC_API void orc_topk256(const float* logits, int64_t n, float* vals, uint32_t* idx) {
  for (int t = 0; t < 256; ++t) {
    float lm = -1e30f;
    uint32_t li = 0;
    for (int64_t i = t; i < n; i += 256)
      if (logits[i] > lm) {
        lm = logits[i];
        li = (uint32_t)i;
      }
    vals[t] = lm;
    idx[t] = li;
  }
}

/* shaders/gelu_mul.wgsl:14-16: GELU(tanh) of gate times up, f32. */
ORC_API void orc_gelu_mul(const float* gate, const float* up, float* out, int64_t n) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  for (int64_t i = 0; i < n; ++i) {
    const float x = gate[i];
    float a = k0 * x * (1.0f + k1 * x * x);
    if (a < -15.0f) a = -15.0f;
    if (a > 15.0f) a = 15.0f;
    const float g = 0.5f * x * (1.0f + tanhf(a));
    out[i] = g * up[i];
  }
}

ORC_API int orc_max_threads(void) { return resolve_threads(0); }
