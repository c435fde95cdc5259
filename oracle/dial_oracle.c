/*
 * dial_oracle.c -- CPU restatement of DIAL's quantized-linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * dial-8b-orin_b200/csrc: only tests/, __graft_entry__.smoke() and the CPU
 * baseline leg of bench.py load it.  No product code path calls it, and the
 * product library fails loudly instead of falling back to it.
 *
 * Parity anchors (paths are inside the reference project lisa301/DIAL-8B-orin):
 *  - W8A16 quantiser: dial-core/src/models/qwen3_vl/worker_w8a16.rs:322-341
 *    (CPU twin dial-core/src/models/qwen3_vl/text.rs:265-278).  Pinned by the
 *    reference's own known-answer test worker_w8a16.rs:483-516, restated in
 *    tests/test_oracle_golden.py.
 *  - W8A16 linear: worker_w8a16.rs:158-181 and :202-222 -- f32 accumulation of
 *    f32(int8) * f32(f16 x), scale applied after the sum, f16 round-to-nearest.
 *  - GGUF Q4_0 / Q8_0: the arithmetic lives in candle-core 0.11.0
 *    (Cargo.lock:509-512, not vendored).  Call sites: worker_gguf.rs:500-505
 *    (QMatMul::from_arc), :593 and :609-610 (forward), :60-61 (dequantize).
 *    Restated from the published GGML block format (ggml-quants reference
 *    quantisers quantize_row_q4_0_ref / quantize_row_q8_0_ref and candle's
 *    k_quants vec_dot_q4_0_q8_0 / vec_dot_q8_0_q8_0).  Pinned against the
 *    independent `gguf` 0.19.0 Python implementation through the fixtures in
 *    tests/golden/ (script: tests/golden/make_golden.py).  candle equality
 *    itself cannot be checked here (no Rust toolchain, candle not vendored).
 *  - GGUF Q4_K / Q6_K (the reference's Q4_K_M files, docs/worker_gguf.md:1-6):
 *    dequantisers restated from the public GGML definitions, pinned bit-for-bit
 *    to gguf 0.19.0 (tests/golden/make_golden_k.py); an exact linear and the
 *    GGML/candle CPU arithmetic (Q8_K activations), the latter unpinned.
 *  - Decoder glue: text.rs:1478-1596 (attention order), text.rs:1636-1688
 *    (residuals), text.rs:816-820 (SwiGLU), llama3/cache.rs:24-64 (RoPE
 *    tables), cache.rs:149-217 (KV append), qwen3_vl.rs:130-143 (argmax).
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).  Contraction
 * must stay off: the GGML quantisers compute `x*id + 8.5f` as two roundings.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* half / bfloat16 conversions (IEEE round-to-nearest-even)                  */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return bits_f32(sign);
    /* subnormal: value = man * 2^-24 (exact in f32) */
    float v = (float)man * 5.9604644775390625e-8f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
  return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

static inline uint16_t f2h(float f) {
  uint32_t x = f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
  if (ax < 0x38800000u) {
    /* result is subnormal or zero: round ax * 2^24 to an integer (RNE) */
    float a = bits_f32(ax);
    float scaled = a * 16777216.0f; /* exact: power of two */
    /* nearbyintf uses the current rounding mode (nearest-even by default) */
    uint32_t m = (uint32_t)nearbyintf(scaled);
    return (uint16_t)(sign | m);
  }
  uint32_t exp = (ax >> 23) - 112u;
  uint32_t man = ax & 0x7fffffu;
  uint32_t h = (exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
  return (uint16_t)(sign | h);
}

static inline float bf2f(uint16_t b) { return bits_f32((uint32_t)b << 16); }

static inline uint16_t f2bf(float f) {
  uint32_t x = f32_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

/* dtype codes shared with include/dial_cuda.h */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

static inline float load_act(const void* p, int dt, int64_t i) {
  switch (dt) {
    case ORC_F16: return h2f(((const uint16_t*)p)[i]);
    case ORC_BF16: return bf2f(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}

static inline void store_act(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case ORC_F16: ((uint16_t*)p)[i] = f2h(v); break;
    case ORC_BF16: ((uint16_t*)p)[i] = f2bf(v); break;
    default: ((float*)p)[i] = v; break;
  }
}

ORC_API void orc_f32_to_f16(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2h(in[i]);
}
ORC_API void orc_f16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]);
}
ORC_API void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}
ORC_API void orc_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]);
}

ORC_API int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* W8A16: per-output-row symmetric int8 (worker_w8a16.rs:322-341)           */
/* ------------------------------------------------------------------------ */

/* Rust's f32::round: half away from zero == C roundf. */
static inline int8_t w8a16_q(float v, float inv_scale) {
  float r = roundf(v * inv_scale);
  if (r > 127.0f) r = 127.0f;
  if (r < -127.0f) r = -127.0f;
  return (int8_t)r;
}

/*
 * w: [N, K] row-major, dtype wdt (F32, or F16 which the reference widens to
 * f32 first, worker_w8a16.rs:323-327).  q: [N, K] int8.  scale_f32: [N].
 * scale_f16 (optional): [N], the f32 scale rounded to f16 -- the int8 values
 * are always those of the f32 scale, so they are identical for either scale
 * dtype.
 */
ORC_API void orc_w8a16_quantize(const void* w, int wdt, int64_t N, int64_t K, int8_t* q,
                                float* scale_f32, uint16_t* scale_f16) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float max_abs = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      float v = fabsf(load_act(w, wdt, n * K + k));
      max_abs = max_abs > v ? max_abs : v; /* fold(0, max) */
    }
    float scale = max_abs > 0.0f ? max_abs / 127.0f : 1.0f;
    float inv = 1.0f / scale;
    for (int64_t k = 0; k < K; ++k) q[n * K + k] = w8a16_q(load_act(w, wdt, n * K + k), inv);
    scale_f32[n] = scale;
    if (scale_f16) scale_f16[n] = f2h(scale);
  }
}

/* Dequantised weight value q * scale, in f32 (one rounding, bit-exact target). */
ORC_API void orc_w8a16_dequantize(const int8_t* q, const void* scale, int sdt, int64_t N,
                                  int64_t K, float* w) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float s = load_act(scale, sdt, n);
    for (int64_t k = 0; k < K; ++k) w[n * K + k] = (float)q[n * K + k] * s;
  }
}

/*
 * y[m, n] = (sum_k f32(q[n,k]) * f32(x[m,k])) * scale[n]   (worker_w8a16.rs:158-181)
 * The sum is accumulated in double here (the order-independent reference the
 * GPU result is compared with); y_out gets the pre-rounding f32 value and,
 * if y_half is given, its f16 (xdt F16) / bf16 (xdt BF16) rounding.
 */
ORC_API void orc_w8a16_linear(const void* x, int xdt, const int8_t* q, const void* scale,
                              int sdt, int64_t M, int64_t K, int64_t N, float* y_out,
                              uint16_t* y_half) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      const int8_t* row = q + n * K;
      for (int64_t k = 0; k < K; ++k) acc += (double)row[k] * (double)load_act(x, xdt, m * K + k);
      float v = (float)acc * load_act(scale, sdt, n);
      y_out[m * N + n] = v;
      if (y_half) y_half[m * N + n] = (xdt == ORC_BF16) ? f2bf(v) : f2h(v);
    }
  }
}

/* Same linear with the f32 sequential accumulation the reference kernel's
 * single-thread order would give (used by the CPU baseline timing, which wants
 * the reference's arithmetic cost, not double precision). */
ORC_API void orc_w8a16_linear_f32(const uint16_t* x_f16, const int8_t* q, const float* scale,
                                  int64_t M, int64_t K, int64_t N, uint16_t* y_f16) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t i = 0; i < M * K; ++i) xf[i] = h2f(x_f16[i]);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      const int8_t* row = q + n * K;
      const float* xr = xf + m * K;
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += (float)row[k] * xr[k];
      y_f16[m * N + n] = f2h(acc * scale[n]);
    }
  }
  free(xf);
}

/* ------------------------------------------------------------------------ */
/* GGUF Q4_0 / Q8_0 (published GGML block format)                            */
/*   Q4_0 block: { f16 d; u8 qs[16]; }  18 bytes / 32 weights                 */
/*     element j     = (qs[j] & 0xF) - 8,  element j+16 = (qs[j] >> 4) - 8     */
/*   Q8_0 block: { f16 d; i8 qs[32]; }  34 bytes / 32 weights                 */
/* ------------------------------------------------------------------------ */

enum { ORC_Q4_0 = 2, ORC_Q8_0 = 8 };
#define QK 32

static void q4_0_block(const float* x, uint8_t* out) {
  float amax = 0.0f, maxv = 0.0f;
  for (int j = 0; j < QK; ++j) {
    float v = x[j];
    if (amax < fabsf(v)) { amax = fabsf(v); maxv = v; }
  }
  float d = maxv / -8.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint16_t dh = f2h(d);
  out[0] = (uint8_t)(dh & 0xff);
  out[1] = (uint8_t)(dh >> 8);
  for (int j = 0; j < QK / 2; ++j) {
    float x0 = x[j] * id;
    float x1 = x[QK / 2 + j] * id;
    x0 = x0 + 8.5f;
    x1 = x1 + 8.5f;
    int i0 = (int)x0; /* C truncation == np.trunc for these finite values */
    int i1 = (int)x1;
    if (i0 > 15) i0 = 15;
    if (i1 > 15) i1 = 15;
    if (i0 < 0) i0 = 0; /* only reachable for NaN-free but id==0 inputs */
    if (i1 < 0) i1 = 0;
    out[2 + j] = (uint8_t)(i0 | (i1 << 4));
  }
}

/* GGML quantize_row_q8_0_ref: d = amax/127, q = roundf(x / d) (via x * (1/d)). */
static void q8_0_block(const float* x, uint8_t* out) {
  float amax = 0.0f;
  for (int j = 0; j < QK; ++j) {
    float v = fabsf(x[j]);
    amax = amax > v ? amax : v;
  }
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint16_t dh = f2h(d);
  out[0] = (uint8_t)(dh & 0xff);
  out[1] = (uint8_t)(dh >> 8);
  for (int j = 0; j < QK; ++j) out[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

ORC_API int64_t orc_gguf_block_bytes(int type) {
  return type == ORC_Q4_0 ? 18 : type == ORC_Q8_0 ? 34 : -1;
}

/* w: [N, K] f32, K % 32 == 0.  blocks: [N, K/32] blocks in native layout. */
ORC_API int orc_gguf_quantize(const float* w, int type, int64_t N, int64_t K, uint8_t* blocks) {
  int64_t bb = orc_gguf_block_bytes(type);
  if (bb < 0 || K % QK) return -1;
  int64_t nb = K / QK;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      const float* src = w + n * K + b * QK;
      uint8_t* dst = blocks + (n * nb + b) * bb;
      if (type == ORC_Q4_0) q4_0_block(src, dst); else q8_0_block(src, dst);
    }
  }
  return 0;
}

static inline float block_d(const uint8_t* blk) { return h2f((uint16_t)(blk[0] | (blk[1] << 8))); }

static inline int block_q(const uint8_t* blk, int type, int j) {
  if (type == ORC_Q8_0) return (int)(int8_t)blk[2 + j];
  return j < QK / 2 ? (int)(blk[2 + j] & 0xf) - 8 : (int)(blk[2 + j - QK / 2] >> 4) - 8;
}

/* Dequantised value d * q in f32 (GGML dequantize_row_*; bit-exact target). */
ORC_API int orc_gguf_dequantize(const uint8_t* blocks, int type, int64_t N, int64_t K, float* w) {
  int64_t bb = orc_gguf_block_bytes(type);
  if (bb < 0 || K % QK) return -1;
  int64_t nb = K / QK;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      const uint8_t* blk = blocks + (n * nb + b) * bb;
      float d = block_d(blk);
      for (int j = 0; j < QK; ++j) w[n * K + b * QK + j] = d * (float)block_q(blk, type, j);
    }
  }
  return 0;
}

/* Exact linear on dequantised weights, double accumulation: y = x . deq(W)^T */
ORC_API int orc_gguf_linear_exact(const void* x, int xdt, const uint8_t* blocks, int type,
                                  int64_t M, int64_t K, int64_t N, double* y) {
  int64_t bb = orc_gguf_block_bytes(type);
  if (bb < 0 || K % QK) return -1;
  int64_t nb = K / QK;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = blocks + (n * nb + b) * bb;
        double d = (double)block_d(blk);
        double s = 0.0;
        for (int j = 0; j < QK; ++j)
          s += (double)block_q(blk, type, j) * (double)load_act(x, xdt, m * K + b * QK + j);
        acc += d * s;
      }
      y[m * N + n] = acc;
    }
  }
  return 0;
}

/*
 * candle's CPU QMatMul semantics (k_quants.rs matmul + vec_dot): each
 * activation row is quantised to Q8_0 blocks (same quantiser as weights,
 * f16 d), then per block an exact integer dot, scaled in f32:
 *     sumf += (f32)sumi * d_w * d_x          (sequential over blocks)
 * y is f32 (the QMatMul output dtype for f32 input).
 */
ORC_API int orc_gguf_linear_candle(const void* x, int xdt, const uint8_t* blocks, int type,
                                   int64_t M, int64_t K, int64_t N, float* y) {
  int64_t bb = orc_gguf_block_bytes(type);
  if (bb < 0 || K % QK) return -1;
  int64_t nb = K / QK;
  uint8_t* xq = (uint8_t*)malloc((size_t)(M * nb * 34));
  float* xrow = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t i = 0; i < M * K; ++i) xrow[i] = load_act(x, xdt, i);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t b = 0; b < nb; ++b) q8_0_block(xrow + m * K + b * QK, xq + (m * nb + b) * 34);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      float sumf = 0.0f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* wb = blocks + (n * nb + b) * bb;
        const uint8_t* xb = xq + (m * nb + b) * 34;
        int sumi = 0;
        for (int j = 0; j < QK; ++j) sumi += block_q(wb, type, j) * (int)(int8_t)xb[2 + j];
        sumf += (float)sumi * block_d(wb) * block_d(xb);
      }
      y[m * N + n] = sumf;
    }
  }
  free(xrow);
  free(xq);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* GGUF K-quants, native GGML super-blocks of 256 weights (the reference's     */
/* deployed Q4_K_M files: docs/worker_gguf.md:1-6; loaded by                  */
/* load_worker_gguf_linear worker_gguf.rs:462-522, arithmetic in candle-core   */
/* 0.11.0, not vendored).  Restated from the public GGML definitions           */
/* (block_q4_K / block_q6_K, dequantize_row_q4_K / dequantize_row_q6_K) and    */
/* pinned against the independent gguf 0.19.0 Python dequantisers through      */
/* tests/golden/gguf_q4_k_q6_k.npz (script: tests/golden/make_golden_k.py).   */
/*   Q4_K 144 B: f16 d, f16 dmin, u8 scales[12], u8 qs[128]                    */
/*   Q6_K 210 B: u8 ql[128], u8 qh[64], i8 scales[16], f16 d                   */
/* ------------------------------------------------------------------------ */
#define ORC_Q4_K 12
#define ORC_Q6_K 14
#define QKK 256

ORC_API int64_t orc_gguf_k_block_bytes(int type) {
  return type == ORC_Q4_K ? 144 : type == ORC_Q6_K ? 210 : -1;
}

/* 6-bit scale and min of Q4_K sub-block j (GGML get_scale_min_k4) */
static void q4_k_scale_min(const uint8_t* q, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* One super-block to 256 f32 values, every product / difference rounded on
 * its own (the file is built with -ffp-contract=off). */
static void k_block_dequant(const uint8_t* blk, int type, float* y) {
  if (type == ORC_Q4_K) {
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
    const uint8_t* scales = blk + 4;
    const uint8_t* q = blk + 16;
    for (int c = 0; c < 4; ++c) {  /* 64 weights: 32 low nibbles, then 32 high */
      int sc, m;
      q4_k_scale_min(scales, 2 * c, &sc, &m);
      const float d1 = d * (float)sc, m1 = dmin * (float)m;
      q4_k_scale_min(scales, 2 * c + 1, &sc, &m);
      const float d2 = d * (float)sc, m2 = dmin * (float)m;
      for (int l = 0; l < 32; ++l) y[64 * c + l] = d1 * (float)(q[32 * c + l] & 0xF) - m1;
      for (int l = 0; l < 32; ++l) y[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - m2;
    }
  } else {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* sc = (const int8_t*)(blk + 192);
    const float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
    for (int h = 0; h < 2; ++h) {  /* 128 weights from 64 ql bytes, 32 qh bytes, 8 scales */
      const uint8_t* L = ql + 64 * h;
      const uint8_t* H = qh + 32 * h;
      const int8_t* S = sc + 8 * h;
      for (int l = 0; l < 32; ++l) {
        const int is = l / 16;
        const int q1 = (int)((L[l] & 0xF) | (((H[l] >> 0) & 3) << 4)) - 32;
        const int q2 = (int)((L[l + 32] & 0xF) | (((H[l] >> 2) & 3) << 4)) - 32;
        const int q3 = (int)((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32;
        const int q4 = (int)((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32;
        float* o = y + 128 * h;
        o[l] = d * (float)S[is] * (float)q1;
        o[l + 32] = d * (float)S[is + 2] * (float)q2;
        o[l + 64] = d * (float)S[is + 4] * (float)q3;
        o[l + 96] = d * (float)S[is + 6] * (float)q4;
      }
    }
  }
}

/* blocks [N, K/256] native -> w [N, K] f32 */
ORC_API int orc_gguf_k_dequantize(const uint8_t* blocks, int type, int64_t N, int64_t K, float* w) {
  const int64_t bb = orc_gguf_k_block_bytes(type);
  if (bb < 0 || K % QKK) return -1;
  const int64_t nb = K / QKK;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t b = 0; b < nb; ++b) k_block_dequant(blocks + (n * nb + b) * bb, type, w + n * K + b * QKK);
  return 0;
}

/* y = x . deq(W)^T, double accumulation over the f32 dequantised weights */
ORC_API int orc_gguf_k_linear_exact(const void* x, int xdt, const uint8_t* blocks, int type,
                                    int64_t M, int64_t K, int64_t N, double* y) {
  const int64_t bb = orc_gguf_k_block_bytes(type);
  if (bb < 0 || K % QKK) return -1;
  const int64_t nb = K / QKK;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float wrow[QKK];
    for (int64_t m = 0; m < M; ++m) y[m * N + n] = 0.0;
    for (int64_t b = 0; b < nb; ++b) {
      k_block_dequant(blocks + (n * nb + b) * bb, type, wrow);
      for (int64_t m = 0; m < M; ++m) {
        double s = 0.0;
        for (int j = 0; j < QKK; ++j) s += (double)wrow[j] * (double)load_act(x, xdt, m * K + b * QKK + j);
        y[m * N + n] += s;
      }
    }
  }
  return 0;
}

/*
 * The CPU arithmetic of GGML / candle k_quants for Q4_K and Q6_K (the scalar
 * vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K): each activation row is quantised per
 * 256 to Q8_K blocks (f32 d, int8 qs[256], int16 sums of every 16), with
 * iscale = -128/max (max = the element of largest magnitude, sign kept),
 * q = min(127, round-half-even(iscale * x)), d = 1/iscale; then per weight
 * block an exact integer dot per sub-block times its 6-bit (Q4_K) or int8
 * (Q6_K) scale, scaled in f32:
 *   Q4_K: sumf += (d_w*d_x) * sum_j sc_j * dot_j  -  (dmin_w*d_x) * sum_j m_j * bsum_j
 *   Q6_K: sumf += (d_w*d_x) * sum_j sc_j * dot_j          (q6 - 32 in the dots)
 * The published algorithm, restated; candle-core 0.11.0 is not vendored, so
 * equality with its code (Q8_K scale and rounding rule, float order) is
 * unverified.  Used as the CPU baseline of the K-quant decode and as a second,
 * looser oracle.  y is f32.
 */
static void q8_k_block(const float* x, float* d, int8_t* qs, int16_t* bsums) {
  float amax = 0.0f, mx = 0.0f;
  for (int j = 0; j < QKK; ++j) {
    const float ax = fabsf(x[j]);
    if (ax > amax) {
      amax = ax;
      mx = x[j];
    }
  }
  if (amax == 0.0f) {
    *d = 0.0f;
    memset(qs, 0, QKK);
    memset(bsums, 0, 16 * sizeof(int16_t));
    return;
  }
  const float iscale = -128.0f / mx;
  for (int j = 0; j < QKK; ++j) {
    const long v = lrintf(iscale * x[j]);
    qs[j] = (int8_t)(v > 127 ? 127 : v);
  }
  for (int g = 0; g < 16; ++g) {
    int s = 0;
    for (int j = 0; j < 16; ++j) s += qs[16 * g + j];
    bsums[g] = (int16_t)s;
  }
  *d = 1.0f / iscale;
}

ORC_API int orc_gguf_k_linear_candle(const void* x, int xdt, const uint8_t* blocks, int type,
                                     int64_t M, int64_t K, int64_t N, float* y) {
  const int64_t bb = orc_gguf_k_block_bytes(type);
  if (bb < 0 || K % QKK) return -1;
  const int64_t nb = K / QKK;
  float* xd = (float*)malloc(sizeof(float) * (size_t)(M * nb));
  int8_t* xq = (int8_t*)malloc((size_t)(M * K));
  int16_t* xs = (int16_t*)malloc(sizeof(int16_t) * (size_t)(M * nb * 16));
  float buf[QKK];
  for (int64_t m = 0; m < M; ++m)
    for (int64_t b = 0; b < nb; ++b) {
      for (int j = 0; j < QKK; ++j) buf[j] = load_act(x, xdt, m * K + b * QKK + j);
      q8_k_block(buf, xd + m * nb + b, xq + m * K + b * QKK, xs + (m * nb + b) * 16);
    }
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      float sumf = 0.0f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* wb = blocks + (n * nb + b) * bb;
        const int8_t* q8 = xq + m * K + b * QKK;
        const float dx = xd[m * nb + b];
        if (type == ORC_Q4_K) {
          const uint8_t* q4 = wb + 16;
          int isum = 0, msum = 0;
          for (int c = 0; c < 4; ++c) {
            int sc0, m0, sc1, m1, dot0 = 0, dot1 = 0;
            q4_k_scale_min(wb + 4, 2 * c, &sc0, &m0);
            q4_k_scale_min(wb + 4, 2 * c + 1, &sc1, &m1);
            for (int l = 0; l < 32; ++l) {
              dot0 += (q4[32 * c + l] & 0xF) * q8[64 * c + l];
              dot1 += (q4[32 * c + l] >> 4) * q8[64 * c + 32 + l];
            }
            isum += sc0 * dot0 + sc1 * dot1;
            const int16_t* bs = xs + (m * nb + b) * 16 + 4 * c;
            msum += m0 * (bs[0] + bs[1]) + m1 * (bs[2] + bs[3]);
          }
          const float d = h2f((uint16_t)(wb[0] | (wb[1] << 8))) * dx;
          const float dmin = h2f((uint16_t)(wb[2] | (wb[3] << 8))) * dx;
          sumf += d * (float)isum;
          sumf -= dmin * (float)msum;
        } else {
          const int8_t* sc = (const int8_t*)(wb + 192);
          int isum = 0;
          for (int h = 0; h < 2; ++h) {
            const uint8_t* L = wb + 64 * h;
            const uint8_t* H = wb + 128 + 32 * h;
            for (int g = 0; g < 4; ++g)
              for (int half = 0; half < 2; ++half) {
                int dot = 0;
                for (int ll = 0; ll < 16; ++ll) {
                  const int l = 16 * half + ll;
                  const int lo = (g & 1) ? L[l + 32] : L[l];
                  const int q = (int)(((g >> 1) ? (lo >> 4) : (lo & 0xF)) | (((H[l] >> (2 * g)) & 3) << 4)) - 32;
                  dot += q * q8[128 * h + 32 * g + l];
                }
                isum += sc[8 * h + 2 * g + half] * dot;
              }
          }
          sumf += h2f((uint16_t)(wb[208] | (wb[209] << 8))) * dx * (float)isum;
        }
      }
      y[m * N + n] = sumf;
    }
  }
  free(xd);
  free(xq);
  free(xs);
  return 0;
}

/* Activation Q8_0 quantisation exposed on its own (the GPU kernels quantise
 * activations the same way before the integer block dots). */
ORC_API int orc_q8_0_quantize_rows(const void* x, int xdt, int64_t M, int64_t K,
                                   int8_t* qs, uint16_t* d) {
  if (K % QK) return -1;
  int64_t nb = K / QK;
  float buf[QK];
  uint8_t blk[34];
  for (int64_t m = 0; m < M; ++m)
    for (int64_t b = 0; b < nb; ++b) {
      for (int j = 0; j < QK; ++j) buf[j] = load_act(x, xdt, m * K + b * QK + j);
      q8_0_block(buf, blk);
      d[m * nb + b] = (uint16_t)(blk[0] | (blk[1] << 8));
      memcpy(qs + m * K + b * QK, blk + 2, QK);
    }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Decoder glue and a whole greedy decoder (f16 or bf16 activations; W8A16   */
/* or GGUF Q4_0 / Q8_0 layers; W8A16 or Q8_0 output head).                    */
/*                                                                          */
/* Order (text.rs:1636-1688 Transformer::forward: rms_1, attention +        */
/* residual, rms_2, MLP + residual; text.rs:1478-1596 QwenAttention: QKV ->  */
/* QK RMSNorm -> RoPE -> KV -> GQA attention -> O; llama3/attention.rs:41-157 */
/* the same without QK-norm; text.rs:816-820 and llama3/mlp.rs:15-21         */
/* silu(gate) * up; qwen3_vl.rs:2420-2451 ln_f -> last position -> lm_head;  */
/* qwen3_vl.rs:130-143 argmax, first index of the maximum).                  */
/*                                                                          */
/* Rounding points.  Every tensor a candle op produces is in the model dtype */
/* T (f16; bf16 as an extension), so each op's result is rounded to T once,  */
/* with the op's inner arithmetic in f32 (sums in double here):              */
/*   RMSNorm     T(h * 1/sqrt(mean(h^2) + eps) * w)                           */
/*   residual    T(a + b)                                                   */
/*   RoPE        candle rotary_emb::rope evaluates x1*c - x2*s and          */
/*               x1*s + x2*c in T (text.rs:1143-1153 with T tables,          */
/*               llama3/cache.rs:49-50): each product and the sum rounded    */
/*   attention   q.k^T is a T matmul, `/ sqrt(D)` an affine op whose          */
/*               multiplier is T(1/sqrt(D)) (text.rs:1278, :1305,            */
/*               llama3/attention.rs:125):  s = T(T(q.k) * T(1/sqrt(D)));    */
/*               softmax over the causal keys; o = T(sum_j p_j v_j)          */
/*               (text.rs:1279-1280).  The reference's probability tensor is */
/*               T as well; here p stays unrounded, like the CUDA kernel's   */
/*               single-pass softmax that never holds normalised             */
/*               probabilities (2^-11 relative per probability in f16).      */
/*   SwiGLU      T(T(silu(g)) * u)                                          */
/* Linears:                                                                  */
/*   W8A16       T(f32(sum q x) * scale)         (worker_w8a16.rs:158-181)  */
/*   GGUF        the worker's hybrid route (worker_gguf_prefill_for_dims     */
/*               worker_gguf.rs:399-421): a run of more than one position    */
/*               multiplies by the dequantised copy T(d q)                   */
/*               (build_worker_gguf_fp16_prefill_linear :423-449); a single  */
/*               position runs QMatMul (forward_worker_gguf :574-611), whose */
/*               CPU arithmetic is orc_gguf_linear_candle's (activations     */
/*               quantised to Q8_0, integer block dots, f32 block scaling).  */
/*               The output head sees one position: QMatMul.                 */
/* ------------------------------------------------------------------------ */

static inline float rnd_dt(float v, int dt) { return dt == ORC_BF16 ? bf2f(f2bf(v)) : h2f(f2h(v)); }
static inline uint16_t enc_dt(float v, int dt) { return dt == ORC_BF16 ? f2bf(v) : f2h(v); }
static inline float dec_dt(uint16_t b, int dt) { return dt == ORC_BF16 ? bf2f(b) : h2f(b); }

/* weight formats: the codes of include/dial_cuda.h (dial_weight_format) */
enum { ORC_WFMT_W8A16 = 0, ORC_WFMT_W8A16_F16S = 1 };

/* y = T(h * (1/sqrt(mean(h^2)+eps)) * w), h = T(x + res) when res != NULL */
static void rmsnorm_dt(const uint16_t* x, const uint16_t* res, uint16_t* h_out, const uint16_t* w,
                       uint16_t* y, int64_t rows, int64_t dim, float eps, int dt) {
  float* h = (float*)malloc(sizeof(float) * (size_t)dim);
  for (int64_t r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (int64_t i = 0; i < dim; ++i) {
      float v = dec_dt(x[r * dim + i], dt);
      if (res) v = rnd_dt(v + dec_dt(res[r * dim + i], dt), dt);
      h[i] = v;
      ss += (double)v * v;
    }
    const float inv = (float)(1.0 / sqrt(ss / (double)dim + (double)eps));
    for (int64_t i = 0; i < dim; ++i) {
      if (h_out) h_out[r * dim + i] = enc_dt(h[i], dt);
      y[r * dim + i] = enc_dt(h[i] * inv * dec_dt(w[i], dt), dt);
    }
  }
  free(h);
}

ORC_API void orc_rmsnorm(const uint16_t* x, const uint16_t* res, uint16_t* h_out,
                         const uint16_t* w, uint16_t* y, int64_t rows, int64_t dim, float eps) {
  rmsnorm_dt(x, res, h_out, w, y, rows, dim, eps, ORC_F16);
}

/* cos/sin [max_pos, D/2] in T: inv_freq = 1/theta^(2i/D) (f32), angle = p*inv_freq
 * (llama3/cache.rs:31-50) */
static void rope_tables_dt(uint16_t* cos_t, uint16_t* sin_t, int64_t max_pos, int D, float theta,
                           int dt) {
  for (int64_t p = 0; p < max_pos; ++p)
    for (int i = 0; i < D / 2; ++i) {
      const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)D);
      const float a = (float)p * inv;
      cos_t[p * (D / 2) + i] = enc_dt(cosf(a), dt);
      sin_t[p * (D / 2) + i] = enc_dt(sinf(a), dt);
    }
}

ORC_API void orc_rope_tables(uint16_t* cos_t, uint16_t* sin_t, int64_t max_pos, int D,
                             float theta) {
  rope_tables_dt(cos_t, sin_t, max_pos, D, theta, ORC_F16);
}

/* One head of D values: optional RMSNorm over the head, then RoPE at position p
 * with every product and sum rounded to T (candle rotary_emb::rope). */
static void head_norm_rope(const uint16_t* src, const uint16_t* nw, int qk_norm, float eps,
                           const uint16_t* cos_t, const uint16_t* sin_t, int p, int D, int dt,
                           uint16_t* dst) {
  float v[256];
  double ss = 0.0;
  for (int i = 0; i < D; ++i) { v[i] = dec_dt(src[i], dt); ss += (double)v[i] * v[i]; }
  if (qk_norm) {
    const float inv = (float)(1.0 / sqrt(ss / (double)D + (double)eps));
    for (int i = 0; i < D; ++i) v[i] = rnd_dt(v[i] * inv * dec_dt(nw[i], dt), dt);
  }
  const int half = D / 2;
  for (int i = 0; i < half; ++i) {
    const float c = dec_dt(cos_t[(int64_t)p * half + i], dt), s = dec_dt(sin_t[(int64_t)p * half + i], dt);
    const float x1 = v[i], x2 = v[i + half];
    dst[i] = enc_dt(rnd_dt(x1 * c, dt) - rnd_dt(x2 * s, dt), dt);
    dst[i + half] = enc_dt(rnd_dt(x1 * s, dt) + rnd_dt(x2 * c, dt), dt);
  }
}

/* Attention of one query head over cache rows 0..len-1 (T K/V [max_seq][D]). */
static void attend(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int len, int D, int dt,
                   uint16_t* out) {
  double* sc = (double*)malloc(sizeof(double) * (size_t)len);
  const float mul = rnd_dt((float)(1.0 / sqrt((double)D)), dt);
  double mx = -1e300;
  for (int j = 0; j < len; ++j) {
    double s = 0.0;
    for (int d = 0; d < D; ++d) s += (double)dec_dt(q[d], dt) * dec_dt(kc[(int64_t)j * D + d], dt);
    sc[j] = (double)rnd_dt(rnd_dt((float)s, dt) * mul, dt);
    if (sc[j] > mx) mx = sc[j];
  }
  double sum = 0.0;
  for (int j = 0; j < len; ++j) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
  for (int d = 0; d < D; ++d) {
    double acc = 0.0;
    for (int j = 0; j < len; ++j) acc += sc[j] * dec_dt(vc[(int64_t)j * D + d], dt);
    out[d] = enc_dt((float)(acc / sum), dt);
  }
  free(sc);
}

/* One linear y[T, N] = x[T, K] W^T in format fmt (see the section comment). */
static void lin_dt(const uint16_t* x, int dt, int fmt, const void* W, const void* S, int64_t T,
                   int64_t K, int64_t N, uint16_t* y) {
  double* xd = (double*)malloc(sizeof(double) * (size_t)(T * K));
  for (int64_t i = 0; i < T * K; ++i) xd[i] = dec_dt(x[i], dt);
  if (fmt == ORC_WFMT_W8A16 || fmt == ORC_WFMT_W8A16_F16S) {
    const int8_t* q = (const int8_t*)W;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      const float s = fmt == ORC_WFMT_W8A16 ? ((const float*)S)[n] : h2f(((const uint16_t*)S)[n]);
      const int8_t* row = q + n * K;
      for (int64_t t = 0; t < T; ++t) {
        double acc = 0.0;
        const double* xr = xd + t * K;
        for (int64_t k = 0; k < K; ++k) acc += (double)row[k] * xr[k];
        y[t * N + n] = enc_dt((float)acc * s, dt);
      }
    }
  } else if (T > 1) { /* the dequantised copy: T(d q) weights, dense product */
    const int64_t bb = orc_gguf_block_bytes(fmt), nb = K / QK;
#pragma omp parallel
    {
      double* wr = (double*)malloc(sizeof(double) * (size_t)K);
#pragma omp for schedule(static)
      for (int64_t n = 0; n < N; ++n) {
        for (int64_t b = 0; b < nb; ++b) {
          const uint8_t* blk = (const uint8_t*)W + (n * nb + b) * bb;
          const float d = block_d(blk);
          for (int j = 0; j < QK; ++j) wr[b * QK + j] = rnd_dt(d * (float)block_q(blk, fmt, j), dt);
        }
        for (int64_t t = 0; t < T; ++t) {
          double acc = 0.0;
          const double* xr = xd + t * K;
          for (int64_t k = 0; k < K; ++k) acc += wr[k] * xr[k];
          y[t * N + n] = enc_dt((float)acc, dt);
        }
      }
      free(wr);
    }
  } else { /* QMatMul: activations to Q8_0, integer block dots, f32 block scaling */
    float* yf = (float*)malloc(sizeof(float) * (size_t)(T * N));
    float* xf = (float*)malloc(sizeof(float) * (size_t)(T * K));
    for (int64_t i = 0; i < T * K; ++i) xf[i] = (float)xd[i];
    orc_gguf_linear_candle(xf, ORC_F32, (const uint8_t*)W, fmt, T, K, N, yf);
    for (int64_t i = 0; i < T * N; ++i) y[i] = enc_dt(yf[i], dt);
    free(xf);
    free(yf);
  }
  free(xd);
}

typedef struct orc_decoder {
  int32_t n_layers, hidden, inter, n_heads, n_kv, head_dim, vocab, qk_norm;
  float eps, theta;
  int32_t act_dtype;     /* ORC_F16 or ORC_BF16 */
  int32_t weight_format; /* layer linears: 0 W8A16 (f32 scale), 1 W8A16 (f16 scale), 2 Q4_0, 8 Q8_0 */
  int32_t head_format;   /* output head, same codes */
} orc_decoder;

/* Per-layer pointer table (12 entries): qkv_w, qkv_s, o_w, o_s, gu_w, gu_s,
 * down_w, down_s (W8A16: int8 [N, K] and scales [N]; GGUF: native blocks
 * [N, K/32] and NULL), input_norm, post_norm, q_norm, k_norm (T bits; the QK
 * norms may be NULL without qk_norm). */
enum { L_QKV_Q, L_QKV_S, L_O_Q, L_O_S, L_GU_Q, L_GU_S, L_DN_Q, L_DN_S, L_IN, L_POST, L_QN, L_KN, L_N };

static int fmt_ok(int f) {
  return f == ORC_WFMT_W8A16 || f == ORC_WFMT_W8A16_F16S || f == ORC_Q4_0 || f == ORC_Q8_0;
}

/* Greedy generation for one sequence: prefill `prompt`, then n_new tokens.
 * out_tokens[n_new]; margins[n_new] = top1 - top2 of each step's T logits;
 * logits_out (optional) [n_new, vocab]: each step's T logits as f32.
 * forced (optional) [n_new]: the token fed back after each step instead of the
 * argmax (teacher forcing; out_tokens still receive the argmax).
 * embed: [vocab, hidden] T bits. */
ORC_API int orc_decoder_run(const orc_decoder* c, const void* const* layer_ptrs,
                            const uint16_t* embed, const uint16_t* final_norm, const void* head_w,
                            const void* head_s, const int32_t* prompt, int n_prompt, int n_new,
                            const int32_t* forced, int32_t* out_tokens, float* margins,
                            float* logits_out, uint16_t* hidden_out) {
  const int dt = c->act_dtype;
  if ((dt != ORC_F16 && dt != ORC_BF16) || !fmt_ok(c->weight_format) || !fmt_ok(c->head_format) ||
      c->head_dim > 256 || c->n_kv <= 0 || c->n_heads % c->n_kv || n_prompt <= 0)
    return -1;
  const int64_t H = c->hidden, I = c->inter, D = c->head_dim, Hq = c->n_heads, Hkv = c->n_kv;
  const int64_t QKV = (Hq + 2 * Hkv) * D, QD = Hq * D, V = c->vocab;
  const int64_t max_seq = n_prompt + n_new + 1;
  const int rep = (int)(Hq / Hkv), wf = c->weight_format;
  uint16_t* kc = (uint16_t*)calloc((size_t)(c->n_layers * Hkv * max_seq * D), 2);
  uint16_t* vc = (uint16_t*)calloc((size_t)(c->n_layers * Hkv * max_seq * D), 2);
  uint16_t* cos_t = (uint16_t*)malloc((size_t)(max_seq * D / 2) * 2);
  uint16_t* sin_t = (uint16_t*)malloc((size_t)(max_seq * D / 2) * 2);
  rope_tables_dt(cos_t, sin_t, max_seq, (int)D, c->theta, dt);
  const int64_t Tmax = n_prompt;
  uint16_t* h = (uint16_t*)malloc((size_t)(Tmax * H) * 2);
  uint16_t* x1 = (uint16_t*)malloc((size_t)(Tmax * H) * 2);
  uint16_t* qkv = (uint16_t*)malloc((size_t)(Tmax * QKV) * 2);
  uint16_t* qr = (uint16_t*)malloc((size_t)(Tmax * QD) * 2);
  uint16_t* att = (uint16_t*)malloc((size_t)(Tmax * QD) * 2);
  uint16_t* dl = (uint16_t*)malloc((size_t)(Tmax * H) * 2);
  uint16_t* gu = (uint16_t*)malloc((size_t)(Tmax * 2 * I) * 2);
  uint16_t* mid = (uint16_t*)malloc((size_t)(Tmax * I) * 2);
  uint16_t* logits = (uint16_t*)malloc((size_t)V * 2);
  int32_t* toks = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n_prompt + n_new));
  memcpy(toks, prompt, sizeof(int32_t) * (size_t)n_prompt);
  int64_t p0 = 0, T = n_prompt;
  for (int step = 0; step < n_new; ++step) {
    for (int64_t t = 0; t < T; ++t) memcpy(h + t * H, embed + (int64_t)toks[p0 + t] * H, (size_t)H * 2);
    for (int l = 0; l < c->n_layers; ++l) {
      const void* const* P = layer_ptrs + (int64_t)l * L_N;
      rmsnorm_dt(h, NULL, NULL, (const uint16_t*)P[L_IN], x1, T, H, c->eps, dt);
      lin_dt(x1, dt, wf, P[L_QKV_Q], P[L_QKV_S], T, H, QKV, qkv);
      uint16_t* kl = kc + (int64_t)l * Hkv * max_seq * D;
      uint16_t* vl = vc + (int64_t)l * Hkv * max_seq * D;
      for (int64_t t = 0; t < T; ++t) {
        const int pos = (int)(p0 + t);
        for (int64_t hh = 0; hh < Hq; ++hh)
          head_norm_rope(qkv + t * QKV + hh * D, (const uint16_t*)P[L_QN], c->qk_norm, c->eps,
                         cos_t, sin_t, pos, (int)D, dt, qr + t * QD + hh * D);
        for (int64_t g = 0; g < Hkv; ++g) {
          head_norm_rope(qkv + t * QKV + (Hq + g) * D, (const uint16_t*)P[L_KN], c->qk_norm, c->eps,
                         cos_t, sin_t, pos, (int)D, dt, kl + (g * max_seq + pos) * D);
          memcpy(vl + (g * max_seq + pos) * D, qkv + t * QKV + (Hq + Hkv + g) * D, (size_t)D * 2);
        }
      }
#pragma omp parallel for collapse(2) schedule(static)
      for (int64_t t = 0; t < T; ++t)
        for (int64_t hh = 0; hh < Hq; ++hh) {
          const int64_t g = hh / rep;
          attend(qr + t * QD + hh * D, kl + g * max_seq * D, vl + g * max_seq * D,
                 (int)(p0 + t + 1), (int)D, dt, att + t * QD + hh * D);
        }
      lin_dt(att, dt, wf, P[L_O_Q], P[L_O_S], T, QD, H, dl);
      rmsnorm_dt(dl, h, h, (const uint16_t*)P[L_POST], x1, T, H, c->eps, dt);
      lin_dt(x1, dt, wf, P[L_GU_Q], P[L_GU_S], T, H, 2 * I, gu);
      for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < I; ++i) {
          const float g = dec_dt(gu[t * 2 * I + i], dt), u = dec_dt(gu[t * 2 * I + I + i], dt);
          const float s = rnd_dt(g / (1.0f + expf(-g)), dt);
          mid[t * I + i] = enc_dt(s * u, dt);
        }
      lin_dt(mid, dt, wf, P[L_DN_Q], P[L_DN_S], T, I, H, dl);
      for (int64_t i = 0; i < T * H; ++i) h[i] = enc_dt(dec_dt(h[i], dt) + dec_dt(dl[i], dt), dt);
    }
    /* head on the last position */
    if (hidden_out) memcpy(hidden_out + (int64_t)step * H, h + (T - 1) * H, (size_t)H * 2);
    rmsnorm_dt(h + (T - 1) * H, NULL, NULL, final_norm, x1, 1, H, c->eps, dt);
    lin_dt(x1, dt, c->head_format, head_w, head_s, 1, H, V, logits);
    float best = -INFINITY, second = -INFINITY;
    int32_t bi = 0;
    for (int64_t v = 0; v < V; ++v) {
      const float lv = dec_dt(logits[v], dt);
      if (lv > best) { second = best; best = lv; bi = (int32_t)v; }
      else if (lv > second) second = lv;
    }
    out_tokens[step] = bi;
    if (margins) margins[step] = best - second;
    if (logits_out)
      for (int64_t v = 0; v < V; ++v) logits_out[(int64_t)step * V + v] = dec_dt(logits[v], dt);
    toks[p0 + T] = forced ? forced[step] : bi;
    p0 += T;
    T = 1;
  }
  free(kc); free(vc); free(cos_t); free(sin_t); free(h); free(x1); free(qkv); free(qr);
  free(att); free(dl); free(gu); free(mid); free(logits); free(toks);
  return 0;
}

ORC_API int orc_decoder_generate(const orc_decoder* c, const void* const* layer_ptrs,
                                 const uint16_t* embed, const uint16_t* final_norm,
                                 const void* head_w, const void* head_s, const int32_t* prompt,
                                 int n_prompt, int n_new, int32_t* out_tokens, float* margins) {
  return orc_decoder_run(c, layer_ptrs, embed, final_norm, head_w, head_s, prompt, n_prompt, n_new,
                         NULL, out_tokens, margins, NULL, NULL);
}
