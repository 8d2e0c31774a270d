/*
 * kvoff_oracle.c - CPU restatement of the reference's KV offload hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker that the CUDA library is
 * compared against (tests, __graft_entry__.smoke, and bench.py's CPU
 * baseline / reference arm). The product never links or calls it.
 *
 * Reference behaviour restated (paths inside the reference project):
 *   fp8_quantize    nanovllm/engine/cpu_prefix_cache.py:20-24
 *   fp8_dequantize  nanovllm/engine/cpu_prefix_cache.py:27-28
 *   block views     cpu_prefix_cache.py:94-100 (slot layout [2, L, BS, H, D],
 *                   scales [2, L, BS, H, 1] in the cache dtype, bf16)
 *   save / restore  cpu_prefix_cache.py:305, 323-326 and 373, 394-397
 *   store_kvcache   nanovllm/layers/attention.py:10-40
 *
 * Rounding is restated from the IEEE definitions with frexp / ldexp /
 * nearbyint (ties-to-even in the default rounding mode) instead of bit
 * tricks, so it shares no code path with the device codec. NaN encodings
 * follow what torch's CPU path produced for the reference quantizer when
 * the golden fixtures were generated (tests/golden/make_golden.py): a NaN
 * row scale is 0xFFFF; x / s keeps x's NaN when x is NaN, else s's NaN;
 * Inf / Inf is the default NaN with the sign set; an e4m3 NaN is 0x7F with the
 * input's sign bit. Dequantized NaN values are 0x7FFF (see dequantize_row).
 *
 * Build: oracle/build.py (gcc -O3 -mavx2 -fopenmp -fno-fast-math -ffp-contract=off).
 */
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API __attribute__((visibility("default")))

static float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}

static float bf16_value(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

/* Round a finite float to a grid of quantum 2^q_exp, ties to even. */
static float round_to_quantum(float f, int q_exp) {
  const double scaled = ldexp((double)f, -q_exp); /* exact: power-of-two scaling */
  return (float)ldexp(nearbyint(scaled), q_exp);  /* exact unless it overflows to Inf */
}

/* fp32 -> bf16 bits, round to nearest even; NaN -> 0xFFFF. */
static uint16_t bf16_from_f32(float f) {
  if (isnan(f)) return 0xFFFF;
  if (isinf(f) || f == 0.0f) return (uint16_t)(f32_to_bits(f) >> 16);
  int e;
  frexp(f, &e); /* |f| = m * 2^e, 0.5 <= m < 1: top bit weight 2^(e-1) */
  int q = e - 8;          /* 8 significant bits */
  if (q < -133) q = -133; /* bf16 subnormal quantum 2^-133 */
  /* A carry past the bf16 maximum gives exactly 2^128, which becomes Inf. */
  const float rf = (float)ldexp(nearbyint(ldexp((double)f, -q)), q);
  return (uint16_t)(f32_to_bits(rf) >> 16); /* rf has at most 8 significant bits */
}

/* fp32 -> float8_e4m3fn (bias 7, 3 mantissa bits, max 448, no Inf), RNE. */
static uint8_t e4m3_from_f32(float f) {
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  if (isnan(f)) return (uint8_t)(0x7F | sign);
  const float a = fabsf(f);
  if (a > 464.0f) return (uint8_t)(0x7F | sign); /* rounds past 448: NaN (non-saturating) */
  int e;
  frexp(a, &e);
  int q = e - 4; /* 4 significant bits */
  if (q < -9) q = -9; /* subnormal quantum 2^-9 */
  const float r = a == 0.0f ? 0.0f : round_to_quantum(a, q);
  if (r == 0.0f) return sign;
  int re;
  const double m = frexp(r, &re); /* r = m * 2^re, m in [0.5, 1) */
  const int exp2 = re - 1;        /* r = 1.xxx * 2^exp2 */
  if (exp2 < -6) {                /* subnormal: r = k * 2^-9, k in 1..7 */
    return (uint8_t)(sign | (uint8_t)ldexp(r, 9));
  }
  const int mant = (int)ldexp(m * 2.0 - 1.0, 3); /* 0..7 */
  return (uint8_t)(sign | ((exp2 + 7) << 3) | mant);
}

static float e4m3_value(uint8_t v) {
  const int sign = v & 0x80;
  const int exp = (v >> 3) & 0xF;
  const int mant = v & 7;
  float r;
  if (exp == 0xF && mant == 7)
    r = NAN;
  else if (exp == 0)
    r = (float)ldexp((double)mant, -9);
  else
    r = (float)ldexp(1.0 + mant / 8.0, exp - 7);
  return sign ? -r : r;
}

/* One row: scale = bf16(max(amax / 448, 1e-30)); payload = e4m3(clamp(x / s)). */
static void quantize_row(const uint16_t* x, int64_t d, uint8_t* out, uint16_t* scale) {
  int any_nan = 0;
  float amax = 0.0f;
  for (int64_t j = 0; j < d; ++j) {
    const float v = bf16_value(x[j]);
    if (isnan(v))
      any_nan = 1;
    else if (fabsf(v) > amax)
      amax = fabsf(v);
  }
  float s32 = any_nan ? NAN : amax / 448.0f;
  if (s32 < 1e-30f) s32 = 1e-30f; /* NaN compares false and stays NaN */
  const uint16_t sb = bf16_from_f32(s32);
  const float s = bf16_value(sb);
  *scale = sb;
  for (int64_t j = 0; j < d; ++j) {
    const float v = bf16_value(x[j]);
    if (isnan(s)) {
      out[j] = isnan(v) ? (uint8_t)(0x7F | (signbit(v) ? 0x80 : 0)) : 0xFF;
    } else if (isinf(s)) {
      out[j] = isinf(v) ? 0xFF : (signbit(v) ? 0x80 : 0x00);
    } else {
      float q = v / s;
      if (q < -448.0f) q = -448.0f;
      if (q > 448.0f) q = 448.0f;
      out[j] = e4m3_from_f32(q);
    }
  }
}

/* Dequantized NaN results are written as 0x7FFF, the canonical NaN of the
 * GPU's fp32 -> bf16 conversion (the reference's own encoding here depends on
 * torch's code path: 0x7FC0 from its scalar CPU loop, 0xFFFF from its vector
 * loop). */
static void dequantize_row(const uint8_t* p, uint16_t scale, int64_t d, uint16_t* out) {
  const float s = bf16_value(scale);
  for (int64_t j = 0; j < d; ++j) {
    const float v = e4m3_value(p[j]) * s;
    out[j] = isnan(v) ? 0x7FFF : bf16_from_f32(v);
  }
}

ORACLE_API void kvo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

ORACLE_API int kvo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

ORACLE_API uint16_t kvo_bf16_from_f32(float f) { return bf16_from_f32(f); }
ORACLE_API uint8_t kvo_e4m3_from_f32(float f) { return e4m3_from_f32(f); }
ORACLE_API float kvo_e4m3_value(uint8_t v) { return e4m3_value(v); }

/* rows of d elements (row stride `stride` elements) -> dense payload/scale. */
ORACLE_API void kvo_fp8_quantize_rows(const uint16_t* x, int64_t rows, int64_t d, int64_t stride,
                                      uint8_t* payload, uint16_t* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) quantize_row(x + r * stride, d, payload + r * d, scale + r);
}

ORACLE_API void kvo_fp8_dequantize_rows(const uint8_t* payload, const uint16_t* scale,
                                        int64_t rows, int64_t d, uint16_t* out, int64_t stride) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) dequantize_row(payload + r * d, scale[r], d, out + r * stride);
}

/*
 * Blocks of a pool (geometry as in include/kvoff.h, strides in elements) to
 * dense slots: slot i occupies payload + i * num_chunks * rows_per_chunk * d
 * and scale + i * num_chunks * rows_per_chunk.
 */
ORACLE_API void kvo_fp8_save_blocks(const uint16_t* pool, int64_t num_chunks, int64_t chunk_stride,
                                    int64_t block_stride, int64_t rows_per_chunk, int64_t d,
                                    const int64_t* ids, int64_t count, uint8_t* payload,
                                    uint16_t* scale) {
  const int64_t rows = num_chunks * rows_per_chunk;
  const int64_t total = count * rows;
#pragma omp parallel for schedule(static)
  for (int64_t q = 0; q < total; ++q) {
    const int64_t i = q / rows, sr = q % rows;
    const int64_t c = sr / rows_per_chunk, r = sr % rows_per_chunk;
    quantize_row(pool + c * chunk_stride + ids[i] * block_stride + r * d, d,
                 payload + (i * rows + sr) * d, scale + i * rows + sr);
  }
}

ORACLE_API void kvo_fp8_restore_blocks(uint16_t* pool, int64_t num_chunks, int64_t chunk_stride,
                                       int64_t block_stride, int64_t rows_per_chunk, int64_t d,
                                       const int64_t* ids, int64_t count, const uint8_t* payload,
                                       const uint16_t* scale) {
  const int64_t rows = num_chunks * rows_per_chunk;
  const int64_t total = count * rows;
#pragma omp parallel for schedule(static)
  for (int64_t q = 0; q < total; ++q) {
    const int64_t i = q / rows, sr = q % rows;
    const int64_t c = sr / rows_per_chunk, r = sr % rows_per_chunk;
    dequantize_row(payload + (i * rows + sr) * d, scale[i * rows + sr], d,
                   pool + c * chunk_stride + ids[i] * block_stride + r * d);
  }
}

/* Byte moves of whole blocks (strides in bytes); direction 0 = pool -> slots. */
ORACLE_API void kvo_copy_blocks(uint8_t* pool, int64_t num_chunks, int64_t chunk_stride,
                                int64_t block_stride, int64_t chunk_bytes, const int64_t* ids,
                                int64_t count, uint8_t* slots, int direction) {
#pragma omp parallel for schedule(static)
  for (int64_t q = 0; q < count * num_chunks; ++q) {
    const int64_t i = q / num_chunks, c = q % num_chunks;
    uint8_t* p = pool + c * chunk_stride + ids[i] * block_stride;
    uint8_t* s = slots + (i * num_chunks + c) * chunk_bytes;
    if (direction == 0)
      memcpy(s, p, (size_t)chunk_bytes);
    else
      memcpy(p, s, (size_t)chunk_bytes);
  }
}

/* k_cache.view(-1, row)[slot_mapping[i]] = key row i (and V) for slot != -1. */
ORACLE_API void kvo_store_kvcache(const uint8_t* key, int64_t key_stride, const uint8_t* value,
                                  int64_t value_stride, uint8_t* k_cache, uint8_t* v_cache,
                                  int64_t row_bytes, const int32_t* slot_mapping, int64_t n,
                                  int64_t num_slots) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slot_mapping[i];
    if (slot < 0 || slot >= num_slots) continue;
    memcpy(k_cache + slot * row_bytes, key + i * key_stride, (size_t)row_bytes);
    memcpy(v_cache + slot * row_bytes, value + i * value_stride, (size_t)row_bytes);
  }
}

/*
 * Exhaustive check of the device quantizer's division-free quotient
 * (csrc/codec.cuh quant_input): for every bf16 scale s a row can produce and
 * every finite bf16 x with |x| <= the largest amax that yields s, compare
 *     e4m3(clamp(x / s))                                   (IEEE division)
 *     e4m3(clamp(fma(-fma(q1, s, -x), r, q1)))            (r = 1/s, q1 = x*r)
 * Returns the number of pairs whose e4m3 bytes differ; *pairs gets the count
 * of pairs checked. Uses only IEEE fp32 operations, which the GPU performs
 * identically (__frcp_rn, __fmul_rn, __fmaf_rn; denormals preserved).
 */
ORACLE_API int64_t kvo_fast_quotient_mismatches(int64_t* pairs) {
  static uint16_t max_amax[65536];
  static unsigned char seen[65536];
  memset(max_amax, 0, sizeof max_amax);
  memset(seen, 0, sizeof seen);
  for (uint32_t ab = 0; ab < 0x7F80; ++ab) {
    float s32 = bf16_value((uint16_t)ab) / 448.0f;
    if (s32 < 1e-30f) s32 = 1e-30f;
    const uint16_t sb = bf16_from_f32(s32);
    seen[sb] = 1;
    if (ab > max_amax[sb]) max_amax[sb] = (uint16_t)ab;
  }
  int64_t bad = 0, checked = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : bad, checked)
  for (int32_t sb = 0; sb < 0x7F80; ++sb) {
    if (!seen[sb]) continue;
    const float s = bf16_value((uint16_t)sb), r = 1.0f / s;
    const float amax = bf16_value(max_amax[sb]);
    for (uint32_t xb = 0; xb < 65536; ++xb) {
      if ((xb & 0x7F80) == 0x7F80) continue;
      const float x = bf16_value((uint16_t)xb);
      if (fabsf(x) > amax) continue;
      ++checked;
      float q = x / s;
      q = q < -448.0f ? -448.0f : (q > 448.0f ? 448.0f : q);
      const float q1 = x * r;
      float f = fmaf(-fmaf(q1, s, -x), r, q1);
      f = f < -448.0f ? -448.0f : (f > 448.0f ? 448.0f : f);
      if (f32_to_bits(q) != f32_to_bits(f) && e4m3_from_f32(q) != e4m3_from_f32(f)) ++bad;
    }
  }
  if (pairs != NULL) *pairs = checked;
  return bad;
}

/*
 * Exhaustive check of the device quantizer's scale (csrc/codec.cuh
 * scale_from_amax): for every finite non-negative bf16 amax, compare
 * bf16(max(amax * RN(1/448), 1e-30)) with the reference's
 * bf16(max(amax / 448, 1e-30)). Returns the number of differing scales.
 */
ORACLE_API int32_t kvo_scale_multiply_mismatches(void) {
  const float inv = 1.0f / 448.0f;
  int32_t bad = 0;
  for (uint32_t ab = 0; ab < 0x7F80; ++ab) {
    const float a = bf16_value((uint16_t)ab);
    float div = a / 448.0f, mul = a * inv;
    if (div < 1e-30f) div = 1e-30f;
    if (mul < 1e-30f) mul = 1e-30f;
    if (bf16_from_f32(div) != bf16_from_f32(mul)) ++bad;
  }
  return bad;
}

/*
 * Fast single-pass port of the same path, for the timed CPU baseline (the
 * bench's reference arm). The reference runs these steps as separate torch
 * ops with fp32 temporaries; this port fuses them per row and rounds with
 * integer bit operations, so it is a faster (conservative) CPU baseline. Its
 * results equal the checker above bit for bit (tests/test_oracle_port.py);
 * rows holding Inf or NaN go through the checker's row routine.
 */
static float g_e4m3_table[256];
static int g_e4m3_table_ready = 0;

static void init_e4m3_table(void) {
  if (g_e4m3_table_ready) return;
  for (int v = 0; v < 256; ++v) g_e4m3_table[v] = e4m3_value((uint8_t)v);
  g_e4m3_table_ready = 1;
}

static inline uint32_t rne16_bits(float f) { /* finite f: bf16 bits, RNE */
  const uint32_t u = f32_to_bits(f);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

/* e4m3 byte of a finite q with |q| <= 448, round to nearest even. */
static inline uint8_t e4m3_bits_clamped(float q) {
  const uint32_t u = f32_to_bits(q);
  const uint32_t a = u & 0x7FFFFFFFu;
  uint32_t mag;
  if (a < 0x3C800000u) /* below 2^-6: grid of 2^-9 (subnormals) */
    mag = (uint32_t)rintf(bits_to_f32(a) * 512.0f);
  else /* keep 3 mantissa bits, rebias the exponent from 127 to 7 */
    mag = ((a + 0x7FFFFu + ((a >> 20) & 1u)) >> 20) - (120u << 3);
  return (uint8_t)(((u >> 24) & 0x80u) | mag);
}

static void quantize_row_fast(const uint16_t* x, int64_t d, uint8_t* out, uint16_t* scale) {
  uint32_t m = 0;
  for (int64_t j = 0; j < d; ++j) {
    const uint32_t a = x[j] & 0x7FFFu;
    m = a > m ? a : m;
  }
  if (m >= 0x7F80u) { /* an Inf or NaN in the row */
    quantize_row(x, d, out, scale);
    return;
  }
  float s32 = bf16_value((uint16_t)m) / 448.0f;
  if (s32 < 1e-30f) s32 = 1e-30f;
  const uint16_t sb = (uint16_t)rne16_bits(s32);
  const float s = bf16_value(sb);
  *scale = sb;
  for (int64_t j = 0; j < d; ++j) {
    float q = bf16_value(x[j]) / s;
    q = q < -448.0f ? -448.0f : (q > 448.0f ? 448.0f : q);
    out[j] = e4m3_bits_clamped(q);
  }
}

static void dequantize_row_fast(const uint8_t* p, uint16_t scale, int64_t d, uint16_t* out) {
  const float s = bf16_value(scale);
  for (int64_t j = 0; j < d; ++j) {
    const float v = g_e4m3_table[p[j]] * s;
    const uint32_t u = f32_to_bits(v);
    out[j] = (u & 0x7FFFFFFFu) > 0x7F800000u ? 0x7FFF : (uint16_t)rne16_bits(v);
  }
}

ORACLE_API void kvo_fp8_save_blocks_fast(const uint16_t* pool, int64_t num_chunks,
                                         int64_t chunk_stride, int64_t block_stride,
                                         int64_t rows_per_chunk, int64_t d, const int64_t* ids,
                                         int64_t count, uint8_t* payload, uint16_t* scale) {
  const int64_t rows = num_chunks * rows_per_chunk;
  const int64_t total = count * rows;
#pragma omp parallel for schedule(static)
  for (int64_t q = 0; q < total; ++q) {
    const int64_t i = q / rows, sr = q % rows;
    const int64_t c = sr / rows_per_chunk, r = sr % rows_per_chunk;
    quantize_row_fast(pool + c * chunk_stride + ids[i] * block_stride + r * d, d,
                      payload + (i * rows + sr) * d, scale + i * rows + sr);
  }
}

ORACLE_API void kvo_fp8_restore_blocks_fast(uint16_t* pool, int64_t num_chunks,
                                            int64_t chunk_stride, int64_t block_stride,
                                            int64_t rows_per_chunk, int64_t d, const int64_t* ids,
                                            int64_t count, const uint8_t* payload,
                                            const uint16_t* scale) {
  init_e4m3_table();
  const int64_t rows = num_chunks * rows_per_chunk;
  const int64_t total = count * rows;
#pragma omp parallel for schedule(static)
  for (int64_t q = 0; q < total; ++q) {
    const int64_t i = q / rows, sr = q % rows;
    const int64_t c = sr / rows_per_chunk, r = sr % rows_per_chunk;
    dequantize_row_fast(payload + (i * rows + sr) * d, scale[i * rows + sr], d,
                        pool + c * chunk_stride + ids[i] * block_stride + r * d);
  }
}
