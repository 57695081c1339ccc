/* Plain-C restatement of the W8A8 integer path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/ load this library (through oracle/c_oracle.py), as a second, independent
 * statement of the arithmetic the torch oracle (oracle/w8a8_oracle.py) and the sm_100a
 * kernels implement; the product never links or calls it. Built by oracle/Makefile into
 * oracle/_build/libw8a8_ref.so.
 *
 * What it restates:
 *  - per-row weight quantisation, fp32 (fni8-serve tests/test_smoke.py:14-18,
 *    fni8serve/models/weights.py:18-25): s = max(absmax, 1e-6) / 127,
 *    q = clamp(round_half_even(w / s), -127, 127);
 *  - per-token activation quantisation (the call contract of
 *    fni8.linear, fni8serve/layers/linear.py:67-69): s = absmax / 127,
 *    q = clamp(round_half_even(x * (127 / absmax)), -127, 127), a zero row gives s = 0, q = 0;
 *  - the int8 x int8 -> int32 contraction, accumulated in int64 and range-checked;
 *  - the dequant epilogue y = (float(acc) * a_scale[m]) * w_scale[n] (+ bias[n])
 *    (+ residual[m, n]) in fp32, rounded once to fp16 or bf16 (round to nearest even);
 *  - per_group_i4 / int4 weights: the nibble unpack and two's-complement decode, the fp16
 *    fallback weight, and the W4A8 linear (exact int32 sum per scale group, groups added
 *    in order in fp32, then the token scale and bias);
 *  - the MoE block's index and combine steps (fni8serve/models/moe.py:97-105): stable
 *    grouping of (token, slot) pairs by expert, and the weighted sum over a token's slots
 *    in slot order in fp32, rounded once.
 *
 * Every floating-point step is one IEEE fp32 operation in the order written (the Makefile
 * builds with -ffp-contract=off, so nothing is fused); fp16/bf16 <-> fp32 conversions are
 * the exact IEEE ones, written out below from the formats' definitions.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { F16 = 0, BF16 = 1 };

static float bits_to_f32(uint32_t x) {
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint32_t f32_to_bits(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  return x;
}

/* binary16: 1 sign, 5 exponent (bias 15), 10 fraction bits; every value is exact in fp32 */
static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) { /* zero or subnormal: m * 2^-24 */
    const float v = (float)m * 5.9604644775390625e-8f;
    return bits_to_f32(f32_to_bits(v) | sign);
  }
  if (e == 31) return bits_to_f32(sign | 0x7f800000u | (m << 13));
  return bits_to_f32(sign | ((e - 15u + 127u) << 23) | (m << 13));
}

static uint16_t f32_to_f16(float f) {
  const uint32_t x = f32_to_bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return sign | 0x7e00u;   /* NaN */
  if (ax >= 0x477ff000u) return sign | 0x7c00u;  /* >= 65520 rounds to infinity */
  if (ax < 0x38800000u) {                         /* below 2^-14: subnormal or zero */
    /* a * 2^24 is exact (a power-of-two scaling of a value >= 2^-149); rintf rounds
       half to even in the default rounding mode; 1024 encodes 2^-14 itself */
    const float m = rintf(bits_to_f32(ax) * 16777216.0f);
    return sign | (uint16_t)m;
  }
  uint32_t h = (((ax >> 23) - 127u + 15u) << 10) | ((ax & 0x7fffffu) >> 13);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* a carry moves into the exponent */
  return sign | (uint16_t)h;
}

/* bfloat16: the upper half of an fp32 */
static float bf16_to_f32(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

static uint16_t f32_to_bf16(float f) {
  const uint32_t x = f32_to_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u); /* quiet NaN */
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

static float load(const uint16_t* p, int64_t i, int dtype) { return dtype == BF16 ? bf16_to_f32(p[i]) : f16_to_f32(p[i]); }

static uint16_t store(float v, int dtype) { return dtype == BF16 ? f32_to_bf16(v) : f32_to_f16(v); }

static int8_t code(float v) {
  float r = rintf(v);
  if (r > 127.0f) r = 127.0f;
  if (r < -127.0f) r = -127.0f;
  return (int8_t)r;
}

/* fp16/bf16 <-> fp32 elementwise (for checking the conversions themselves) */
void fni8o_to_f32(const uint16_t* x, int dtype, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = load(x, i, dtype);
}

void fni8o_from_f32(const float* x, int dtype, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = store(x[i], dtype);
}

/* w: fp32 [N, K] -> q int8 [N, K], s fp32 [N] */
void fni8o_quantize_weight_rows(const float* w, int64_t N, int64_t K, int8_t* q, float* s) {
  for (int64_t n = 0; n < N; ++n) {
    const float* row = w + n * K;
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(row[k]));
    const float sc = fmaxf(amax, 1e-6f) / 127.0f;
    for (int64_t k = 0; k < K; ++k) q[n * K + k] = code(row[k] / sc);
    s[n] = sc;
  }
}

/* x: fp16/bf16 [M, K] -> q int8 [M, K], s fp32 [M] */
void fni8o_quantize_rows(const uint16_t* x, int dtype, int64_t M, int64_t K, int8_t* q, float* s) {
  for (int64_t m = 0; m < M; ++m) {
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(load(x, m * K + k, dtype)));
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    for (int64_t k = 0; k < K; ++k) q[m * K + k] = code(load(x, m * K + k, dtype) * inv);
    s[m] = amax / 127.0f;
  }
}

/* acc[m, n] = sum_k a[m, k] * w[n, k]; returns 1 if a sum leaves the int32 range */
int fni8o_gemm_i32(const int8_t* a, const int8_t* w, int64_t M, int64_t N, int64_t K, int32_t* acc) {
  int overflow = 0;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      int64_t t = 0;
      for (int64_t k = 0; k < K; ++k) t += (int64_t)a[m * K + k] * (int64_t)w[n * K + k];
      if (t > INT32_MAX || t < INT32_MIN) overflow = 1;
      acc[m * N + n] = (int32_t)t;
    }
  return overflow;
}

/* y[m, n] = (float(acc) * a_scale[m]) * w_scale[n] (+ bias[n]) (+ residual[m, n]) -> dtype */
void fni8o_dequant(const int32_t* acc, const float* a_scale, const float* w_scale, const uint16_t* bias,
                   const uint16_t* residual, int dtype, int64_t M, int64_t N, uint16_t* out) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float y = (float)acc[m * N + n] * a_scale[m];
      y = y * w_scale[n];
      if (bias) y = y + load(bias, n, dtype);
      if (residual) y = y + load(residual, m * N + n, dtype);
      out[m * N + n] = store(y, dtype);
    }
}

/* fni8.linear restated: quantise rows, contract, dequant (acc_ws: int32 [M, N] scratch,
   q_ws: int8 [M, K], s_ws: fp32 [M]); returns 1 on int32 overflow */
int fni8o_linear_w8a8(const uint16_t* x, int dtype, int64_t M, int64_t K, const int8_t* wq, const float* ws,
                      int64_t N, const uint16_t* bias, int8_t* q_ws, float* s_ws, int32_t* acc_ws, uint16_t* out) {
  fni8o_quantize_rows(x, dtype, M, K, q_ws, s_ws);
  const int ovf = fni8o_gemm_i32(q_ws, wq, M, N, K, acc_ws);
  fni8o_dequant(acc_ws, s_ws, ws, bias, NULL, dtype, M, N, out);
  return ovf;
}

/* ---------------------------------------------------------------- W4A8 (per_group_i4, int4)
 * Packed bytes [N, K/2]: element 2j in the low nibble of byte j, element 2j+1 in the high
 * nibble, two's complement (fni8serve/convert.py:69-80, fni8serve/layers/linear.py:33-40). */
void fni8o_unpack_i4(const uint8_t* packed, int64_t N, int64_t K, int8_t* codes) {
  for (int64_t i = 0; i < N * (K / 2); ++i) {
    const int lo = packed[i] & 0xf, hi = packed[i] >> 4;
    codes[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
    codes[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
  }
}

/* LinearW8A8's fp16 fallback weight: code * scale[n, k / group] in fp32, rounded once
   (fni8serve/layers/linear.py:41-45) */
void fni8o_dequant_weight_i4(const uint8_t* packed, const float* scale, int64_t N, int64_t K, int64_t group,
                             int8_t* codes_ws, uint16_t* out) {
  fni8o_unpack_i4(packed, N, K, codes_ws);
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k)
      out[n * K + k] = f32_to_f16((float)codes_ws[n * K + k] * scale[n * (K / group) + k / group]);
}

/* fni8.linear for per_group_i4: per-token int8 rows; per group g an exact int32 sum acc_g;
   y = sum over g in order of float(acc_g) * scale[n, g] (each product and each sum rounded
   in fp32); out = y * a_scale[m] (+ bias[n]), rounded once to dtype */
void fni8o_linear_w4a8(const uint16_t* x, int dtype, int64_t M, int64_t K, const uint8_t* packed, const float* scale,
                       int64_t N, int64_t group, const uint16_t* bias, int8_t* q_ws, float* s_ws, int8_t* codes_ws,
                       uint16_t* out) {
  const int64_t G = K / group;
  fni8o_quantize_rows(x, dtype, M, K, q_ws, s_ws);
  fni8o_unpack_i4(packed, N, K, codes_ws);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float y = 0.0f;
      for (int64_t g = 0; g < G; ++g) {
        int32_t acc = 0; /* |acc| <= 127 * 8 * group: far inside int32 */
        for (int64_t k = g * group; k < (g + 1) * group; ++k) acc += (int32_t)q_ws[m * K + k] * codes_ws[n * K + k];
        const float term = (float)acc * scale[n * G + g];
        y = y + term;
      }
      y = y * s_ws[m];
      if (bias) y = y + load(bias, n, dtype);
      out[m * N + n] = store(y, dtype);
    }
}

/* ---------------------------------------------------------------- MoE (fni8serve/models/moe.py:97-105)
 * Stable grouping of the T*k (token, slot) pairs by expert: counts[E], offsets[E+1]
 * (exclusive prefix sums), slot_of_row[rows] (the slots of expert 0 in slot order, then
 * expert 1's, ...) and row_of_slot[T*k] (its inverse; -1 for an expert id outside [0, E),
 * which is not grouped). Returns the number of grouped rows. */
int64_t fni8o_moe_plan(const int32_t* topi, int64_t n, int32_t E, int32_t* counts, int32_t* offsets,
                       int32_t* row_of_slot, int32_t* slot_of_row, int32_t* cursor_ws) {
  for (int32_t e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t i = 0; i < n; ++i)
    if (topi[i] >= 0 && topi[i] < E) counts[topi[i]] += 1;
  offsets[0] = 0;
  for (int32_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  for (int32_t e = 0; e < E; ++e) cursor_ws[e] = offsets[e];
  for (int64_t i = 0; i < n; ++i) {
    const int32_t e = topi[i];
    if (e < 0 || e >= E) {
      row_of_slot[i] = -1;
      continue;
    }
    const int32_t row = cursor_ws[e]++;
    row_of_slot[i] = row;
    slot_of_row[row] = (int32_t)i;
  }
  return offsets[E];
}

/* out[t] = sum over j = 0..k-1 in order of topw[t, j] * y[row_of_slot[t*k + j]] in fp32
 * (each product and each sum rounded), skipping slots with no row, rounded once to dtype.
 * y: [rows, H] fp16/bf16; topw fp32 [T, k]. */
void fni8o_moe_combine(const uint16_t* y, int dtype, const int32_t* row_of_slot, const float* topw, int64_t T,
                       int64_t k, int64_t H, uint16_t* out) {
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      float acc = 0.0f;
      for (int64_t j = 0; j < k; ++j) {
        const int32_t r = row_of_slot[t * k + j];
        if (r < 0) continue;
        const float term = topw[t * k + j] * load(y, (int64_t)r * H + h, dtype);
        acc = acc + term;
      }
      out[t * H + h] = store(acc, dtype);
    }
}
