/*
 * CPU restatement of blockfp8's block quantizers -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity oracle for the CUDA quantizer.  Only tests/, the
 * smoke check in __graft_entry__.py and bench.py's CPU-baseline leg load it;
 * the blockfp8_b200 package never does.
 *
 * What it restates (reference = simon-jd/blockfp8):
 *   blockfp8/quant.py:25-28  _scale_from_amax: max(amax, eps) / 448 as a true
 *                            float32 division (not a multiply by 1/448)
 *   blockfp8/quant.py:31-36  _group_amax: amax of |x| over [rows x cols]
 *                            blocks, ragged edge blocks allowed
 *   blockfp8/quant.py:39-64  quantize_activations: 1 x 128 groups,
 *                            q = e4m3(clamp(x / scale, -448, 448))
 *   blockfp8/quant.py:67-79  quantize_weights: 128 x 128 blocks, same math
 * The float -> e4m3fn rounding is written here from the format definition
 * (1 sign bit, 4 exponent bits with bias 7, 3 mantissa bits, no infinities,
 * largest finite 448, subnormal step 2^-9), rounding to nearest, ties to
 * even, which is what torch's Tensor.to(torch.float8_e4m3fn) does.
 *
 * NaN: torch's amax propagates NaN, so a group holding a NaN gets a NaN
 * scale and NaN codes (0x7f with the input's sign); this file does the same.
 *
 * Build: cc -O3 -fopenmp -ffp-contract=off -shared -fPIC (see oracle/build.py).
 * -ffp-contract=off keeps every multiply and add separately rounded, as the
 * reference's torch operations are.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define FP8_MAX 448.0f

static inline uint32_t f32_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}

/* float -> float8_e4m3fn, round to nearest even; |v| > 448 saturates to
 * +-448 (the quantizer clamps first, so this never triggers there). */
uint8_t oracle_e4m3_from_float(float v) {
  const uint32_t u = f32_bits(v);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  float a = fabsf(v);
  if (isnan(v)) return (uint8_t)(sign | 0x7fu);
  if (a >= FP8_MAX) return (uint8_t)(sign | 0x7eu); /* 0x7e = 1.75 * 2^8 = 448 */
  if (a < 0.015625f) {
    /* Subnormal range (below 2^-6): multiples of 2^-9.  a * 512 is exact
     * (a power-of-two scaling of a float far from overflow) and rintf rounds
     * to nearest even under the default rounding mode.  k == 8 is 2^-6, the
     * smallest normal, whose code 0x08 is the same integer. */
    const int k = (int)rintf(a * 512.0f);
    return (uint8_t)(sign | (uint8_t)k);
  }
  /* Normal range: keep 3 of float's 23 mantissa bits, rounding the other 20
   * to nearest even; a carry out of the mantissa bumps the exponent, which
   * the encoding absorbs because exponent and mantissa are adjacent. */
  const uint32_t ua = f32_bits(a);
  const int exp = (int)((ua >> 23) & 0xffu) - 127; /* -6 .. 8 */
  uint32_t man = ua & 0x7fffffu;
  uint32_t keep = man >> 20;
  const uint32_t rest = man & 0xfffffu;
  const uint32_t half = 0x80000u;
  if (rest > half || (rest == half && (keep & 1u))) keep += 1u;
  uint32_t code = ((uint32_t)(exp + 7) << 3) + keep;
  if (code > 0x7eu) code = 0x7eu; /* 464 and up would round past 448 */
  return (uint8_t)(sign | code);
}

float oracle_e4m3_to_float(uint8_t c) {
  const int sign = c & 0x80;
  const int e = (c >> 3) & 0xf;
  const int m = c & 7;
  float v;
  if (e == 0xf && m == 7) return sign ? -NAN : NAN;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else
    v = ldexpf((float)(8 + m), e - 10);
  return sign ? -v : v;
}

/* NaN-propagating max, as torch.amax: a NaN anywhere wins. */
static inline float amax_step(float acc, float v) {
  const float a = fabsf(v);
  if (isnan(acc) || isnan(a)) return NAN;
  return a > acc ? a : acc;
}

/* Block quantizer shared by both entry points: x [R, C] float32 (row stride
 * ldx) in blocks of br x 128; q [R, C] codes (row stride ldq); the scale of
 * block (i, j) goes to s[i * s_i + j * s_j].  Follows quant.py:25-36, 61. */
static void quantize_blocks(const float* x, int64_t R, int64_t C, int64_t ldx, int64_t br,
                            float eps, uint8_t* q, int64_t ldq, float* s, int64_t s_i,
                            int64_t s_j) {
  const int64_t rb = (R + br - 1) / br, cb = (C + 127) / 128;
  const float feps = (float)eps;
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t i = 0; i < rb; ++i) {
    for (int64_t j = 0; j < cb; ++j) {
      const int64_t r0 = i * br, r1 = r0 + br < R ? r0 + br : R;
      const int64_t c0 = j * 128, c1 = c0 + 128 < C ? c0 + 128 : C;
      float amax = 0.0f; /* the reference pads with zeros, which leave amax alone */
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t c = c0; c < c1; ++c) amax = amax_step(amax, x[r * ldx + c]);
      if (!isnan(amax) && amax < feps) amax = feps; /* clamp_min(eps) */
      const float scale = amax / FP8_MAX;           /* true division */
      s[i * s_i + j * s_j] = scale;
      for (int64_t r = r0; r < r1; ++r) {
        for (int64_t c = c0; c < c1; ++c) {
          float v = x[r * ldx + c] / scale;
          if (!isnan(v)) v = v < -FP8_MAX ? -FP8_MAX : (v > FP8_MAX ? FP8_MAX : v);
          q[r * ldq + c] = oracle_e4m3_from_float(v);
        }
      }
    }
  }
}

/* quantize_activations (quant.py:39-64): 1 x 128 groups.  The caller picks
 * the scale layout through (s_m, s_k): (1, M) is the reference's default
 * M-major layout, (kb, 1) the row-major one. */
void oracle_quantize_activations(const float* x, int64_t M, int64_t K, int64_t ldx, float eps,
                                 uint8_t* q, int64_t ldq, float* s, int64_t s_m, int64_t s_k) {
  quantize_blocks(x, M, K, ldx, 1, eps, q, ldq, s, s_m, s_k);
}

/* quantize_weights (quant.py:67-79): 128 x 128 blocks, scales [nb, kb]
 * row-major. */
void oracle_quantize_weights(const float* w, int64_t N, int64_t K, int64_t ldw, float eps,
                             uint8_t* q, int64_t ldq, float* s) {
  const int64_t kb = (K + 127) / 128;
  quantize_blocks(w, N, K, ldw, 128, eps, q, ldq, s, kb, 1);
}

/* Decode a whole array of codes (used to build float64 operands). */
void oracle_e4m3_decode(const uint8_t* c, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_float(c[i]);
}

/* Decode straight to float64 (the GEMM's operand type); parallel, so the
 * first touch of a large output array is spread over all threads. */
void oracle_e4m3_decode_f64(const uint8_t* c, int64_t n, double* out) {
  double table[256];
  for (int i = 0; i < 256; ++i) table[i] = (double)oracle_e4m3_to_float((uint8_t)i);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = table[c[i]];
}

int oracle_abi_version(void) { return 1; }
