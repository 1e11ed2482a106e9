// The activation quantizer's arithmetic for one 1 x 128 group, shared by the
// quantization kernel and the kernels that quantize their own activations.
// The result is defined by the reference's sequence (blockfp8/quant.py:25-64,
// csrc/quant_sm89.cu:38-59), and bit-exactness with it is the contract:
//   amax  = max(eps, max |x|) over the group (NaN dropped, as fmaxf does),
//   scale = amax / 448  (IEEE division),
//   code  = e4m3(clamp(x / scale, -448, 448)), round to nearest even,
//           saturating.
// A half-warp holds one group, 8 bf16 values per lane.
//
// Two ways to the same codes:
// - group_codes_exact: the sequence above, one IEEE division per value;
// - group_codes_fast: x / scale as x * r corrected once (Markstein, "Computation
//   of elementary functions on the IBM RISC System/6000 processor", IBM J.
//   Res. Dev. 34(1), 1990): r = RN(1 / scale), q = RN(x r),
//   e = x - q scale (exact, one fma), q' = RN(q + e r); then the saturating
//   conversion, which equals clamp-then-convert for finite quotients, and
//   x's sign ORed into each code (it only changes x = -0, whose quotient
//   the sequence returns as +0).  Three packed f32x2 operations per pair of
//   values instead of two divisions.  The scale itself is amax / 448 by the
//   same correction with the constant y = RN(1 / 448): q = RN(amax y),
//   e = amax - 448 q, scale = RN(q + e y) -- three operations instead of a
//   division (amax below 2^-100 divides).  The input domain is small -- x is bf16 and amax is eps or a
//   bf16 magnitude -- and tests/test_quant_fast_gpu.py compares the fast
//   codes with the division on every (x, amax) pair of it and the fast
//   scale with the division on every finite non-negative float, so both are
//   exact by exhaustion, not by argument.  Groups holding a NaN or an
//   infinity take the exact path (their quotients are not finite).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace bfp8 {

// 8 bf16 values (one 16-byte load) as floats.
__device__ __forceinline__ void bf16x8_to_float(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}

// The group's scale, from the floats: every lane of the half-warp passes its
// 8 values; all 32 lanes of the warp must call it (the shuffles stay inside
// each half-warp).
__device__ __forceinline__ float group_scale(const float (&f)[8], float eps) {
  float amax = eps;
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  return amax / 448.f;
}

// The largest bf16 magnitude bit pattern of the group (|x| as a 16-bit
// integer; the order of non-negative floats is the order of their bits), on
// every lane of the half-warp; 0x7F80 or more means an infinity or NaN is in
// the group.  All 32 lanes must call it (one warp reduction per half-warp).
__device__ __forceinline__ uint32_t group_max_bits(const uint4& v) {
  const uint32_t m2 = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                               __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return __reduce_max_sync(0xFFFFu << (threadIdx.x & 16u), max(m2 & 0xFFFFu, m2 >> 16));
}

// amax / 448, correctly rounded, for finite amax >= 0 (see the file comment).
// Below 2^-100 the correction step can underflow (the quotient nears the
// subnormal range), so there the division itself runs; eps keeps amax far
// above that in practice.
__device__ __forceinline__ float scale_of(float amax) {
  constexpr float kInv448 = 1.f / 448.f;  // RN(1 / 448)
  if (amax < 0x1p-100f) return amax / 448.f;
  const float q = __fmul_rn(amax, kInv448);
  const float e = __fmaf_rn(-q, 448.f, amax);
  return __fmaf_rn(e, kInv448, q);
}

// The 8 e4m3 codes of a lane's values by the reference's sequence, packed
// little-endian into two words.
__device__ __forceinline__ uint2 group_codes_exact(const float (&f)[8], float scale) {
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 u = make_float2(fminf(fmaxf(f[2 * e] / scale, -448.f), 448.f),
                                 fminf(fmaxf(f[2 * e + 1] / scale, -448.f), 448.f));
    const uint32_t pair = __nv_cvt_float2_to_fp8x2(u, __NV_SATFINITE, __NV_E4M3);
    packed[e >> 1] |= pair << (16 * (e & 1));
  }
  return make_uint2(packed[0], packed[1]);
}

// Packed fp32 pairs: {a0, a1} * {b0, b1} + {c0, c1}, each rounded to nearest.
__device__ __forceinline__ float2 fma_x2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 ra, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// The same codes for a group with finite values (see the file comment),
// given scale and r = RN(1 / scale).
__device__ __forceinline__ uint2 group_codes_fast(const uint4& v, float scale, float r) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const float2 rr = make_float2(r, r), nss = make_float2(-scale, -scale), nz = make_float2(-0.f, -0.f);
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = make_float2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xFFFF0000u));
    const float2 q = fma_x2(x, rr, nz);     // RN(x r)  (adding -0 leaves every product as it is)
    const float2 err = fma_x2(q, nss, x);   // x - q scale, exact
    const float2 qq = fma_x2(err, rr, q);   // RN(q + err r)
    const uint32_t pair = __nv_cvt_float2_to_fp8x2(qq, __NV_SATFINITE, __NV_E4M3);
    packed[e >> 1] |= pair << (16 * (e & 1));
  }
  // x / scale has x's sign and so has its code; the sequence only loses it
  // for x = -0 (+0 plus -0 is +0).  The high byte of each bf16 carries its
  // sign in bit 7, the bit of the e4m3 sign.
  packed[0] |= __byte_perm(v.x, v.y, 0x7531) & 0x80808080u;
  packed[1] |= __byte_perm(v.z, v.w, 0x7531) & 0x80808080u;
  return make_uint2(packed[0], packed[1]);
}

// One group: the scale (same value on every lane of the half-warp) and this
// lane's 8 codes.  All 32 lanes must call it.
struct GroupQuant {
  float scale;
  uint2 codes;
};

__device__ __forceinline__ GroupQuant quantize_group(const uint4& v, float eps) {
  GroupQuant g;
  const uint32_t mbits = group_max_bits(v);
  if (mbits < 0x7F80u) {  // finite group (uniform across the half-warp)
    const float amax = fmaxf(eps, __uint_as_float(mbits << 16));
    g.scale = scale_of(amax);
    g.codes = group_codes_fast(v, g.scale, __frcp_rn(g.scale));
  } else {  // an infinity or NaN: the reference's sequence as it stands
    float f[8];
    bf16x8_to_float(v, f);
    float amax = eps;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    // the other lanes of the half-warp took the same branch (mbits is the
    // half-warp's), so the shuffles name just those 16 lanes
    const uint32_t half_mask = 0xFFFFu << (threadIdx.x & 16u);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(half_mask, amax, o));
    g.scale = amax / 448.f;
    g.codes = group_codes_exact(f, g.scale);
  }
  return g;
}

}  // namespace bfp8
