// exp_f32.h -- the f32 exponential of the hot paths, in f32 arithmetic.
//
// 2^(y * log2(b)) for an f32 y and the two bases the reference uses: e
// (expf: sigmoid) and the f32 constant E = 2.7182817f (powf(E, y): ELU,
// SELU, SoftMax).  The method is P. T. P. Tang's table-driven exponential
// ("Table-driven implementation of the exponential function in IEEE
// floating-point arithmetic", ACM TOMS 15(2), 1989) with 16 table entries:
//
//   k   = round(16 * y * log2(b))          by adding 1.5 * 2^23 (k in the low bits)
//   z   = 16 * y * log2(b) - k             two fused multiply-adds with
//                                          16 * log2(b) split as mh + ml;
//                                          |z| <= 1/2, absolute error <= 2^-25
//   p   = 2^(z/16) - 1                     degree-4 Taylor polynomial in z
//                                          (truncation error < 2^-34)
//   s   = T[j] + (T[j] * p + t[j])         j = k mod 16, 2^(j/16) = T[j] + t[j];
//                                          the one rounding that matters is
//                                          this last addition
//   result = s * 2^(k div 16)              added to the exponent field
//
// The fast path covers y in [-86, 87], where the result is a normal f32;
// other y (and NaN) return false, and the caller takes the f64 evaluation
// (exp2_scaled) instead.  Against glibc's expf and powf(2.7182817f, y),
// every f32 y in that range was compared on the host: at most one ulp apart,
// 99.92 % identical overall and 99.1-99.3 % for |y| in [0.01, 20]
// (tests/test_exp_cpu.py re-checks a sample).
//
// The same source compiles for the host (g++, strict IEEE: -ffp-contract=off)
// so the host test evaluates exactly the operations the kernels do.
#pragma once

#include <cstdint>
#include <cstring>

#include "exp_table.h"

#if defined(__CUDACC__)
#define TRS_EXP_HD __host__ __device__ __forceinline__
#else
#include <cmath>
#define TRS_EXP_HD inline
#endif

namespace trs {

namespace expf32 {

TRS_EXP_HD float fma_rn(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return std::fmaf(a, b, c);
#endif
}
TRS_EXP_HD float add_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
TRS_EXP_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
TRS_EXP_HD uint32_t bits(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
#endif
}
TRS_EXP_HD float from_bits(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float x;
  std::memcpy(&x, &u, 4);
  return x;
#endif
}

// Base e and base E = 2.7182817f: 16 * log2(b) as an f32 pair.
struct Base {
  float mh, ml;
};
constexpr Base kBaseE = {kExp16LogEHi, kExp16LogELo};
constexpr Base kBaseEf32 = {kExp16LogEf32Hi, kExp16LogEf32Lo};

// The fast path: *s in [0.69, 1.45] and *ex with b^y ~= *s * 2^*ex.  Returns
// false when y is outside the fast range (or NaN); *s and *ex are then
// meaningless, but the table index stays in bounds for every y.  NONPOS: the
// caller guarantees y <= 0 or NaN, so only the lower bound is checked.
template <bool NONPOS>
TRS_EXP_HD bool parts(float y, Base b, float* s, int* ex) {
  const bool fast = NONPOS ? (y >= -86.0f) : (y >= -86.0f && y <= 87.0f);
  const float kShift = 12582912.0f;  // 1.5 * 2^23
  const float t = fma_rn(y, b.mh, kShift);
  const int k = (int)(bits(t) - bits(kShift));
  const float kf = add_rn(t, -kShift);
  const float z = fma_rn(y, b.ml, fma_rn(y, b.mh, -kf));
  float u = fma_rn(z, kExpC4, kExpC3);
  u = fma_rn(z, u, kExpC2);
  u = fma_rn(z, u, kExpC1);
  const float p = mul_rn(z, u);
  const int j = k & 15;
#if defined(__CUDA_ARCH__)
  const float2 tj = __ldg(reinterpret_cast<const float2*>(&kExp2Tab16[0][0]) + j);
  const float th = tj.x, tl = tj.y;
#else
  const float th = kExp2Tab16[j][0], tl = kExp2Tab16[j][1];
#endif
  *s = add_rn(th, fma_rn(th, p, tl));
  *ex = k >> 4;  // arithmetic shift: floor(k / 16)
  return fast;
}

// s * 2^ex for the fast path's parts (a normal f32).
TRS_EXP_HD float scale(float s, int ex) { return from_bits(bits(s) + ((uint32_t)ex << 23)); }

// b^y for y <= 0 or NaN, branch-free (sigmoid's exp(-|x|), softmax's
// E^(x - max)): y is clamped to -104 (below it every result rounds to 0; a
// NaN passes the compare and propagates through s), the parts are those of
// `parts` above, and the scaling is s * 2^(ex + 64) (exact: a normal f32)
// times 2^-64, which rounds once.  Normal results are therefore identical to
// the fast path's; subnormal ones (y < -87.3) carry the rounding of s as
// well, at most one ulp from the correctly rounded value.  The exponent field
// of 2^(ex + 64) comes from the bits of t: with t = 1.5 * 2^23 + k,
// (bits(t) << 19) masked to the exponent field is (k div 16) << 23, because
// the bits of 1.5 * 2^23 shift out.
TRS_EXP_HD float exp_nonpos(float y, Base b) {
  y = y < -104.0f ? -104.0f : y;
  const float kShift = 12582912.0f;  // 1.5 * 2^23
  const float t = fma_rn(y, b.mh, kShift);
  const uint32_t tb = bits(t);
  const float kf = add_rn(t, -kShift);
  const float z = fma_rn(y, b.ml, fma_rn(y, b.mh, -kf));
  float u = fma_rn(z, kExpC4, kExpC3);
  u = fma_rn(z, u, kExpC2);
  u = fma_rn(z, u, kExpC1);
  const float p = mul_rn(z, u);
  const uint32_t j = tb & 15u;
#if defined(__CUDA_ARCH__)
  const float2 tj = __ldg(reinterpret_cast<const float2*>(&kExp2Tab16[0][0]) + j);
  const float th = tj.x, tl = tj.y;
#else
  const float th = kExp2Tab16[j][0], tl = kExp2Tab16[j][1];
#endif
  const float s = add_rn(th, fma_rn(th, p, tl));
  const float p2 = from_bits(((tb << 19) & 0xFF800000u) + (191u << 23));  // 2^(ex + 64)
  return mul_rn(mul_rn(s, p2), 0x1p-64f);
}

// num / (1 + e) for the two quotients of the reference's sigmoid
// (autodiff/ops.rs:586-593): num = 1 (x >= 0) or num = e (x < 0), where
// e = exp(-|x|) in [0, 1], so the denominator d = RN(1 + e) lies in [1, 2].
// P. Markstein's division ("Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): a reciprocal
// seed y0 within one ulp of 1/d, one Newton step y1 = y0 + y0 (1 - d y0),
// q0 = num y1, the exact remainder r = num - q0 d, and q = q0 + r y1 rounded
// once.  The Newton step can land on 1/2 for d = 2 - 2^-23 (an exact tie at
// the binade boundary), where the correction then rounds the wrong way;
// 1/d >= 1/2 + 2^-24 for every d < 2, so y1 is floored there (for d = 2 the
// floored y1 still corrects to 1/2).  With that floor the result equals the
// IEEE quotient num / d for every f32 e in [0, 1] and both numerators, for
// each seed within one ulp of 1/d: tests/test_exp_cpu.py checks all of them.
// NaN in e propagates through num.
TRS_EXP_HD float sigmoid_div(float num, float d, float y0) {
  // the floor as a maximum: a NaN y1 (only for a NaN d, where num is NaN as
  // well) becomes the floor, and num carries the NaN on
  const float y1 = fmaxf(fma_rn(y0, fma_rn(-d, y0, 1.0f), y0), 0x1.000002p-1f);
  const float q0 = mul_rn(num, y1);
  return fma_rn(fma_rn(-q0, d, num), y1, q0);
}

#if defined(__CUDACC__)
// The reference's sigmoid, x >= 0 ? 1 / (1 + e) : e / (1 + e) with
// e = exp(-|x|): both branches take the same e, and the seed of the division
// is the hardware's approximate reciprocal (at most one ulp from 1/d).
__device__ __forceinline__ float sigmoid(float x) {
  const float e = exp_nonpos(-fabsf(x), kBaseE);
  const float d = add_rn(1.0f, e);
  float y0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d));
  return sigmoid_div(x >= 0.0f ? 1.0f : e, d, y0);
}

// exp_nonpos2: `exp_nonpos` of two values at once; sigmoid2: `sigmoid` of two
// values at once -- both on sm_100's packed f32x2 add / multiply /
// fused multiply-add (each lane rounded to nearest exactly as the scalar
// instruction rounds, subnormals kept), so each pair costs one issue slot
// where `sigmoid` above takes two.  Unlike the scalar __fmul_rn / __fadd_rn,
// a packed multiply whose result feeds a packed add may be fused into one
// multiply-add by the compiler; the only such pair here is e = (s * 2^(ex+64))
// * 2^-64 feeding d = 1 + e, where the scaling is exact (or e < 2^-126, and
// 1 + e rounds to 1 either way), so a fused form gives the same d.  The operations are those of `sigmoid` and
// `exp_nonpos`, step for step, with every negated operand folded into an
// exact product by -1 or a sign-symmetric rounding:
//   shift - t        = fma(t, -1, shift)  (exact: both integers in [2^23, 2^24))
//   -RN(1 + e)       = fma(e, -1, -1)
//   RN(1 - d y0)     = fma(-d, y0, 1)
//   RN(num - q0 d)   = fma(q0, -d, num)
// so each lane's result is bit-identical to `sigmoid` of that lane.  The
// clamp at -104 is max.NaN (a NaN passes through, as the scalar compare
// lets it); the table loads, the exponent scaling, the reciprocal seed, the
// reciprocal floor and the numerator choice stay per lane.
__device__ __forceinline__ float2 exp_nonpos2(float2 y, Base b) {
  asm("max.NaN.f32 %0, %1, 0fC2D00000;" : "=f"(y.x) : "f"(y.x));  // max(y, -104)
  asm("max.NaN.f32 %0, %1, 0fC2D00000;" : "=f"(y.y) : "f"(y.y));
  const float2 mh = make_float2(b.mh, b.mh), ml = make_float2(b.ml, b.ml);
  const float2 shift = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const float2 m1 = make_float2(-1.0f, -1.0f);
  const float2 t = __ffma2_rn(y, mh, shift);
  const uint32_t tbx = __float_as_uint(t.x), tby = __float_as_uint(t.y);
  const float2 nkf = __ffma2_rn(t, m1, shift);  // -(t - shift)
  const float2 z = __ffma2_rn(y, ml, __ffma2_rn(y, mh, nkf));
  float2 u = __ffma2_rn(z, make_float2(kExpC4, kExpC4), make_float2(kExpC3, kExpC3));
  u = __ffma2_rn(z, u, make_float2(kExpC2, kExpC2));
  u = __ffma2_rn(z, u, make_float2(kExpC1, kExpC1));
  const float2 p = __fmul2_rn(z, u);
  const float2* tab = reinterpret_cast<const float2*>(&kExp2Tab16[0][0]);
  const float2 tjx = __ldg(tab + (tbx & 15u)), tjy = __ldg(tab + (tby & 15u));
  const float2 th = make_float2(tjx.x, tjy.x), tl = make_float2(tjx.y, tjy.y);
  const float2 s = __fadd2_rn(th, __ffma2_rn(th, p, tl));
  // 2^(ex + 64): bits 4..12 of t are ex (two's complement), so
  // ((t >> 4) << 23) + (191 << 23) modulo 2^32 is its f32 bit pattern
  const float2 p2 = make_float2(__uint_as_float((tbx >> 4) * (1u << 23) + (191u << 23)),
                                __uint_as_float((tby >> 4) * (1u << 23) + (191u << 23)));
  return __fmul2_rn(__fmul2_rn(s, p2), make_float2(0x1p-64f, 0x1p-64f));
}

__device__ __forceinline__ float2 sigmoid2(float2 x) {
  const float2 m1 = make_float2(-1.0f, -1.0f), one = make_float2(1.0f, 1.0f);
  const float2 e = exp_nonpos2(make_float2(-fabsf(x.x), -fabsf(x.y)), kBaseE);
  const float2 d = __fadd2_rn(one, e);
  const float2 nd = __ffma2_rn(e, m1, m1);  // -d
  float2 y0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0.y) : "f"(d.y));
  float2 y1 = __ffma2_rn(y0, __ffma2_rn(nd, y0, one), y0);
  y1.x = fmaxf(y1.x, 0x1.000002p-1f);
  y1.y = fmaxf(y1.y, 0x1.000002p-1f);
  const float2 num = make_float2(x.x >= 0.0f ? 1.0f : e.x, x.y >= 0.0f ? 1.0f : e.y);
  const float2 q0 = __fmul2_rn(num, y1);
  return __ffma2_rn(__ffma2_rn(q0, nd, num), y1, q0);
}
#endif

}  // namespace expf32
}  // namespace trs
