// Host check of the kernels' f32 exponential (tensorrs_b200/csrc/exp_f32.h):
// the same source, compiled by g++ with strict IEEE arithmetic, evaluated on
// f32 inputs and compared with glibc's expf(y) and powf(2.7182817f, y), the
// functions the reference calls.  Prints one line per (function, range):
//   name lo hi count identical max_ulp
// Arguments: the bit stride of the whole-range sweep (1 = every f32).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "exp_f32.h"

using namespace trs::expf32;

static int64_t ulp_distance(float a, float b) {
  int32_t ia, ib;
  std::memcpy(&ia, &a, 4);
  std::memcpy(&ib, &b, 4);
  if (ia < 0) ia = INT32_MIN - ia;
  if (ib < 0) ib = INT32_MIN - ib;
  const int64_t d = (int64_t)ia - ib;
  return d < 0 ? -d : d;
}

// Every stride-th f32 whose bits lie between those of lo and hi.
static void sweep(const char* name, bool pow_e, float lo, float hi, uint32_t stride) {
  const Base b = pow_e ? kBaseEf32 : kBaseE;
  uint32_t a = bits(lo), z = bits(hi);
  if (a > z) { const uint32_t t = a; a = z; z = t; }
  int64_t count = 0, same = 0, worst = 0, not_fast = 0;
#pragma omp parallel for reduction(+ : count, same, not_fast) reduction(max : worst) schedule(static)
  for (int64_t u = a; u <= (int64_t)z; u += stride) {
    const float y = from_bits((uint32_t)u);
    float s;
    int ex;
    if (!parts<false>(y, b, &s, &ex)) { ++not_fast; continue; }
    if (y <= 0.0f) {  // the NONPOS variant must agree
      float s2;
      int ex2;
      if (!parts<true>(y, b, &s2, &ex2) || s2 != s || ex2 != ex) ++not_fast;
    }
    const float got = scale(s, ex);
    const float want = pow_e ? powf(2.7182817f, y) : expf(y);
    const int64_t d = ulp_distance(got, want);
    ++count;
    if (d == 0) ++same;
    if (d > worst) worst = d;
  }
  std::printf("%s %.9g %.9g %lld %lld %lld %lld\n", name, (double)lo, (double)hi, (long long)count,
              (long long)same, (long long)worst, (long long)not_fast);
}

// exp_nonpos over every stride-th f32 from -0 down to -inf (bits 0x80000000
// .. 0xFF800000), NaN included: at most one ulp from glibc (0 below the
// subnormals, NaN for NaN), and equal to the fast path wherever that applies.
static void sweep_nonpos(const char* name, bool pow_e, uint32_t stride) {
  const Base b = pow_e ? kBaseEf32 : kBaseE;
  int64_t count = 0, same = 0, worst = 0, mismatch = 0;
  const int64_t n_stride = (0xFF800000ll - 0x80000000ll) / stride + 1;
#pragma omp parallel for reduction(+ : count, same, mismatch) reduction(max : worst) schedule(static)
  for (int64_t i = 0; i < n_stride + 3; ++i) {
    // the strided sweep, then -inf and two NaNs
    const int64_t u = i < n_stride ? 0x80000000ll + i * stride : 0xFF800000ll + (i - n_stride);
    const float y = from_bits((uint32_t)u);
    const float got = exp_nonpos(y, b);
    const float want = pow_e ? powf(2.7182817f, y) : expf(y);
    if (want != want || got != got) {
      if ((want != want) != (got != got)) ++mismatch;
      continue;
    }
    float s;
    int ex;
    if (parts<true>(y, b, &s, &ex) && scale(s, ex) != got) ++mismatch;
    const int64_t d = ulp_distance(got, want);
    ++count;
    if (d == 0) ++same;
    if (d > worst) worst = d;
  }
  std::printf("%s-nonpos -inf 0 %lld %lld %lld %lld\n", name, (long long)count, (long long)same, (long long)worst,
              (long long)mismatch);
}

// sigmoid_div against the IEEE quotient, for every f32 e in [0, 1] (d = 1 + e),
// both numerators (1 and e) and the seeds RN(1/d) and its two neighbours
// (every f32 within one ulp of 1/d): prints the count and the mismatches.
static void check_sigmoid_div() {
  int64_t count = 0, bad = 0;
#pragma omp parallel for reduction(+ : count, bad) schedule(static)
  for (int64_t u = 0; u <= (int64_t)bits(1.0f); ++u) {
    const float e = from_bits((uint32_t)u);
    const float d = 1.0f + e;
    const float rn = 1.0f / d;
    const float seeds[3] = {std::nextafter(rn, 0.0f), rn, std::nextafter(rn, 2.0f)};
    for (int n = 0; n < 2; ++n) {
      const float num = n ? e : 1.0f;
      const float want = num / d;
      for (float y0 : seeds) {
        ++count;
        if (bits(sigmoid_div(num, d, y0)) != bits(want)) ++bad;
      }
    }
  }
  std::printf("sigmoid_div 0 1 %lld %lld 0 %lld\n", (long long)count, (long long)(count - bad), (long long)bad);
}

// The whole sigmoid (exp_nonpos, then sigmoid_div with the seed RN(1/d))
// against the reference's two branches on glibc's expf, every stride-th f32.
static void sweep_sigmoid(uint32_t stride) {
  int64_t count = 0, same = 0, worst = 0, mismatch = 0;
  const int64_t n = (int64_t)(0xFFFFFFFFull / stride) + 1;
#pragma omp parallel for reduction(+ : count, same, mismatch) reduction(max : worst) schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float x = from_bits((uint32_t)(i * stride));
    const float e = exp_nonpos(-std::fabs(x), kBaseE);
    const float d = 1.0f + e;
    const float got = sigmoid_div(x >= 0.0f ? 1.0f : e, d, 1.0f / d);
    float want;
    if (x >= 0.0f) {
      want = 1.0f / (1.0f + expf(-x));
    } else {
      const float ee = expf(x);
      want = ee / (1.0f + ee);
    }
    if (want != want || got != got) {
      if ((want != want) != (got != got)) ++mismatch;
      continue;
    }
    const int64_t dist = ulp_distance(got, want);
    ++count;
    if (dist == 0) ++same;
    if (dist > worst) worst = dist;
  }
  std::printf("sigmoid -inf inf %lld %lld %lld %lld\n", (long long)count, (long long)same, (long long)worst,
              (long long)mismatch);
}

int main(int argc, char** argv) {
  const uint32_t stride = argc > 1 ? (uint32_t)std::strtoul(argv[1], nullptr, 10) : 1;
  for (int f = 0; f < 2; ++f) {
    const char* name = f ? "powE" : "expf";
    sweep(name, f, -86.0f, -0.0f, stride);
    sweep(name, f, 0.0f, 87.0f, stride);
    sweep(name, f, -20.0f, -1.0f, stride > 16 ? stride / 16 : 1);
    sweep(name, f, -1.0f, -0.01f, stride > 16 ? stride / 16 : 1);
    sweep(name, f, 1.0f, 20.0f, stride > 16 ? stride / 16 : 1);
    sweep_nonpos(name, f, stride);
  }
  check_sigmoid_div();
  sweep_sigmoid(stride);
  return 0;
}
