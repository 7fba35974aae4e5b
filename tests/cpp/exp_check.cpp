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
  return 0;
}
