// device_ops.cuh -- element arithmetic with the reference's rounding.
//
// Every f32/f64 operation goes through an explicitly rounded intrinsic
// (__fadd_rn, __fmul_rn, __fdiv_rn, ... ), which the compiler never fuses
// into an FMA, so each step rounds exactly once as the reference's separate
// Rust operations do.  The library is also built with -fmad=false.
//
// Transcendentals: the reference calls glibc (expf, tanhf, powf, logf and the
// f64 forms).  The exponentials of the f32 hot paths (expf in sigmoid,
// powf(E, x) in softmax) are the f32 table-driven exponential of exp_f32.h,
// at most one ulp from glibc; its rare inputs outside the normal result range
// take exp2_scaled below (f64, rounded once).  ELU and SELU, which subtract 1
// from E^x, take exp2_scaled for every input (the correctly rounded E^x).  tanh, ln and the
// general powf evaluate CUDA's f64 functions and round once to f32, within one
// ulp of the correctly rounded result.  For f64 the kernels call CUDA's f64
// functions.
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda_runtime.h>

#include "../../include/trs.h"
#include "exp_f32.h"

namespace trs {

// 2^(y * k2) for an f32 argument y, evaluated in f64 and returned unrounded
// (the caller rounds it once to f32); k2 is log2 of a base near e (log2(e)
// for expf, log2(2.7182817f) for powf(E, .)).
//
// Method: Cody and Waite's additive argument reduction followed by a minimax
// polynomial (J.-M. Muller, "Elementary Functions: Algorithms and
// Implementation", ch. 6 and 11).  k = round(y*k2) by adding 1.5*2^52, which
// leaves k in the low word; f = y*k2 - k in [-1/2, 1/2] by one fused
// multiply-add; 2^f by the degree-8 polynomial of least maximum relative
// error on [-1/2, 1/2] (Remez exchange; error 7.8e-13); 2^k added to the
// exponent field.  The result is within 1e-12 relative of 2^(y*k2): rounded
// to f32 it is the correctly rounded value except within 1e-12 of a rounding
// boundary, where it is one ulp away.  y is clamped to [-110, 90] first
// (beyond it the f32 result is already 0 or +inf, and 2^k stays a normal
// exponent); a NaN passes the clamps (the compares are false), keeps k = 0
// and yields NaN.  NONPOS: the caller guarantees y <= 0 or NaN (softmax's
// x - max), so the upper clamp is skipped.
template <bool NONPOS = false>
__device__ __forceinline__ double exp2_scaled(float y, double k2) {
  y = y < -110.0f ? -110.0f : y;
  if constexpr (!NONPOS) y = y > 90.0f ? 90.0f : y;
  const double yd = (double)y;
  const double kShift = 6755399441055744.0;  // 1.5 * 2^52
  const double sh = __fma_rn(yd, k2, kShift);
  const int k = y == y ? __double2loint(sh) : 0;
  const double f = __fma_rn(yd, k2, -__dsub_rn(sh, kShift));
  double q = 1.3175867143282797e-06;
  q = __fma_rn(q, f, 1.5309737219754944e-05);
  q = __fma_rn(q, f, 0.0001540385170493416);
  q = __fma_rn(q, f, 0.00133334520632859);
  q = __fma_rn(q, f, 0.009618128542934786);
  q = __fma_rn(q, f, 0.05550410939340186);
  q = __fma_rn(q, f, 0.2402265069887989);
  q = __fma_rn(q, f, 0.6931471805465147);
  q = __fma_rn(q, f, 0.9999999999997624);
  // q in [0.70, 1.42] and |k| <= 159: the scaled value is a normal f64
  return __hiloint2double(__double2hiint(q) + (int)((unsigned)k << 20), __double2loint(q));
}

constexpr double kLog2E = 1.4426950408889634;  // log2(e) rounded to f64

// b^y in f32 for the bases of exp_f32.h: the table-driven fast path, or the
// f64 evaluation (k2 = log2(b) in f64) for y outside it (results that are
// subnormal, zero or infinite, and NaN).
template <bool NONPOS = false>
__device__ __forceinline__ float exp_tab(float y, expf32::Base b, double k2) {
  float s;
  int ex;
  if (expf32::parts<NONPOS>(y, b, &s, &ex)) return expf32::scale(s, ex);
  return (float)exp2_scaled<NONPOS>(y, k2);
}

template <class T> struct Arith;

template <> struct Arith<float> {
  using Acc = double;  // accumulator type of sums
  static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
  static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
  static __device__ __forceinline__ float div(float a, float b, int*) { return __fdiv_rn(a, b); }
  static __device__ __forceinline__ float neg(float a) { return -a; }
  static __device__ __forceinline__ float abs(float a) { return fabsf(a); }
  static __device__ __noinline__ float pow(float a, float b) {
    return (float)::pow((double)a, (double)b);
  }
  // powf(E_f32, x); `log2_e` is log2 of the f32 E in f64 (for the inputs
  // outside the table path).
  static __device__ __forceinline__ float pow_e_inline(float x, double log2_e) {
    return exp_tab(x, expf32::kBaseEf32, log2_e);
  }
  static __device__ __forceinline__ float pow_e(float x, double log2_e) { return pow_e_inline(x, log2_e); }
  // E^x rounded once from the f64 evaluation: ELU and SELU subtract 1 from
  // it, which turns a one-ulp difference near x = 0 into many ulps of the
  // result, so there the value has to be the correctly rounded one (as
  // glibc's powf gives it, to within its hard cases)
  static __device__ __forceinline__ float pow_e_rounded_once(float x, double log2_e) {
    return (float)exp2_scaled<false>(x, log2_e);
  }
  static __device__ __forceinline__ float exp(float a) { return exp_tab(a, expf32::kBaseE, kLog2E); }
  // expf and powf(E, .) for a <= 0 or NaN (sigmoid's exp(-|x|), softmax's
  // E^(x - max)): the branch-free form
  static __device__ __forceinline__ float exp_nonpos(float a) { return expf32::exp_nonpos(a, expf32::kBaseE); }
  static __device__ __forceinline__ float pow_e_nonpos(float a, double) {
    return expf32::exp_nonpos(a, expf32::kBaseEf32);
  }
  // tanh: for |x| >= 1 through expm1 in f32 steps, 1 - 2/(expm1(2|x|) + 2),
  // the classical formulation (the one glibc's f32 tanh evaluates), with
  // expm1 rounded once from f64; below 1 the f64 tanh rounded once, because
  // there the formulation's -t/(t+2) amplifies a one-ulp difference in t.
  static __device__ __noinline__ float tanh(float a) {
    const float ax = fabsf(a);
    if (!(ax >= 1.0f)) return (float)::tanh((double)a);  // |x| < 1, and NaN
    float z;
    if (ax >= 22.0f) {
      z = 1.0f;
    } else {
      const float t = (float)::expm1((double)__fmul_rn(2.0f, ax));
      z = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(t, 2.0f)));
    }
    return a < 0.0f ? -z : z;
  }
  static __device__ __noinline__ float ln(float a) { return (float)::log((double)a); }
  static __device__ __forceinline__ float from(const trs_scalar& s) { return (float)s.f; }
  static __device__ __forceinline__ double to_acc(float a) { return (double)a; }
  static __device__ __forceinline__ float from_acc(double a) { return (float)a; }
};

template <> struct Arith<double> {
  using Acc = double;
  static __device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
  static __device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
  static __device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
  static __device__ __forceinline__ double div(double a, double b, int*) { return __ddiv_rn(a, b); }
  static __device__ __forceinline__ double neg(double a) { return -a; }
  static __device__ __forceinline__ double abs(double a) { return fabs(a); }
  static __device__ __noinline__ double pow(double a, double b) { return ::pow(a, b); }
  // powf(E_f64, x): f64 has no wider type to hide the rounding of x*ln(E),
  // so this calls pow with the f64 E itself.
  static __device__ __forceinline__ double pow_e_inline(double x, double e) { return ::pow(e, x); }
  static __device__ __noinline__ double pow_e(double x, double e) { return pow_e_inline(x, e); }
  static __device__ __noinline__ double exp(double a) { return ::exp(a); }
  static __device__ __forceinline__ double exp_nonpos(double a) { return exp(a); }
  static __device__ __forceinline__ double pow_e_nonpos(double x, double e) { return pow_e(x, e); }
  static __device__ __forceinline__ double pow_e_rounded_once(double x, double e) { return pow_e(x, e); }
  static __device__ __noinline__ double tanh(double a) { return ::tanh(a); }
  static __device__ __noinline__ double ln(double a) { return ::log(a); }
  static __device__ __forceinline__ double from(const trs_scalar& s) { return s.f; }
  static __device__ __forceinline__ double to_acc(double a) { return a; }
  static __device__ __forceinline__ double from_acc(double a) { return a; }
};

// Integers: add/sub/mul wrap (the reference's release build); division by
// zero and MIN / -1 set a flag the host turns into TRS_ERR_DIV_ZERO (the
// reference panics on both) and produce 0.
template <class I, class U>
struct IntArith {
  using Acc = U;  // sums wrap; unsigned keeps the wrap well defined
  static __device__ __forceinline__ I add(I a, I b) { return (I)((U)a + (U)b); }
  static __device__ __forceinline__ I sub(I a, I b) { return (I)((U)a - (U)b); }
  static __device__ __forceinline__ I mul(I a, I b) { return (I)((U)a * (U)b); }
  static __device__ __forceinline__ I div(I a, I b, int* flag) {
    if (b == 0) { if (flag) atomicOr(flag, 1); return 0; }
    if (b == (I)-1 && a == (I)((U)1 << (sizeof(I) * 8 - 1))) { if (flag) atomicOr(flag, 2); return 0; }
    return a / b;
  }
  static __device__ __forceinline__ I neg(I a) { return (I)((U)0 - (U)a); }
  static __device__ __forceinline__ I abs(I a) { return a < 0 ? neg(a) : a; }
  static __device__ __forceinline__ I pow(I, I) { return 0; }
  static __device__ __forceinline__ I pow_e(I, double) { return 0; }
  static __device__ __forceinline__ I pow_e_rounded_once(I, double) { return 0; }
  static __device__ __forceinline__ I pow_e_inline(I, double) { return 0; }
  static __device__ __forceinline__ I exp(I) { return 0; }
  static __device__ __forceinline__ I exp_nonpos(I) { return 0; }
  static __device__ __forceinline__ I pow_e_nonpos(I, double) { return 0; }
  static __device__ __forceinline__ I tanh(I) { return 0; }
  static __device__ __forceinline__ I ln(I) { return 0; }
  static __device__ __forceinline__ I from(const trs_scalar& s) { return (I)s.i; }
  static __device__ __forceinline__ U to_acc(I a) { return (U)a; }
  static __device__ __forceinline__ I from_acc(U a) { return (I)a; }
};
template <> struct Arith<int32_t> : IntArith<int32_t, uint32_t> {};
template <> struct Arith<int64_t> : IntArith<int64_t, uint64_t> {};

template <class T> struct IsFloat { static constexpr bool value = false; };
template <> struct IsFloat<float> { static constexpr bool value = true; };
template <> struct IsFloat<double> { static constexpr bool value = true; };

// Parameters every element-wise kernel needs beyond its operands.
struct EwParams {
  int n_in;
  int op1, op2, epi;
  trs_scalar p0, p1;
  double e_const;  // log2(E_f32) for f32, E_f64 for f64 (see Arith::pow_e)
  int* div_flag;
};

template <class T>
__device__ __forceinline__ T apply_binop(int op, T a, T b, int* flag) {
  using A = Arith<T>;
  switch (op) {
    case TRS_ADD: return A::add(a, b);
    case TRS_SUB: return A::sub(a, b);
    case TRS_MUL: return A::mul(a, b);
    case TRS_DIV: return A::div(a, b, flag);
    default: return A::pow(a, b);
  }
}

// The unary maps of trs_unop, each in the order of operations of the
// reference code cited in include/trs.h.
template <class T>
__device__ __forceinline__ T apply_unop(const EwParams& p, T v) {
  using A = Arith<T>;
  const T one = T(1), zero = T(0);
  switch (p.epi) {
    case TRS_UN_NONE: return v;
    case TRS_UN_NEG: return A::neg(v);
    case TRS_UN_RELU: {  // x & map(x > 0 ? 1 : 0)
      return A::mul(v, v > zero ? one : zero);
    }
    case TRS_UN_SIGMOID: {  // autodiff/ops.rs:586-593
      // x >= 0: 1 / (1 + exp(-x)); otherwise e / (1 + e) with e = exp(x).
      // Both branches take exp(-|x|), so one exponential serves either
      // (a NaN fails x >= 0 and gives exp(NaN) / ..., NaN, as the reference).
      if constexpr (std::is_same<T, float>::value) {
        return expf32::sigmoid(v);  // the same steps, with Markstein's division
      } else {
        const T e = A::exp_nonpos(A::neg(A::abs(v)));
        return A::div(v >= zero ? one : e, A::add(one, e), nullptr);
      }
    }
    case TRS_UN_TANH: return A::tanh(v);
    case TRS_UN_ELU: {  // elu.rs:47-63
      T pos = A::mul(v, v > zero ? one : zero);
      T ex = A::pow_e_rounded_once(v, p.e_const);
      T neg = A::mul(A::mul(A::sub(ex, one), A::from(p.p0)), v <= zero ? one : zero);
      return A::add(pos, neg);
    }
    case TRS_UN_LEAKY_RELU: {  // leaky_relu.rs:39-52
      T pos = A::mul(v, v > zero ? one : zero);
      T neg = A::mul(A::mul(v, A::from(p.p0)), v <= zero ? one : zero);
      return A::add(pos, neg);
    }
    case TRS_UN_SELU: {  // selu.rs:52-70; p0 = alpha, p1 = lambda
      T lambda = A::from(p.p1), alpha = A::from(p.p0);
      T pos = A::mul(A::mul(v, lambda), v > zero ? one : zero);
      T ex = A::pow_e_rounded_once(v, p.e_const);
      T scale = A::mul(lambda, alpha);
      T neg = A::mul(A::mul(A::sub(ex, one), scale), v <= zero ? one : zero);
      return A::add(pos, neg);
    }
    case TRS_UN_EXP: return A::pow_e(v, p.e_const);
    case TRS_UN_LN: return A::ln(v);
    case TRS_UN_ABS: return A::abs(v);
    case TRS_UN_SIGN: return v > zero ? one : (v == zero ? zero : A::neg(one));
    case TRS_UN_CLAMP: {
      T lo = A::from(p.p0), hi = A::from(p.p1);
      return v < lo ? lo : (v > hi ? hi : v);
    }
    case TRS_UN_ADD_SCALAR: return A::add(v, A::from(p.p0));
    case TRS_UN_SUB_SCALAR: return A::sub(v, A::from(p.p0));
    case TRS_UN_RSUB_SCALAR: return A::sub(A::from(p.p0), v);
    case TRS_UN_MUL_SCALAR: return A::mul(v, A::from(p.p0));
    case TRS_UN_DIV_SCALAR: return A::div(v, A::from(p.p0), p.div_flag);
    case TRS_UN_POW_SCALAR: return A::pow(v, A::from(p.p0));
    case TRS_UN_RPOW_SCALAR: return A::pow(A::from(p.p0), v);
  }
  return v;
}

// The whole fused program on one element.
template <class T>
__device__ __forceinline__ T apply_program(const EwParams& p, T a, T b, T c) {
  T v = a;
  if (p.n_in >= 2) v = apply_binop<T>(p.op1, v, b, p.div_flag);
  if (p.n_in >= 3) v = apply_binop<T>(p.op2, v, c, p.div_flag);
  return apply_unop<T>(p, v);
}

// Programs without transcendentals (the host checks with is_simple_program):
// the same arithmetic as apply_program with no out-of-line calls, so the
// streaming kernels keep their registers for loads in flight.
template <class T>
__device__ __forceinline__ T apply_binop_simple(int op, T a, T b, int* flag) {
  using A = Arith<T>;
  switch (op) {
    case TRS_ADD: return A::add(a, b);
    case TRS_SUB: return A::sub(a, b);
    case TRS_MUL: return A::mul(a, b);
    default: return A::div(a, b, flag);
  }
}

template <class T>
__device__ __forceinline__ T apply_unop_simple(const EwParams& p, T v) {
  using A = Arith<T>;
  const T one = T(1), zero = T(0);
  switch (p.epi) {
    case TRS_UN_NEG: return A::neg(v);
    case TRS_UN_RELU: return A::mul(v, v > zero ? one : zero);
    case TRS_UN_LEAKY_RELU: {
      T pos = A::mul(v, v > zero ? one : zero);
      T neg = A::mul(A::mul(v, A::from(p.p0)), v <= zero ? one : zero);
      return A::add(pos, neg);
    }
    case TRS_UN_ABS: return A::abs(v);
    case TRS_UN_SIGN: return v > zero ? one : (v == zero ? zero : A::neg(one));
    case TRS_UN_CLAMP: {
      T lo = A::from(p.p0), hi = A::from(p.p1);
      return v < lo ? lo : (v > hi ? hi : v);
    }
    case TRS_UN_ADD_SCALAR: return A::add(v, A::from(p.p0));
    case TRS_UN_SUB_SCALAR: return A::sub(v, A::from(p.p0));
    case TRS_UN_RSUB_SCALAR: return A::sub(A::from(p.p0), v);
    case TRS_UN_MUL_SCALAR: return A::mul(v, A::from(p.p0));
    case TRS_UN_DIV_SCALAR: return A::div(v, A::from(p.p0), p.div_flag);
    default: return v;
  }
}

template <class T>
__device__ __forceinline__ T apply_program_simple(const EwParams& p, T a, T b, T c) {
  T v = a;
  if (p.n_in >= 2) v = apply_binop_simple<T>(p.op1, v, b, p.div_flag);
  if (p.n_in >= 3) v = apply_binop_simple<T>(p.op2, v, c, p.div_flag);
  return apply_unop_simple<T>(p, v);
}

// ---- programs known at compile time ---------------------------------------
// The hot fused patterns get their own kernel instantiations, so the element
// loop carries no op-code switch: PROG is a code from this list, or one of
// the kRun* codes (op codes read at run time, for every other program).
enum ProgCode {
  kRunSimple1 = 0, kRunSimple2, kRunSimple3,  // runtime ops, no transcendental
  kRunFull1, kRunFull2, kRunFull3,            // runtime ops, any
  kPack,          // x
  kAdd, kSub, kMul, kDiv,                     // a op b
  kMulAdd,        // (a & b) + c
  kMulAddRelu,    // ReLU((a & b) + c)
  kMulSigmoid,    // sigmoid(a & b)
  kSigmoid, kTanh, kRelu,                     // f(x)
  kNumProgs
};

__host__ __device__ constexpr int prog_inputs(int code) {
  return code == kRunSimple1 || code == kRunFull1 || code == kPack || code == kSigmoid || code == kTanh ||
                 code == kRelu
             ? 1
             : (code == kRunSimple3 || code == kRunFull3 || code == kMulAdd || code == kMulAddRelu ? 3 : 2);
}
__host__ __device__ constexpr bool prog_is_runtime(int code) { return code <= kRunFull3; }
__host__ __device__ constexpr bool prog_is_full_runtime(int code) { return code >= kRunFull1 && code <= kRunFull3; }

template <class T, int PROG>
__device__ __forceinline__ T apply_prog(const EwParams& p, T a, T b, T c) {
  using A = Arith<T>;
  const T one = T(1), zero = T(0);
  if constexpr (PROG <= kRunSimple3) {
    return apply_program_simple<T>(p, a, b, c);
  } else if constexpr (PROG <= kRunFull3) {
    return apply_program<T>(p, a, b, c);
  } else if constexpr (PROG == kPack) {
    return a;
  } else if constexpr (PROG == kAdd) {
    return A::add(a, b);
  } else if constexpr (PROG == kSub) {
    return A::sub(a, b);
  } else if constexpr (PROG == kMul) {
    return A::mul(a, b);
  } else if constexpr (PROG == kDiv) {
    return A::div(a, b, p.div_flag);
  } else if constexpr (PROG == kMulAdd) {
    return A::add(A::mul(a, b), c);
  } else if constexpr (PROG == kMulAddRelu) {
    const T v = A::add(A::mul(a, b), c);
    return A::mul(v, v > zero ? one : zero);
  } else if constexpr (PROG == kMulSigmoid) {
    EwParams q = p;
    q.epi = TRS_UN_SIGMOID;
    return apply_unop<T>(q, A::mul(a, b));
  } else if constexpr (PROG == kSigmoid) {
    EwParams q = p;
    q.epi = TRS_UN_SIGMOID;
    return apply_unop<T>(q, a);
  } else if constexpr (PROG == kTanh) {
    return A::tanh(a);
  } else {  // kRelu
    return A::mul(a, a > zero ? one : zero);
  }
}

// ---- reductions ------------------------------------------------------------

// Sum of one f64 (or wrapping integer) value per thread over a block whose
// size is a multiple of 32; the result is valid in thread 0.  The order of the
// additions is fixed, so the result is deterministic.
template <class Acc>
__device__ __forceinline__ Acc block_sum(Acc v, Acc* smem /* >= 32 */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = v + __shfl_down_sync(0xffffffffu, v, o);
  __syncthreads();  // smem may be reused from a previous call
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (warp == 0) {
    v = lane < nw ? smem[lane] : Acc(0);
    for (int o = 16; o > 0; o >>= 1) v = v + __shfl_down_sync(0xffffffffu, v, o);
  }
  return v;
}

// Running maximum with the reference's semantics (max_axis, base.rs:1404-1411;
// argmax_axis, base.rs:1467-1478): strict `>` from the first element, so a NaN
// never replaces a value and ties keep the lowest index.  A partial state
// covers a subset of the axis: `idx` < 0 means it holds no candidate yet.
// NaNs are skipped here; a NaN at index 0 (which the reference keeps) is
// applied by the caller after the reduction.
template <class T>
struct MaxState {
  T val;
  int64_t idx;
};

template <class T>
__device__ __forceinline__ bool is_nan_val(T v) { return v != v; }

template <class T>
__device__ __forceinline__ void max_push(MaxState<T>& s, T v, int64_t k) {
  if (is_nan_val(v)) return;
  if (s.idx < 0 || v > s.val) { s.val = v; s.idx = k; }
}

// Combine two partial states; ties go to the lower index.
template <class T>
__device__ __forceinline__ MaxState<T> max_combine(MaxState<T> a, MaxState<T> b) {
  if (a.idx < 0) return b;
  if (b.idx < 0) return a;
  if (b.val > a.val) return b;
  if (a.val > b.val) return a;
  return b.idx < a.idx ? b : a;
}

template <class T>
__device__ __forceinline__ MaxState<T> shfl_down_max(MaxState<T> s, int o) {
  MaxState<T> r;
  r.val = __shfl_down_sync(0xffffffffu, s.val, o);
  r.idx = __shfl_down_sync(0xffffffffu, s.idx, o);
  return r;
}

template <class T>
__device__ __forceinline__ MaxState<T> warp_max(MaxState<T> s) {
  for (int o = 16; o > 0; o >>= 1) s = max_combine(s, shfl_down_max(s, o));
  return s;
}

template <class T>
__device__ __forceinline__ MaxState<T> block_max(MaxState<T> s, MaxState<T>* smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  s = warp_max(s);
  __syncthreads();
  if (lane == 0) smem[warp] = s;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (warp == 0) {
    MaxState<T> e;
    e.val = T(0);
    e.idx = -1;
    s = lane < nw ? smem[lane] : e;
    s = warp_max(s);
  }
  return s;
}

}  // namespace trs
