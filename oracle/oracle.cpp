// oracle.cpp -- CPU restatement of tensorrs' strided broadcast-elementwise and
// axis-reduction algorithms (GooseKIller/Tensors, crate `tensorrs` 0.4.1).
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker the GPU path is compared
// against, and the CPU baseline the benchmark reports beside it.  Nothing in
// the shipped library links, loads or calls it.
//
// Each function restates the reference function cited above it, step by step
// and in the same order of floating-point operations, so that f32/f64 results
// round exactly as the reference's do.  Transcendentals call glibc's libm
// (expf, tanhf, powf, logf and their f64 forms), which is what Rust's std
// calls on x86_64-linux-gnu.  Build flags (Makefile): -O2 -ffp-contract=off
// -fno-fast-math, so no FMA contraction and no reassociation.
//
// Parallelism mirrors the reference's rayon split (ops.rs:10-25): loops over
// output elements run on OpenMP threads when they have PARALLEL_THRESHOLD or
// more outputs, serially otherwise; the index-vector builds (storage_indices)
// and the `sum` fold stay serial as in the reference.  Results do not depend
// on the thread count.
//
// Pinned against the reference's own unit tests and doctests through the
// golden vectors in tests/golden/reference_kats.json.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>
#include <omp.h>

namespace {

constexpr int kMaxDims = 8;
constexpr int64_t kParallelThreshold = 8192;  // ops.rs:12

// Same layout as trs_view in include/trs.h, but `data` is a host pointer.
struct View {
  void* data;
  int64_t storage_len;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[kMaxDims];
  int64_t strides[kMaxDims];
  int64_t offset;
};

enum Dtype { F32 = 0, F64 = 1, I32 = 2, I64 = 3 };
enum Status { OK = 0, NONE = 1, ERR_SHAPE = 2, ERR_AXIS = 3, ERR_EMPTY = 4,
              ERR_DTYPE = 6, ERR_ARG = 12, ERR_DIV_ZERO = 13 };
enum BinOp { ADD = 0, SUB = 1, MUL = 2, DIV = 3, POW = 4 };
enum UnOp { UN_NONE = 0, UN_NEG, UN_RELU, UN_SIGMOID, UN_TANH, UN_ELU,
            UN_LEAKY_RELU, UN_SELU, UN_EXP, UN_LN, UN_ABS, UN_SIGN, UN_CLAMP,
            UN_ADD_S, UN_SUB_S, UN_RSUB_S, UN_MUL_S, UN_DIV_S, UN_POW_S,
            UN_RPOW_S };

int g_threads = 1;

// A tensor as the reference holds it: shape, signed strides, offset, storage.
template <class T>
struct Tensor {
  const T* data;
  std::vector<int64_t> shape;
  std::vector<int64_t> strides;
  int64_t offset;
  std::vector<T> owned;  // storage when this tensor owns its data

  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

template <class T>
Tensor<T> from_view(const View* v) {
  Tensor<T> t;
  t.data = static_cast<const T*>(v->data);
  t.shape.assign(v->shape, v->shape + v->ndim);
  t.strides.assign(v->strides, v->strides + v->ndim);
  t.offset = v->offset;
  return t;
}

// compute_strides (base.rs:37-45): row-major strides of a shape.
std::vector<int64_t> compute_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  int64_t step = 1;
  for (int i = (int)shape.size() - 1; i >= 0; --i) {
    s[i] = step;
    step *= shape[i];
  }
  return s;
}

// Tensor::new (base.rs:183-197): owned contiguous tensor.
template <class T>
Tensor<T> make_tensor(std::vector<T>&& data, std::vector<int64_t> shape) {
  Tensor<T> t;
  t.owned = std::move(data);
  t.data = t.owned.data();
  t.strides = compute_strides(shape);
  t.shape = std::move(shape);
  t.offset = 0;
  return t;
}

// Tensor::scalar (base.rs:212-219): shape [1], stride [0].
template <class T>
Tensor<T> make_scalar(T v) {
  Tensor<T> t;
  t.owned = {v};
  t.data = t.owned.data();
  t.shape = {1};
  t.strides = {0};
  t.offset = 0;
  return t;
}

template <class T>
Tensor<T> view_of(const Tensor<T>& t) {  // shallow_copy (base.rs:450-457)
  Tensor<T> v;
  v.data = t.data;
  v.shape = t.shape;
  v.strides = t.strides;
  v.offset = t.offset;
  return v;
}

// Runs f(i) for i in [0, n): on OpenMP threads when n >= PARALLEL_THRESHOLD
// (the rayon split of ops.rs:16-25 and base.rs:1060-1103), serially below.
template <class F>
void for_outputs(int64_t n, F f) {
  if (n < kParallelThreshold || g_threads <= 1) {
    for (int64_t i = 0; i < n; ++i) f(i);
  } else {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t i = 0; i < n; ++i) f(i);
  }
}

// broadcast_shape (ops.rs:27-45).
bool broadcast_shape(const std::vector<int64_t>& a, const std::vector<int64_t>& b,
                     std::vector<int64_t>* out) {
  size_t nd = a.size() > b.size() ? a.size() : b.size();
  std::vector<int64_t> r;
  for (size_t i = 0; i < nd; ++i) {
    int64_t da = i < a.size() ? a[a.size() - 1 - i] : 1;
    int64_t db = i < b.size() ? b[b.size() - 1 - i] : 1;
    if (da == db || da == 1 || db == 1)
      r.push_back(da > db ? da : db);
    else
      return false;
  }
  out->assign(r.rbegin(), r.rend());
  return true;
}

// broadcast_to (base.rs:556-599): stride 0 on every broadcast dimension.
template <class T>
bool broadcast_to(const Tensor<T>& t, const std::vector<int64_t>& target, Tensor<T>* out) {
  size_t src = t.shape.size(), dst = target.size();
  if (src > dst) return false;
  std::vector<int64_t> ns(dst, 0);
  for (size_t i = 0; i < dst; ++i) {
    int64_t dd = target[dst - 1 - i];
    int64_t sd = i < src ? t.shape[src - 1 - i] : 1;
    int64_t ss = i < src ? t.strides[src - 1 - i] : 0;
    if (sd == dd)
      ns[dst - 1 - i] = ss;
    else if (sd == 1)
      ns[dst - 1 - i] = 0;
    else
      return false;
  }
  out->data = t.data;
  out->shape = target;
  out->strides = ns;
  out->offset = t.offset;
  return true;
}

// storage_indices (base.rs:404-428): serial logical -> storage index list.
template <class T>
std::vector<int64_t> storage_indices(const Tensor<T>& t) {
  size_t nd = t.shape.size();
  if (nd == 0) return {};
  int64_t n = t.numel();
  std::vector<int64_t> suffix(nd, 1);
  for (int i = (int)nd - 2; i >= 0; --i) suffix[i] = suffix[i + 1] * t.shape[i + 1];
  std::vector<int64_t> idx;
  idx.reserve(n);
  for (int64_t linear = 0; linear < n; ++linear) {
    int64_t rem = linear, at = t.offset;
    for (size_t i = 0; i < nd; ++i) {
      int64_t coord = rem / suffix[i];
      rem %= suffix[i];
      at += t.strides[i] * coord;
    }
    idx.push_back(at);
  }
  return idx;
}

// packed_data (base.rs:430-434).
template <class T>
std::vector<T> packed_data(const Tensor<T>& t) {
  std::vector<int64_t> idx = storage_indices(t);
  std::vector<T> out(idx.size());
  for (size_t i = 0; i < idx.size(); ++i) out[i] = t.data[idx[i]];
  return out;
}

// is_contiguous (base.rs:616-631): size-1 dimensions are skipped.
template <class T>
bool is_contiguous(const Tensor<T>& t) {
  int64_t expected = 1;
  for (int i = (int)t.shape.size() - 1; i >= 0; --i) {
    if (t.shape[i] == 1) continue;
    if (t.strides[i] != expected) return false;
    expected *= t.shape[i];
  }
  return true;
}

// ---- scalar arithmetic of the element types --------------------------------

template <class T> struct Arith;

template <> struct Arith<float> {
  static float add(float a, float b) { return a + b; }
  static float sub(float a, float b) { return a - b; }
  static float mul(float a, float b) { return a * b; }
  static bool div(float a, float b, float* r) { *r = a / b; return true; }
  static float pow(float a, float b) { return ::powf(a, b); }
  static float exp(float a) { return ::expf(a); }
  static float tanh(float a) { return ::tanhf(a); }
  static float ln(float a) { return ::logf(a); }
  static float e() { return 2.7182817f; }  // std::f32::consts::E rounded to f32
  static float from(double f, int64_t) { return (float)f; }
  static float neg(float a) { return -a; }
  static float abs(float a) { return std::fabs(a); }
};

template <> struct Arith<double> {
  static double add(double a, double b) { return a + b; }
  static double sub(double a, double b) { return a - b; }
  static double mul(double a, double b) { return a * b; }
  static bool div(double a, double b, double* r) { *r = a / b; return true; }
  static double pow(double a, double b) { return ::pow(a, b); }
  static double exp(double a) { return ::exp(a); }
  static double tanh(double a) { return ::tanh(a); }
  static double ln(double a) { return ::log(a); }
  static double e() { return 2.718281828459045; }  // std::f64::consts::E
  static double from(double f, int64_t) { return f; }
  static double neg(double a) { return -a; }
  static double abs(double a) { return std::fabs(a); }
};

// Integers wrap on add/sub/mul (the reference's release build) and panic on
// division by zero or MIN / -1 (Rust panics on both in every build).
template <class I>
struct IntArith {
  using U = typename std::make_unsigned<I>::type;
  static I add(I a, I b) { return (I)((U)a + (U)b); }
  static I sub(I a, I b) { return (I)((U)a - (U)b); }
  static I mul(I a, I b) { return (I)((U)a * (U)b); }
  static bool div(I a, I b, I* r) {
    if (b == 0) return false;
    if (b == -1 && a == std::numeric_limits<I>::min()) return false;
    *r = a / b;
    return true;
  }
  static I pow(I, I) { return 0; }
  static I exp(I) { return 0; }
  static I tanh(I) { return 0; }
  static I ln(I) { return 0; }
  static I e() { return 0; }
  static I from(double, int64_t i) { return (I)i; }
  static I neg(I a) { return (I)((U)0 - (U)a); }
  static I abs(I a) { return a < 0 ? neg(a) : a; }
};
template <> struct Arith<int32_t> : IntArith<int32_t> {};
template <> struct Arith<int64_t> : IntArith<int64_t> {};

template <class T>
bool apply_bin(int op, T a, T b, T* r) {
  using A = Arith<T>;
  switch (op) {
    case ADD: *r = A::add(a, b); return true;
    case SUB: *r = A::sub(a, b); return true;
    case MUL: *r = A::mul(a, b); return true;
    case DIV: return A::div(a, b, r);
    case POW: *r = A::pow(a, b); return true;
  }
  return false;
}

const char* bin_msg(int op) {
  switch (op) {
    case ADD: return "!!!Add: incompatible shapes!!!";
    case SUB: return "!!!Sub: incompatible shapes!!!";
    case MUL: return "!!!MulElems: incompatible shapes!!!";
    case DIV: return "!!!DIV: incompatible shapes!!!";
    default: return "!!!Powf: incompatible shapes!!!";
  }
}

thread_local const char* g_msg = "";
thread_local std::string g_msg_buf;  // formatted panic texts (g_msg points here)

std::string shape_text(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

// binary_op (ops.rs:240-300), fast path and broadcast path.
template <class T>
int binary_op(int op, const Tensor<T>& a, const Tensor<T>& b, Tensor<T>* out) {
  if (a.shape == b.shape && is_contiguous(a) && is_contiguous(b)) {
    int64_t n = a.numel();
    const T* ad = a.data + a.offset;
    const T* bd = b.data + b.offset;
    std::vector<T> o(n);
    int bad = 0;
    for_outputs(n, [&](int64_t i) {
      if (!apply_bin<T>(op, ad[i], bd[i], &o[i])) bad = 1;
    });
    if (bad) { g_msg = "attempt to divide by zero"; return ERR_DIV_ZERO; }
    *out = make_tensor(std::move(o), a.shape);
    return OK;
  }
  std::vector<int64_t> shape;
  if (!broadcast_shape(a.shape, b.shape, &shape)) { g_msg = bin_msg(op); return ERR_SHAPE; }
  Tensor<T> av, bv;
  // broadcast_shape maps a (0, 1) pair to 1, after which broadcast_to fails and
  // the reference panics with this message (ops.rs:271-272)
  if (!broadcast_to(a, shape, &av) || !broadcast_to(b, shape, &bv)) {
    g_msg = "broadcast_to failed (bug)";
    return ERR_SHAPE;
  }
  std::vector<int64_t> ai = storage_indices(av);
  std::vector<int64_t> bi = storage_indices(bv);
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  std::vector<T> o(n);
  int bad = 0;
  for_outputs(n, [&](int64_t i) {
    if (!apply_bin<T>(op, a.data[ai[i]], b.data[bi[i]], &o[i])) bad = 1;
  });
  if (bad) { g_msg = "attempt to divide by zero"; return ERR_DIV_ZERO; }
  *out = make_tensor(std::move(o), shape);
  return OK;
}

// Tensor::map (base.rs:1708-1716): packed copy, then f on every element.
template <class T, class F>
Tensor<T> map(const Tensor<T>& t, F f) {
  std::vector<T> d = packed_data(t);
  for_outputs((int64_t)d.size(), [&](int64_t i) { d[i] = f(d[i]); });
  return make_tensor(std::move(d), t.shape);
}

template <class T>
Tensor<T> mask_pos(const Tensor<T>& x) {  // map(v > 0 ? 1 : 0), relu.rs:36-39
  return map(x, [](T v) { return v > T(0) ? T(1) : T(0); });
}
template <class T>
Tensor<T> mask_nonpos(const Tensor<T>& x) {  // map(v <= 0 ? 1 : 0), elu.rs:51-54
  return map(x, [](T v) { return v <= T(0) ? T(1) : T(0); });
}

template <class T>
int bin(int op, const Tensor<T>& a, const Tensor<T>& b, Tensor<T>* out) {
  return binary_op<T>(op, a, b, out);
}

// The unary maps, each as the reference's caller composes it.
template <class T>
int unary(int op, const Tensor<T>& x, T p0, T p1, Tensor<T>* out) {
  using A = Arith<T>;
  int st = OK;
  switch (op) {
    case UN_NONE:  // packed_data (base.rs:430)
      *out = make_tensor(packed_data(x), x.shape);
      return OK;
    case UN_NEG:  // Neg for &Tensor (ops.rs:168-175)
      *out = map(x, [](T v) { return A::neg(v); });
      return OK;
    case UN_RELU: {  // ReLU::forward (relu.rs:32-42): x & mask
      Tensor<T> m = mask_pos(x);
      return bin(MUL, x, m, out);
    }
    case UN_SIGMOID:  // sigmoid_op (autodiff/ops.rs:585-594)
      *out = map(x, [](T v) {
        if (v >= T(0)) return (T)(T(1) / (T(1) + A::exp(-v)));
        T e = A::exp(v);
        return (T)(e / (T(1) + e));
      });
      return OK;
    case UN_TANH:  // tanh_op (autodiff/ops.rs:547-548)
      *out = map(x, [](T v) { return A::tanh(v); });
      return OK;
    case UN_ELU: {  // ELU::forward (elu.rs:43-64)
      Tensor<T> mp = mask_pos(x), mn = mask_nonpos(x), pos, ex, t1, t2, neg;
      if ((st = bin(MUL, x, mp, &pos))) return st;
      if ((st = bin(POW, make_scalar(A::e()), x, &ex))) return st;
      if ((st = bin(SUB, ex, make_scalar(T(1)), &t1))) return st;
      if ((st = bin(MUL, t1, make_scalar(p0), &t2))) return st;
      if ((st = bin(MUL, t2, mn, &neg))) return st;
      return bin(ADD, pos, neg, out);
    }
    case UN_LEAKY_RELU: {  // LeakyReLU::forward (leaky_relu.rs:35-53)
      Tensor<T> mp = mask_pos(x), mn = mask_nonpos(x), pos, t1, neg;
      if ((st = bin(MUL, x, mp, &pos))) return st;
      if ((st = bin(MUL, x, make_scalar(p0), &t1))) return st;
      if ((st = bin(MUL, t1, mn, &neg))) return st;
      return bin(ADD, pos, neg, out);
    }
    case UN_SELU: {  // SELU::forward (selu.rs:48-71); p0 = alpha, p1 = lambda
      Tensor<T> mp = mask_pos(x), mn = mask_nonpos(x), t0, pos, ex, t1, t2, neg;
      if ((st = bin(MUL, x, make_scalar(p1), &t0))) return st;
      if ((st = bin(MUL, t0, mp, &pos))) return st;
      if ((st = bin(POW, make_scalar(A::e()), x, &ex))) return st;
      T scale = A::mul(p1, p0);  // self.lambda * self.alpha
      if ((st = bin(SUB, ex, make_scalar(T(1)), &t1))) return st;
      if ((st = bin(MUL, t1, make_scalar(scale), &t2))) return st;
      if ((st = bin(MUL, t2, mn, &neg))) return st;
      return bin(ADD, pos, neg, out);
    }
    case UN_EXP:  // Tensor::scalar(E) ^ x (elu.rs:58-60)
      return bin(POW, make_scalar(A::e()), x, out);
    case UN_LN:
      *out = map(x, [](T v) { return A::ln(v); });
      return OK;
    case UN_ABS:
      *out = map(x, [](T v) { return A::abs(v); });
      return OK;
    case UN_SIGN:  // Float::sign (src/lib.rs:151-159)
      *out = map(x, [](T v) { return v > T(0) ? T(1) : (v == T(0) ? T(0) : T(-1)); });
      return OK;
    case UN_CLAMP:  // clamp_op (autodiff/ops.rs:247)
      *out = map(x, [p0, p1](T v) { return v < p0 ? p0 : (v > p1 ? p1 : v); });
      return OK;
    // scalar operators (ops.rs:52-233): packed copy then x op= s in place
    case UN_ADD_S: *out = map(x, [p0](T v) { return A::add(v, p0); }); return OK;
    case UN_SUB_S: *out = map(x, [p0](T v) { return A::sub(v, p0); }); return OK;
    case UN_RSUB_S: *out = map(x, [p0](T v) { return A::sub(p0, v); }); return OK;
    case UN_MUL_S: *out = map(x, [p0](T v) { return A::mul(v, p0); }); return OK;
    case UN_DIV_S: {
      int bad = 0;
      *out = map(x, [p0, &bad](T v) { T r{}; if (!A::div(v, p0, &r)) bad = 1; return r; });
      if (bad) { g_msg = "attempt to divide by zero"; return ERR_DIV_ZERO; }
      return OK;
    }
    case UN_POW_S:  // VarRef ^ scalar = powf_op(x, scalar leaf) (impl_ops.rs:95-99)
      return bin(POW, x, make_scalar(p0), out);
    case UN_RPOW_S:  // Tensor::scalar(s) ^ x
      return bin(POW, make_scalar(p0), x, out);
  }
  g_msg = "unknown unary op";
  return ERR_ARG;
}

// sum (base.rs:1024-1030): packed copy, then a serial left-to-right fold.
template <class T>
T sum_all(const Tensor<T>& t) {
  T ans = T(0);
  std::vector<T> d = packed_data(t);
  for (T v : d) ans = Arith<T>::add(ans, v);
  return ans;
}

// sum_axis (base.rs:1051-1107) and sum_axis_keepdim (base.rs:1534-1594):
// per output, a sequential sum over the axis in increasing k, from 0.
template <class T>
int sum_axis(const Tensor<T>& t, int axis, bool keepdim, Tensor<T>* out) {
  if (axis < 0 || axis >= (int)t.shape.size()) { g_msg = "!!!Axis index out of range!!!"; return ERR_AXIS; }
  std::vector<int64_t> out_shape = t.shape;
  int64_t rdim = t.shape[axis];
  std::vector<int64_t> oshape_nokeep = t.shape;
  oshape_nokeep.erase(oshape_nokeep.begin() + axis);
  if (keepdim) out_shape[axis] = 1; else out_shape = oshape_nokeep;
  int64_t n = 1;
  for (int64_t d : oshape_nokeep) n *= d;
  std::vector<T> o(n);
  int64_t stride = t.strides[axis];
  for_outputs(n, [&](int64_t oi) {
    int64_t tmp = oi, base = t.offset;
    for (int i = (int)oshape_nokeep.size() - 1; i >= 0; --i) {
      int64_t d = oshape_nokeep[i];
      int64_t idx = tmp % d;
      tmp /= d;
      int in_axis = i >= axis ? i + 1 : i;
      base += idx * t.strides[in_axis];
    }
    T acc = T(0);
    for (int64_t k = 0; k < rdim; ++k) acc = Arith<T>::add(acc, t.data[base + k * stride]);
    o[oi] = acc;
  });
  *out = make_tensor(std::move(o), out_shape);
  return OK;
}

// max_axis (base.rs:1396-1436) / argmax_axis (base.rs:1458-1505): strict `>`
// running maximum seeded with the first element along the axis.
template <class T>
int max_argmax_axis(const Tensor<T>& t, int axis, std::vector<T>* vals,
                    std::vector<int64_t>* idxs, std::vector<int64_t>* out_shape) {
  if (axis < 0 || axis >= (int)t.shape.size()) { g_msg = "!!!Axis index out of range!!!"; return ERR_AXIS; }
  std::vector<int64_t> os = t.shape;
  int64_t rdim = os[axis];
  os.erase(os.begin() + axis);
  if (rdim <= 0) { g_msg = "!!!Cannot reduce an empty axis!!!"; return ERR_EMPTY; }
  int64_t n = 1;
  for (int64_t d : os) n *= d;
  vals->assign(n, T(0));
  idxs->assign(n, 0);
  int64_t stride = t.strides[axis];
  for_outputs(n, [&](int64_t oi) {
    int64_t tmp = oi, base = t.offset;  // reduce_base_offset (base.rs:1519-1531)
    for (int i = (int)os.size() - 1; i >= 0; --i) {
      int64_t idx = tmp % os[i];
      tmp /= os[i];
      int in_axis = i >= axis ? i + 1 : i;
      base += idx * t.strides[in_axis];
    }
    T best = t.data[base];
    int64_t at = 0;
    for (int64_t k = 1; k < rdim; ++k) {
      T v = t.data[base + k * stride];
      if (v > best) { best = v; at = k; }
    }
    (*vals)[oi] = best;
    (*idxs)[oi] = at;
  });
  *out_shape = os;
  return OK;
}

// reduce_broadcast_grad (base.rs:1651-1686).
template <class T>
int reduce_broadcast_grad(const Tensor<T>& g, const std::vector<int64_t>& target, Tensor<T>* out) {
  if (g.shape.size() < target.size()) {
    if (g.numel() == 1) {  // a scalar broadcasts to any shape (from_num)
      T v = g.data[g.offset];
      int64_t n = 1;
      for (int64_t d : target) n *= d;
      *out = make_tensor(std::vector<T>(n, v), target);
      return OK;
    }
    std::vector<int64_t> es(target.size() - g.shape.size(), 1);
    es.insert(es.end(), g.shape.begin(), g.shape.end());
    Tensor<T> t = make_tensor(packed_data(g), es);
    return reduce_broadcast_grad(t, target, out);
  }
  Tensor<T> cur = view_of(g);
  std::vector<Tensor<T>> keep;  // keeps the intermediates alive
  while (cur.shape.size() > target.size()) {
    Tensor<T> nx;
    sum_axis(cur, 0, false, &nx);
    keep.push_back(std::move(nx));
    cur = view_of(keep.back());
  }
  for (size_t i = 0; i < target.size(); ++i) {
    int64_t s = cur.shape[i], tt = target[i];
    if (s == tt) continue;
    if (tt == 1) {
      Tensor<T> nx;
      sum_axis(cur, (int)i, true, &nx);
      keep.push_back(std::move(nx));
      cur = view_of(keep.back());
    } else {
      return NONE;
    }
  }
  // a rank-0 result holds one element (see write_out)
  *out = make_tensor(cur.shape.empty() ? std::vector<T>{cur.data[cur.offset]} : packed_data(cur), cur.shape);
  return OK;
}

// SoftMax::forward (activation/softmax.rs:42-68), last axis.
template <class T>
int softmax_lastdim(const Tensor<T>& x, Tensor<T>* out) {
  int axis = (int)x.shape.size() - 1;
  std::vector<T> mv;
  std::vector<int64_t> mi, os;
  int st = max_argmax_axis(x, axis, &mv, &mi, &os);
  if (st) return st;
  std::vector<int64_t> kd = x.shape;
  kd[axis] = 1;
  Tensor<T> mx = make_tensor(std::move(mv), kd), shifted, ex, s;
  if ((st = bin(SUB, x, mx, &shifted))) return st;
  if ((st = bin(POW, make_scalar(Arith<T>::e()), shifted, &ex))) return st;
  if ((st = sum_axis(ex, axis, true, &s))) return st;
  return bin(DIV, ex, s, out);
}

// Copies a result out in row-major order.  A rank-0 result (what summing
// every axis away leaves) is written as its one element; the reference's
// storage_indices would list no element for it (base.rs:406-408).
template <class T>
void write_out(const Tensor<T>& t, void* out, int64_t* out_shape, int32_t* out_ndim) {
  std::vector<T> d = t.shape.empty() ? std::vector<T>{t.data[t.offset]}
                     : is_contiguous(t) && t.offset == 0 && t.owned.size() == (size_t)t.numel()
                         ? t.owned : packed_data(t);
  std::memcpy(out, d.data(), d.size() * sizeof(T));
  if (out_shape) for (size_t i = 0; i < t.shape.size(); ++i) out_shape[i] = t.shape[i];
  if (out_ndim) *out_ndim = (int32_t)t.shape.size();
}

template <class T>
T scalar_of(double f, int64_t i) { return Arith<T>::from(f, i); }

// splitmix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014): the i-th output of the stream seeded by `seed`.
inline uint64_t splitmix64(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// unfold_2d (linalg/tensor/conv.rs:360-418): every window of a packed
// [batch, channels, height, width] image as a row of channels * kh * kw values
// in (c, i, j) order, rows in (n, oh, ow) order; a window position inside the
// padding stays 0.
template <class T>
std::vector<T> unfold_2d(const std::vector<T>& src, int64_t batch, int64_t channels, int64_t height,
                         int64_t width, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                         int64_t* out_h, int64_t* out_w) {
  const int64_t oh_n = (height + 2 * ph - kh) / sh + 1, ow_n = (width + 2 * pw - kw) / sw + 1;
  const int64_t patch = channels * kh * kw;
  std::vector<T> data((size_t)(batch * oh_n * ow_n * patch), T(0));
  for_outputs(batch * oh_n * ow_n, [&](int64_t row) {
    const int64_t ow = row % ow_n, oh = (row / ow_n) % oh_n, n = row / (oh_n * ow_n);
    T* out = data.data() + row * patch;
    for (int64_t c = 0; c < channels; ++c)
      for (int64_t i = 0; i < kh; ++i) {
        const int64_t y = oh * sh + i - ph;
        if (y < 0 || y >= height) continue;
        for (int64_t j = 0; j < kw; ++j) {
          const int64_t x = ow * sw + j - pw;
          if (x < 0 || x >= width) continue;
          out[c * kh * kw + i * kw + j] = src[(size_t)(((n * channels + c) * height + y) * width + x)];
        }
      }
  });
  *out_h = oh_n;
  *out_w = ow_n;
  return data;
}

// fold_2d (conv.rs:434-488): adds the rows of an unfold back into a zeroed
// [batch, channels, height, width] image, image by image, rows in (oh, ow)
// order, each row in (c, i, j) order.
template <class T>
std::vector<T> fold_2d(const std::vector<T>& src, int64_t batch, int64_t channels, int64_t height, int64_t width,
                       int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw) {
  const int64_t oh_n = (height + 2 * ph - kh) / sh + 1, ow_n = (width + 2 * pw - kw) / sw + 1;
  const int64_t patch = channels * kh * kw;
  std::vector<T> data((size_t)(batch * channels * height * width), T(0));
  for_outputs(batch, [&](int64_t n) {
    T* image = data.data() + n * channels * height * width;
    for (int64_t oh = 0; oh < oh_n; ++oh)
      for (int64_t ow = 0; ow < ow_n; ++ow) {
        const int64_t row = (n * oh_n + oh) * ow_n + ow;
        for (int64_t c = 0; c < channels; ++c)
          for (int64_t i = 0; i < kh; ++i) {
            const int64_t y = oh * sh + i - ph;
            if (y < 0 || y >= height) continue;
            for (int64_t j = 0; j < kw; ++j) {
              const int64_t x = ow * sw + j - pw;
              if (x < 0 || x >= width) continue;
              T& px = image[(c * height + y) * width + x];
              px = Arith<T>::add(px, src[(size_t)(row * patch + c * kh * kw + i * kw + j)]);
            }
          }
      }
  });
  return data;
}

// Tensor::matmul (linalg/tensor/base.rs:896-1013): A [..., M, K] times
// B [..., K, N], the batch dimensions broadcast against each other (1 against
// anything; a 0 against a 1 gives 1, as in broadcast_shape); every output is
// `acc = acc + a * b` over k = 0 .. K-1 from acc = 0 in the element type, both
// operands read through their strides.
template <class T>
int matmul(const Tensor<T>& a, const Tensor<T>& b, std::vector<T>* out, std::vector<int64_t>* out_shape) {
  const size_t an = a.shape.size(), bn = b.shape.size();
  if (an < 2 || bn < 2) { g_msg = "matmul: both tensors must be at least 2D"; return ERR_SHAPE; }
  const int64_t m = a.shape[an - 2], k = a.shape[an - 1], n = b.shape[bn - 1];
  if (k != b.shape[bn - 2]) {
    g_msg = "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])";
    return ERR_SHAPE;
  }
  std::vector<int64_t> ab(a.shape.begin(), a.shape.end() - 2), bb(b.shape.begin(), b.shape.end() - 2), batch;
  if (!broadcast_shape(ab, bb, &batch)) { g_msg = "matmul: batch shapes not broadcastable"; return ERR_SHAPE; }
  std::vector<int64_t> os = batch;
  os.push_back(m);
  os.push_back(n);
  int64_t len = 1;
  for (int64_t d : os) len *= d;
  const size_t on = os.size();
  std::vector<int64_t> suffix(on, 1);
  for (int i = (int)on - 2; i >= 0; --i) suffix[i] = suffix[i + 1] * os[i + 1];
  auto batch_offset = [&](const Tensor<T>& t, const int64_t* coords) {
    const size_t tn = t.shape.size();
    int64_t off = t.offset;
    for (size_t ax = 0; ax + 2 < tn; ++ax) {
      const size_t oax = on - tn + ax;
      const int64_t c = t.shape[ax] == 1 ? 0 : coords[oax];
      off += t.strides[ax] * c;
    }
    return off;
  };
  out->assign((size_t)len, T(0));
  T* o = out->data();
  for_outputs(len, [&](int64_t idx) {
    int64_t coords[kMaxDims + 2];
    int64_t rem = idx;
    for (size_t ax = 0; ax < on; ++ax) {
      coords[ax] = rem / suffix[ax];
      rem %= suffix[ax];
    }
    const int64_t i = coords[on - 2], j = coords[on - 1];
    const int64_t a_base = batch_offset(a, coords) + a.strides[an - 2] * i;
    const int64_t b_base = batch_offset(b, coords) + b.strides[bn - 1] * j;
    const int64_t a_step = a.strides[an - 1], b_step = b.strides[bn - 2];
    T acc = T(0);
    for (int64_t kk = 0; kk < k; ++kk)
      acc = Arith<T>::add(acc, Arith<T>::mul(a.data[a_base + a_step * kk], b.data[b_base + b_step * kk]));
    o[idx] = acc;
  });
  *out_shape = os;
  return OK;
}

// unfold_dims (linalg/tensor/conv.rs:490-510): the checks of unfold_2d.
template <class T>
int unfold_dims(const Tensor<T>& x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw) {
  if (x.shape.size() != 4) {
    g_msg_buf = "!!!unfold_2d() expects [batch, channels, height, width], got " + shape_text(x.shape) + "!!!";
    g_msg = g_msg_buf.c_str();
    return ERR_SHAPE;
  }
  if (sh <= 0 || sw <= 0) { g_msg = "!!!unfold_2d(): stride must be positive!!!"; return ERR_ARG; }
  if (kh < 0 || kw < 0 || ph < 0 || pw < 0 || x.shape[2] + 2 * ph < kh || x.shape[3] + 2 * pw < kw) {
    g_msg_buf = "!!!unfold_2d(): a (" + std::to_string(kh) + ", " + std::to_string(kw) +
                ") kernel does not fit a " + std::to_string(x.shape[2]) + "x" + std::to_string(x.shape[3]) +
                " input padded by (" + std::to_string(ph) + ", " + std::to_string(pw) + ")!!!";
    g_msg = g_msg_buf.c_str();
    return ERR_SHAPE;
  }
  return OK;
}

// The checks of pool_dims (nn/pool.rs:36-41), with_stride (pool.rs:115-118)
// and unfold_dims (conv.rs:490-510).
template <class T>
int pool_dims(const Tensor<T>& x, int64_t kh, int64_t kw, int64_t sh, int64_t sw) {
  if (x.shape.size() != 4) { g_msg = "!!!MaxPool2d expects [batch, channels, height, width]!!!"; return ERR_SHAPE; }
  if (sh <= 0 || sw <= 0) { g_msg = "!!!MaxPool2d: stride must be positive!!!"; return ERR_ARG; }
  if (kh < 0 || kw < 0 || x.shape[2] < kh || x.shape[3] < kw) { g_msg = "input smaller than the kernel"; return ERR_SHAPE; }
  return OK;
}

// MaxPool2d::forward (pool.rs:137-144) and AvgPool2d::forward (pool.rs:223-233):
// windows_per_channel (pool.rs:25-33: reshape to [N*C, 1, H, W], unfold), then
// max_axis(1), or sum_axis(1) divided by kh*kw -- a VarRef divided by a scalar
// leaf, i.e. binary_op's division (ops.rs:498) against a [1] tensor.
template <class T>
int pool2d(bool is_max, const Tensor<T>& x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, std::vector<T>* out,
           std::vector<int64_t>* out_shape) {
  int st = pool_dims(x, kh, kw, sh, sw);
  if (st) return st;
  const int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
  int64_t oh, ow;
  std::vector<T> cols = unfold_2d(packed_data(x), N * C, 1, H, W, kh, kw, sh, sw, 0, 0, &oh, &ow);
  Tensor<T> ct = make_tensor(std::move(cols), {N * C * oh * ow, kh * kw});
  if (is_max) {
    std::vector<T> v;
    std::vector<int64_t> idx, os;
    st = max_argmax_axis(ct, 1, &v, &idx, &os);
    if (st) return st;
    *out = std::move(v);
  } else {
    Tensor<T> summed, q;
    st = sum_axis(ct, 1, false, &summed);
    if (st) return st;
    st = bin(DIV, summed, make_scalar<T>((T)(kh * kw)), &q);
    if (st) return st;
    *out = packed_data(q);
  }
  *out_shape = {N, C, oh, ow};
  return OK;
}

// The gradient MaxPool2d passes to its input: reshape's backward (the same
// elements), max_axis's backward (autodiff/core.rs:352-375: each row's gradient
// to its argmax, 0 elsewhere), unfold's backward fold_2d (core.rs:397-405),
// reshape back, and the accumulation `current + grad` (autodiff/traits.rs:
// 141-150) when `current` is given.  The intermediate gradients the reference
// also accumulates from 0 (0 + g) only turn -0 into +0, which fold_2d's sum
// from 0 does anyway.
template <class T>
int max_pool2d_backward(const Tensor<T>& x, const Tensor<T>& g, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                        const T* current, std::vector<T>* out) {
  int st = pool_dims(x, kh, kw, sh, sw);
  if (st) return st;
  const int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
  int64_t oh, ow;
  std::vector<T> cols = unfold_2d(packed_data(x), N * C, 1, H, W, kh, kw, sh, sw, 0, 0, &oh, &ow);
  const int64_t rows = N * C * oh * ow, patch = kh * kw;
  if (g.shape != std::vector<int64_t>{N, C, oh, ow}) { g_msg = "grad_out shape"; return ERR_SHAPE; }
  Tensor<T> ct = make_tensor(std::move(cols), {rows, patch});
  std::vector<T> v;
  std::vector<int64_t> winners, os;
  st = max_argmax_axis(ct, 1, &v, &winners, &os);
  if (st) return st;
  std::vector<T> grad = packed_data(g);
  std::vector<T> data((size_t)(rows * patch), T(0));
  for (int64_t r = 0; r < rows; ++r) data[(size_t)(r * patch + winners[r])] = grad[(size_t)r];
  std::vector<T> img = fold_2d(data, N * C, 1, H, W, kh, kw, sh, sw, 0, 0);
  if (current)
    for (size_t i = 0; i < img.size(); ++i) img[i] = Arith<T>::add(current[i], img[i]);
  *out = std::move(img);
  return OK;
}

}  // namespace

#define DISPATCH(dt, ...)                                          \
  switch (dt) {                                                    \
    case F32: { using T = float; __VA_ARGS__; } break;             \
    case F64: { using T = double; __VA_ARGS__; } break;            \
    case I32: { using T = int32_t; __VA_ARGS__; } break;           \
    case I64: { using T = int64_t; __VA_ARGS__; } break;           \
    default: g_msg = "bad dtype"; return ERR_DTYPE;                 \
  }

// One optimiser step for one parameter, element by element, as the
// reference's chain of tensor calls computes it (each call rounds once):
//   kind 0, SGD::step (optim/sgd.rs:29-37):     p = p - grad * lr
//   kind 1, RMSprop::step (optim/rmsprop.rs:30-46):
//     v = v * alpha + (grad & grad) * (1 - alpha)     [alpha in b2]
//     p = p - (grad * lr) / map(v, |x| x.sqrt() + eps)
//   kind 2, Adam::step (optim/adam.rs:119-144), step number t:
//     m = m * b1 + grad * (1 - b1);  v = v * b2 + (grad & grad) * (1 - b2)
//     m_hat = m / (1 - b1.powf(t));  v_hat = v / (1 - b2.powf(t))
//     p = p - (m_hat * lr) / map(v_hat, |x| x.sqrt() + eps)
// The scalars are the reference's: T::from_f64(..), T::one() - b and powf in T.
template <class T>
static void opt_step_t(int kind, T* p, const T* g, T* m, T* v, int64_t n, double lr_d, double b1_d,
                       double b2_d, double eps_d, int64_t t) {
  const T lr = (T)lr_d, b1 = (T)b1_d, b2 = (T)b2_d, eps = (T)eps_d, one = (T)1;
  const T omb1 = one - b1, omb2 = one - b2;
  const T tt = (T)t;
  const T bc1 = one - std::pow(b1, tt), bc2 = one - std::pow(b2, tt);
  for (int64_t i = 0; i < n; ++i) {
    if (kind == 0) {
      const T upd = g[i] * lr;
      p[i] = p[i] - upd;
    } else if (kind == 1) {
      const T gsq = g[i] * g[i];
      const T a = v[i] * b2, b = gsq * omb2;
      v[i] = a + b;
      const T vs = std::sqrt(v[i]) + eps;
      const T gl = g[i] * lr;
      const T upd = gl / vs;
      p[i] = p[i] - upd;
    } else {
      const T a = m[i] * b1, b = g[i] * omb1;
      m[i] = a + b;
      const T gsq = g[i] * g[i];
      const T c = v[i] * b2, d = gsq * omb2;
      v[i] = c + d;
      const T mh = m[i] / bc1, vh = v[i] / bc2;
      const T vs = std::sqrt(vh) + eps;
      const T ml = mh * lr;
      const T upd = ml / vs;
      p[i] = p[i] - upd;
    }
  }
}

extern "C" {

int orc_fill_uniform_at(int dtype, void* out, int64_t first, int64_t n, uint64_t seed, double lo,
                        double hi);

const char* orc_last_message(void) { return g_msg; }

void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int orc_get_max_threads(void) { return omp_get_num_procs(); }

int orc_storage_indices(const View* v, int64_t* out) {
  DISPATCH(v->dtype, {
    std::vector<int64_t> idx = storage_indices(from_view<T>(v));
    std::memcpy(out, idx.data(), idx.size() * sizeof(int64_t));
  });
  return OK;
}

int orc_broadcast_shape(const int64_t* a, int an, const int64_t* b, int bn,
                        int64_t* out, int32_t* on) {
  std::vector<int64_t> r;
  if (!broadcast_shape(std::vector<int64_t>(a, a + an), std::vector<int64_t>(b, b + bn), &r))
    return ERR_SHAPE;
  for (size_t i = 0; i < r.size(); ++i) out[i] = r[i];
  *on = (int32_t)r.size();
  return OK;
}

// binary_op; `out` receives the packed result (broadcast-shape numel elements).
int orc_binary(int op, const View* a, const View* b, void* out, int64_t* out_shape, int32_t* out_ndim) {
  if (a->dtype != b->dtype) return ERR_DTYPE;
  if (op == POW && (a->dtype == I32 || a->dtype == I64)) return ERR_DTYPE;
  DISPATCH(a->dtype, {
    Tensor<T> r;
    int st = binary_op<T>(op, from_view<T>(a), from_view<T>(b), &r);
    if (st) return st;
    write_out(r, out, out_shape, out_ndim);
  });
  return OK;
}

int orc_unary(int op, const View* x, double p0f, int64_t p0i, double p1f, int64_t p1i, void* out) {
  DISPATCH(x->dtype, {
    Tensor<T> r;
    int st = unary<T>(op, from_view<T>(x), scalar_of<T>(p0f, p0i), scalar_of<T>(p1f, p1i), &r);
    if (st) return st;
    write_out(r, out, nullptr, nullptr);
  });
  return OK;
}

// A fused program as the chain of separate reference calls it stands for.
int orc_program(int n_in, int op1, int op2, int epi, double p0f, int64_t p0i,
                double p1f, int64_t p1i, const View* in, void* out,
                int64_t* out_shape, int32_t* out_ndim) {
  DISPATCH(in[0].dtype, {
    Tensor<T> v = from_view<T>(&in[0]), t;
    int st;
    if (n_in >= 2) { if ((st = bin<T>(op1, v, from_view<T>(&in[1]), &t))) return st; v = std::move(t); v.data = v.owned.data(); }
    if (n_in >= 3) { if ((st = bin<T>(op2, v, from_view<T>(&in[2]), &t))) return st; v = std::move(t); v.data = v.owned.data(); }
    Tensor<T> r;
    if ((st = unary<T>(epi, v, scalar_of<T>(p0f, p0i), scalar_of<T>(p1f, p1i), &r))) return st;
    write_out(r, out, out_shape, out_ndim);
  });
  return OK;
}

int orc_sum(const View* x, void* out) {
  DISPATCH(x->dtype, {
    T s = sum_all(from_view<T>(x));
    std::memcpy(out, &s, sizeof(T));
  });
  return OK;
}

int orc_sum_axis(const View* x, int axis, int keepdim, void* out, int64_t* out_shape, int32_t* out_ndim) {
  DISPATCH(x->dtype, {
    Tensor<T> r;
    int st = sum_axis(from_view<T>(x), axis, keepdim != 0, &r);
    if (st) return st;
    write_out(r, out, out_shape, out_ndim);
  });
  return OK;
}

// mean as nn/layer_norm.rs:26 builds it: sum_axis_op(..) / T::from_usize(n).
int orc_mean_axis(const View* x, int axis, int keepdim, void* out, int64_t* out_shape, int32_t* out_ndim) {
  if (x->dtype != F32 && x->dtype != F64) return ERR_DTYPE;
  DISPATCH(x->dtype, {
    Tensor<T> r, m;
    Tensor<T> xt = from_view<T>(x);
    int st = sum_axis(xt, axis, keepdim != 0, &r);
    if (st) return st;
    if ((st = bin(DIV, r, make_scalar((T)xt.shape[axis]), &m))) return st;
    write_out(m, out, out_shape, out_ndim);
  });
  return OK;
}

int orc_max_axis(const View* x, int axis, void* out_vals, int64_t* out_idx) {
  DISPATCH(x->dtype, {
    std::vector<T> v;
    std::vector<int64_t> i, os;
    int st = max_argmax_axis(from_view<T>(x), axis, &v, &i, &os);
    if (st) return st;
    if (out_vals) std::memcpy(out_vals, v.data(), v.size() * sizeof(T));
    if (out_idx) std::memcpy(out_idx, i.data(), i.size() * sizeof(int64_t));
  });
  return OK;
}

int orc_reduce_broadcast_grad(const View* g, const int64_t* target, int tn, void* out,
                              int64_t* out_shape, int32_t* out_ndim) {
  DISPATCH(g->dtype, {
    Tensor<T> r;
    int st = reduce_broadcast_grad(from_view<T>(g), std::vector<int64_t>(target, target + tn), &r);
    if (st) return st;
    write_out(r, out, out_shape, out_ndim);
  });
  return OK;
}

int orc_softmax_lastdim(const View* x, void* out) {
  if (x->dtype != F32 && x->dtype != F64) return ERR_DTYPE;
  DISPATCH(x->dtype, {
    Tensor<T> r;
    int st = softmax_lastdim(from_view<T>(x), &r);
    if (st) return st;
    write_out(r, out, nullptr, nullptr);
  });
  return OK;
}

// Exact-order-free reference sums for error bounds: sum in long double with
// Neumaier compensation, and the sum of absolute values.
int orc_sum_f64(const View* x, double* sum, double* sum_abs) {
  DISPATCH(x->dtype, {
    Tensor<T> t = from_view<T>(x);
    std::vector<int64_t> idx = storage_indices(t);
    long double s = 0, c = 0, a = 0;
    for (int64_t i : idx) {
      long double v = (long double)t.data[i];
      long double u = s + v;
      if (fabsl(s) >= fabsl(v)) c += (s - u) + v; else c += (v - u) + s;
      s = u;
      a += fabsl(v);
    }
    *sum = (double)(s + c);
    *sum_abs = (double)a;
  });
  return OK;
}

// Seeded inputs.  Uniform: lo + (hi - lo) * u in f64, rounded once, with
// u = (splitmix64(seed, i) >> 40) * 2^-24.
int orc_fill_uniform(int dtype, void* out, int64_t n, uint64_t seed, double lo, double hi) {
  return orc_fill_uniform_at(dtype, out, 0, n, seed, lo, hi);
}

int orc_fill_uniform_at(int dtype, void* out, int64_t first, int64_t n, uint64_t seed, double lo,
                        double hi) {
  const double scale = 1.0 / 16777216.0;
  if (dtype == F32) {
    float* o = (float*)out;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      double u = (double)(splitmix64(seed, (uint64_t)(first + i)) >> 40) * scale;
      o[i] = (float)(lo + (hi - lo) * u);
    }
  } else if (dtype == F64) {
    double* o = (double*)out;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      double u = (double)(splitmix64(seed, (uint64_t)(first + i)) >> 40) * scale;
      o[i] = lo + (hi - lo) * u;
    }
  } else {
    return ERR_DTYPE;
  }
  return OK;
}

// Normal: Box-Muller over uniforms 2i and 2i+1, u1 in (0, 1], in f64 with
// glibc's log/cos/sqrt, rounded once.  orc_fill_normal_at writes elements
// first .. first + n - 1 of the stream (a second tensor drawn from the same
// seed continues where the first ended).
int orc_fill_normal_at(int dtype, void* out, int64_t first, int64_t n, uint64_t seed) {
  if (dtype != F32 && dtype != F64) return ERR_DTYPE;
  const double scale = 1.0 / 16777216.0;
  const double two_pi = 6.283185307179586;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t k = (uint64_t)(first + i);
    double u1 = (double)((splitmix64(seed, 2 * k) >> 40) + 1) * scale;
    double u2 = (double)(splitmix64(seed, 2 * k + 1) >> 40) * scale;
    double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
    if (dtype == F32) ((float*)out)[i] = (float)z;
    else ((double*)out)[i] = z;
  }
  return OK;
}

int orc_fill_normal(int dtype, void* out, int64_t n, uint64_t seed) {
  return orc_fill_normal_at(dtype, out, 0, n, seed);
}

// The sharded workload Y = A & B + c, sum(Y) with A, B f32 [rows, cols] and c
// f32 [cols] drawn as U(-1, 1) from seeds sa, sb, sc (element (i, j) of A is
// element i * cols + j of its stream), checked without holding any of it:
// every y is regenerated from the seeds.
//  * ref_fold: the reference's `sum` (base.rs:1024-1030): packed data folded
//    left to right in f32 from 0, each y = fl(fl(a * b) + c) as binary_op
//    computes `&(&a & &b) + &c` (ops.rs:240-300);
//  * exact / sum_abs: the sum and the sum of |y| in long double with Neumaier
//    compensation (per row, then over rows in order);
//  * row_bits (nullable, `rows` entries): per row, the sum of the int32 bit
//    patterns of its y as int64 -- a checksum that any single differing
//    element changes.
// The fold runs on its own thread beside the parallel pass.
int orc_fma_sum_stream(int64_t rows, int64_t cols, uint64_t sa, uint64_t sb, uint64_t sc, double* exact,
                       double* sum_abs, float* ref_fold, int64_t* row_bits) {
  if (rows < 0 || cols < 0) return ERR_ARG;
  const double scale = 1.0 / 16777216.0;
  auto uni = [scale](uint64_t seed, uint64_t i) -> float {
    double u = (double)(splitmix64(seed, i) >> 40) * scale;
    return (float)(-1.0 + 2.0 * u);
  };
  std::vector<float> c((size_t)cols);
  for (int64_t j = 0; j < cols; ++j) c[(size_t)j] = uni(sc, (uint64_t)j);
  auto y_at = [&](int64_t i, int64_t j) -> float {
    const uint64_t k = (uint64_t)(i * cols + j);
    volatile float t = uni(sa, k) * uni(sb, k);  // rounded to f32 before the add
    return t + c[(size_t)j];
  };
  float fold = 0.0f;
  std::thread folder([&]() {
    float acc = 0.0f;
    for (int64_t i = 0; i < rows; ++i)
      for (int64_t j = 0; j < cols; ++j) acc = acc + y_at(i, j);
    fold = acc;
  });
  std::vector<long double> rs((size_t)rows), rc((size_t)rows), ra((size_t)rows);
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t i = 0; i < rows; ++i) {
    long double s = 0, cmp = 0, a = 0;
    int64_t bits = 0;
    for (int64_t j = 0; j < cols; ++j) {
      const float y = y_at(i, j);
      int32_t b;
      std::memcpy(&b, &y, 4);
      bits += b;
      const long double v = (long double)y;
      const long double u = s + v;
      if (fabsl(s) >= fabsl(v)) cmp += (s - u) + v; else cmp += (v - u) + s;
      s = u;
      a += fabsl(v);
    }
    rs[(size_t)i] = s;
    rc[(size_t)i] = cmp;
    ra[(size_t)i] = a;
    if (row_bits) row_bits[i] = bits;
  }
  long double s = 0, cmp = 0, a = 0;
  for (int64_t i = 0; i < rows; ++i) {
    const long double v = rs[(size_t)i] + rc[(size_t)i];
    const long double u = s + v;
    if (fabsl(s) >= fabsl(v)) cmp += (s - u) + v; else cmp += (v - u) + s;
    s = u;
    a += ra[(size_t)i];
  }
  folder.join();
  *exact = (double)(s + cmp);
  *sum_abs = (double)a;
  *ref_fold = fold;
  return OK;
}

int orc_opt_step(int kind, int dtype, void* p, const void* g, void* m, void* v, int64_t n, double lr,
                 double b1, double b2, double eps, int64_t t) {
  if (kind < 0 || kind > 2 || n < 0) return ERR_ARG;
  if (dtype == F32)
    opt_step_t<float>(kind, (float*)p, (const float*)g, (float*)m, (float*)v, n, lr, b1, b2, eps, t);
  else if (dtype == F64)
    opt_step_t<double>(kind, (double*)p, (const double*)g, (double*)m, (double*)v, n, lr, b1, b2, eps, t);
  else
    return ERR_DTYPE;
  return OK;
}

// MaxPool2d / AvgPool2d forward (is_max 1 / 0); `out` receives the packed
// [N, C, OH, OW] result and out_shape its 4 dimensions.
int orc_pool2d(int is_max, const View* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, void* out,
               int64_t* out_shape) {
  if (x->dtype != F32 && x->dtype != F64) return ERR_DTYPE;
  DISPATCH(x->dtype, {
    std::vector<T> r;
    std::vector<int64_t> os;
    int st = pool2d(is_max != 0, from_view<T>(x), kh, kw, sh, sw, &r, &os);
    if (st) return st;
    std::memcpy(out, r.data(), r.size() * sizeof(T));
    for (int i = 0; i < 4; ++i) out_shape[i] = os[i];
  });
  return OK;
}

// MaxPool2d's gradient to x, packed [N, C, H, W]; `current` (packed, nullable)
// is the gradient it is accumulated onto.
int orc_max_pool2d_backward(const View* x, const View* g, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                            const void* current, void* out) {
  if (x->dtype != F32 && x->dtype != F64) return ERR_DTYPE;
  if (g->dtype != x->dtype) return ERR_DTYPE;
  DISPATCH(x->dtype, {
    std::vector<T> r;
    int st = max_pool2d_backward(from_view<T>(x), from_view<T>(g), kh, kw, sh, sw,
                                 static_cast<const T*>(current), &r);
    if (st) return st;
    std::memcpy(out, r.data(), r.size() * sizeof(T));
  });
  return OK;
}

// Tensor::matmul; out_shape receives the result's ndim dimensions.
int orc_matmul(const View* a, const View* b, void* out, int64_t* out_shape, int32_t* out_ndim) {
  if (a->dtype != b->dtype) { g_msg = "dtype mismatch"; return ERR_DTYPE; }
  DISPATCH(a->dtype, {
    std::vector<T> r;
    std::vector<int64_t> os;
    int st = matmul(from_view<T>(a), from_view<T>(b), &r, &os);
    if (st) return st;
    std::memcpy(out, r.data(), r.size() * sizeof(T));
    for (size_t d = 0; d < os.size(); ++d) out_shape[d] = os[d];
    *out_ndim = (int32_t)os.size();
  });
  return OK;
}

// Tensor::unfold_2d (conv.rs:360-418) of a [batch, channels, height, width]
// view; out_shape receives [batch * out_h * out_w, channels * kh * kw].
int orc_unfold_2d(const View* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, void* out,
                  int64_t* out_shape) {
  DISPATCH(x->dtype, {
    Tensor<T> t = from_view<T>(x);
    int st = unfold_dims(t, kh, kw, sh, sw, ph, pw);
    if (st) return st;
    int64_t oh, ow;
    std::vector<T> r = unfold_2d(packed_data(t), t.shape[0], t.shape[1], t.shape[2], t.shape[3], kh, kw, sh, sw,
                                 ph, pw, &oh, &ow);
    std::memcpy(out, r.data(), r.size() * sizeof(T));
    out_shape[0] = t.shape[0] * oh * ow;
    out_shape[1] = t.shape[1] * kh * kw;
  });
  return OK;
}

// Tensor::fold_2d (conv.rs:434-488) of a 2-D view into [batch, channels,
// height, width] = shape.
int orc_fold_2d(const View* cols, const int64_t* shape, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                int64_t pw, void* out) {
  DISPATCH(cols->dtype, {
    Tensor<T> t = from_view<T>(cols);
    if (sh <= 0 || sw <= 0) { g_msg = "!!!fold_2d(): stride must be positive!!!"; return ERR_ARG; }
    const int64_t B = shape[0], C = shape[1], H = shape[2], W = shape[3];
    bool ok = kh >= 0 && kw >= 0 && ph >= 0 && pw >= 0 && H + 2 * ph >= kh && W + 2 * pw >= kw;
    int64_t oh = 0, ow = 0;
    if (ok) {
      oh = (H + 2 * ph - kh) / sh + 1;
      ow = (W + 2 * pw - kw) / sw + 1;
      ok = t.shape == std::vector<int64_t>{B * oh * ow, C * kh * kw};
    }
    if (!ok) {
      g_msg_buf = "!!!fold_2d(): shape " + shape_text(t.shape) + " does not match an unfold of [" +
                  std::to_string(B) + ", " + std::to_string(C) + ", " + std::to_string(H) + ", " + std::to_string(W) +
                  "]!!!";
      g_msg = g_msg_buf.c_str();
      return ERR_SHAPE;
    }
    std::vector<T> r = fold_2d(packed_data(t), B, C, H, W, kh, kw, sh, sw, ph, pw);
    std::memcpy(out, r.data(), r.size() * sizeof(T));
  });
  return OK;
}

}  // extern "C"
