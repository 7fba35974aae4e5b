// trs_tensor.hpp -- C++17 host-side mirror of tensorrs' `Tensor<T>` API
// (src/linalg/tensor/base.rs, src/linalg/tensor/ops.rs) over the C ABI of
// trs.h, with device-resident storage.
//
// Names, argument meaning and error behaviour follow the reference:
//   - views (slice, step_slice, permute, transpose, reshape, shallow_copy)
//     share storage and copy nothing (base.rs:324-554);
//   - every op returns a new tensor with fresh contiguous storage;
//   - where the reference panics, a trs::Panic carrying the reference's text
//     is thrown; where it returns Option, std::optional is returned.
// Element access that the reference hands out by reference (Index, get) is
// served by a download; closure `map` has named replacements (relu, sigmoid,
// tanh, ...) because a closure cannot run on the GPU.
//
// The header uses only the ABI (trs_malloc / trs_memcpy_* / trs_free for
// memory), the way a Rust `-sys` crate binding the same symbols would.
#pragma once

#include <cstdint>
#include <cstring>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "trs.h"

namespace trs {

// A panic of the reference, as an exception.
struct Panic : std::runtime_error {
  trs_status status;
  Panic(trs_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

inline std::string last_error_text() {
  char buf[1024];
  trs_last_error(buf, sizeof(buf));
  return buf;
}

// Turns a failing status into a Panic; returns true for TRS_OK, false for TRS_NONE.
inline bool check(trs_status s) {
  if (s == TRS_OK) return true;
  if (s == TRS_NONE) return false;
  throw Panic(s, last_error_text());
}

template <class T> struct DtypeOf;
template <> struct DtypeOf<float> { static constexpr int32_t value = TRS_F32; };
template <> struct DtypeOf<double> { static constexpr int32_t value = TRS_F64; };
template <> struct DtypeOf<int32_t> { static constexpr int32_t value = TRS_I32; };
template <> struct DtypeOf<int64_t> { static constexpr int32_t value = TRS_I64; };

// Device storage shared between views (the reference's Arc<Storage<T>>).
struct Storage {
  void* ptr = nullptr;
  int64_t len = 0;
  int64_t bytes = 0;
  Storage(int64_t n, int es) : len(n), bytes(n * es) {
    if (bytes > 0) check(trs_malloc(&ptr, (size_t)bytes));
  }
  ~Storage() {
    if (ptr) trs_free(ptr);
  }
  Storage(const Storage&) = delete;
  Storage& operator=(const Storage&) = delete;
};

inline int64_t product(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

// compute_strides (base.rs:37-45).
inline std::vector<int64_t> compute_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  int64_t step = 1;
  for (int i = (int)shape.size() - 1; i >= 0; --i) {
    s[i] = step;
    step *= shape[i];
  }
  return s;
}

template <class T>
class Tensor {
 public:
  // ---- construction (base.rs:183-219, 816) ----

  // Tensor::new: data in row-major order; panics when the sizes disagree.
  static Tensor new_(const std::vector<T>& data, std::vector<int64_t> shape) {
    if ((int64_t)data.size() != product(shape))
      throw Panic(TRS_ERR_SHAPE, "!!!Inconsistent data and dimensions combination for tensor!!!");
    Tensor t = empty(std::move(shape));
    if (!data.empty()) {
      check(trs_memcpy_htod(t.storage_->ptr, data.data(), data.size() * sizeof(T), nullptr));
      check(trs_stream_synchronize(nullptr));
    }
    return t;
  }

  // Tensor::scalar: shape [1], stride [0].
  static Tensor scalar(T v) {
    Tensor t = new_({v}, {1});
    t.strides_ = {0};
    return t;
  }

  // Tensor::from_num.
  static Tensor from_num(T v, std::vector<int64_t> shape) {
    return new_(std::vector<T>((size_t)product(shape), v), std::move(shape));
  }

  // A contiguous tensor with uninitialised device storage.
  static Tensor empty(std::vector<int64_t> shape) {
    Tensor t;
    t.storage_ = std::make_shared<Storage>(product(shape) > 0 ? product(shape) : 1, (int)sizeof(T));
    t.strides_ = compute_strides(shape);
    t.shape_ = std::move(shape);
    t.offset_ = 0;
    return t;
  }

  // ---- data access ----

  std::vector<int64_t> get_shape() const { return shape_; }
  const std::vector<int64_t>& strides() const { return strides_; }
  int64_t offset() const { return offset_; }
  int64_t numel() const { return product(shape_); }

  // get_data (base.rs:252-254): the elements packed in row-major order.
  std::vector<T> get_data() const {
    Tensor p = is_packed() ? *this : clone();
    std::vector<T> out((size_t)numel());
    if (!out.empty()) {
      check(trs_memcpy_dtoh(out.data(), static_cast<const T*>(p.storage_->ptr) + p.offset_,
                            out.size() * sizeof(T), nullptr));
      check(trs_stream_synchronize(nullptr));
    }
    return out;
  }

  // item (base.rs:233-236).
  T item() const {
    if (numel() != 1) throw Panic(TRS_ERR_SHAPE, "!!!item() requires numel == 1!!!");
    T v;
    check(trs_memcpy_dtoh(&v, static_cast<const T*>(storage_->ptr) + offset_, sizeof(T), nullptr));
    check(trs_stream_synchronize(nullptr));
    return v;
  }

  // get (base.rs:287-301): None for a wrong rank or an index out of range.
  std::optional<T> get(const std::vector<int64_t>& idx) const {
    if (idx.size() != shape_.size()) return std::nullopt;
    int64_t at = offset_;
    for (size_t i = 0; i < idx.size(); ++i) {
      if (idx[i] < 0 || idx[i] >= shape_[i]) return std::nullopt;
      at += strides_[i] * idx[i];
    }
    T v;
    check(trs_memcpy_dtoh(&v, static_cast<const T*>(storage_->ptr) + at, sizeof(T), nullptr));
    check(trs_stream_synchronize(nullptr));
    return v;
  }

  // ---- views (no copy) ----

  // slice (base.rs:324-346).
  std::optional<Tensor> slice(const std::vector<int64_t>& start, const std::vector<int64_t>& shape) const {
    if (start.size() != shape_.size() || shape.size() != shape_.size()) return std::nullopt;
    int64_t off = offset_;
    for (size_t i = 0; i < start.size(); ++i) {
      if (start[i] + shape[i] > shape_[i]) return std::nullopt;
      off += strides_[i] * start[i];
    }
    Tensor v = *this;
    v.shape_ = shape;
    v.offset_ = off;
    return v;
  }

  // step_slice (base.rs:369-398): negative steps walk backwards.
  std::optional<Tensor> step_slice(const std::vector<int64_t>& start, const std::vector<int64_t>& shape,
                                   const std::vector<int64_t>& steps) const {
    const size_t n = shape_.size();
    if (start.size() != n || shape.size() != n || steps.size() != n) return std::nullopt;
    int64_t off = offset_;
    std::vector<int64_t> ns;
    for (size_t i = 0; i < n; ++i) {
      const int64_t end = start[i] + steps[i] * (shape[i] - 1);
      if (start[i] < 0 || end < 0 || start[i] >= shape_[i] || end >= shape_[i]) return std::nullopt;
      off += strides_[i] * start[i];
      ns.push_back(strides_[i] * steps[i]);
    }
    Tensor v = *this;
    v.shape_ = shape;
    v.strides_ = ns;
    v.offset_ = off;
    return v;
  }

  // permute (base.rs:510-537): None unless `axes` is a permutation.
  std::optional<Tensor> permute(const std::vector<int64_t>& axes) const {
    if (axes.size() != shape_.size()) return std::nullopt;
    std::vector<bool> seen(axes.size(), false);
    for (int64_t a : axes) {
      if (a < 0 || a >= (int64_t)axes.size() || seen[a]) return std::nullopt;
      seen[a] = true;
    }
    Tensor v = *this;
    for (size_t i = 0; i < axes.size(); ++i) {
      v.shape_[i] = shape_[axes[i]];
      v.strides_[i] = strides_[axes[i]];
    }
    return v;
  }

  // transpose (base.rs:550-554).
  Tensor transpose() const {
    if (shape_.size() != 2)
      throw Panic(TRS_ERR_SHAPE, "!!!transpose(): only 2D tensors supported!!!\n        \nTry to use permute");
    return *permute({1, 0});
  }

  // reshape (base.rs:475-487): contiguous tensors only.
  Tensor reshape(std::vector<int64_t> shape) const {
    if (product(shape) != numel()) throw Panic(TRS_ERR_SHAPE, "!!!Reshape size mismatch!!!");
    if (!is_contiguous()) throw Panic(TRS_ERR_VIEW, "!!!Non-contiguous reshape not supported!!!");
    Tensor v = *this;
    v.strides_ = compute_strides(shape);
    v.shape_ = std::move(shape);
    return v;
  }

  // shallow_copy (base.rs:450-457).
  Tensor shallow_copy() const { return *this; }

  // Clone (base.rs:1934-1945): a packed, contiguous copy.
  Tensor clone() const {
    Tensor out = empty(shape_);
    trs_view x = view(), o = out.view();
    check(trs_pack(&x, &o, nullptr));
    return out;
  }

  // is_contiguous (base.rs:616-631): size-1 dimensions are skipped.
  bool is_contiguous() const {
    int64_t expected = 1;
    for (int i = (int)shape_.size() - 1; i >= 0; --i) {
      if (shape_[i] == 1) continue;
      if (strides_[i] != expected) return false;
      expected *= shape_[i];
    }
    return true;
  }

  // can_inplace (base.rs:757-761).
  bool can_inplace() const {
    if (!is_contiguous() || storage_.use_count() != 1) return false;
    for (int64_t s : strides_)
      if (s == 0) return false;
    return true;
  }

  // ---- reductions ----

  // sum (base.rs:1024-1030).
  Tensor sum() const {
    Tensor out = empty({1});
    trs_view x = view(), o = out.view();
    check(trs_sum(&x, &o, nullptr));
    return out;
  }

  // sum_axis (base.rs:1051-1107).
  Tensor sum_axis(int64_t axis) const { return axis_op(axis, false, 0); }
  // sum_axis_keepdim (base.rs:1534-1594).
  Tensor sum_axis_keepdim(int64_t axis) const { return axis_op(axis, true, 0); }
  // sum_axis_op(..) / n, the mean of nn/layer_norm.rs:26.
  Tensor mean_axis(int64_t axis, bool keepdim) const { return axis_op(axis, keepdim, 1); }
  // max_axis (base.rs:1396-1436).
  Tensor max_axis(int64_t axis) const { return axis_op(axis, false, 2); }

  // argmax_axis (base.rs:1458-1505): usize indices as int64.
  std::vector<int64_t> argmax_axis(int64_t axis) const {
    if (axis < 0 || axis >= (int64_t)shape_.size()) throw Panic(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
    std::vector<int64_t> os = shape_;
    os.erase(os.begin() + axis);
    Tensor<int64_t> out = Tensor<int64_t>::empty(os);
    trs_view x = view(), o = out.view();
    check(trs_argmax_axis(&x, (int32_t)axis, &o, nullptr));
    return out.get_data();
  }

  // reduce_broadcast_grad (base.rs:1651-1686).
  std::optional<Tensor> reduce_broadcast_grad(const std::vector<int64_t>& target) const {
    Tensor out = empty(target);
    trs_view x = view(), o = out.view();
    if (!check(trs_reduce_broadcast_grad(&x, target.data(), (int32_t)target.size(), &o, nullptr)))
      return std::nullopt;
    return out;
  }
  // reduce_to_shape (base.rs:1617-1620).
  std::optional<Tensor> reduce_to_shape(const std::vector<int64_t>& target) const {
    return reduce_broadcast_grad(target);
  }

  // ---- element-wise (ops.rs:240-507) ----

  static Tensor binary(int32_t op, const Tensor& a, const Tensor& b) {
    std::vector<int64_t> shape(TRS_MAX_DIMS);
    int32_t nd = 0;
    if (trs_broadcast_shape(a.shape_.data(), (int32_t)a.shape_.size(), b.shape_.data(),
                            (int32_t)b.shape_.size(), shape.data(), &nd) != TRS_OK)
      throw Panic(TRS_ERR_SHAPE, shape_message(op));
    shape.resize(nd);
    Tensor out = empty(shape);
    trs_view x = a.view(), y = b.view(), o = out.view();
    trs_status s = trs_binary(op, &x, &y, &o, nullptr);
    if (s == TRS_ERR_SHAPE && last_error_text().find("broadcast_to") == std::string::npos)
      throw Panic(s, shape_message(op));
    check(s);
    return out;
  }

  Tensor unary(int32_t op, double p0 = 0, double p1 = 0) const {
    Tensor out = empty(shape_);
    trs_scalar params[2] = {{p0, (int64_t)p0}, {p1, (int64_t)p1}};
    trs_view x = view(), o = out.view();
    check(trs_unary(op, &x, params, &o, nullptr));
    return out;
  }

  friend Tensor operator+(const Tensor& a, const Tensor& b) { return binary(TRS_ADD, a, b); }
  friend Tensor operator-(const Tensor& a, const Tensor& b) { return binary(TRS_SUB, a, b); }
  // `&` is element-wise multiplication (ops.rs:428-452); `*` is matmul in the reference.
  friend Tensor operator&(const Tensor& a, const Tensor& b) { return binary(TRS_MUL, a, b); }
  friend Tensor operator/(const Tensor& a, const Tensor& b) { return binary(TRS_DIV, a, b); }
  // `^` is powf (ops.rs:491-495).
  friend Tensor operator^(const Tensor& a, const Tensor& b) { return binary(TRS_POW, a, b); }
  Tensor mul_elem(const Tensor& b) const { return binary(TRS_MUL, *this, b); }
  Tensor powf(const Tensor& b) const { return binary(TRS_POW, *this, b); }

  friend Tensor operator+(const Tensor& a, T s) { return a.unary(TRS_UN_ADD_SCALAR, (double)s); }
  friend Tensor operator-(const Tensor& a, T s) { return a.unary(TRS_UN_SUB_SCALAR, (double)s); }
  friend Tensor operator-(T s, const Tensor& a) { return a.unary(TRS_UN_RSUB_SCALAR, (double)s); }
  friend Tensor operator*(const Tensor& a, T s) { return a.unary(TRS_UN_MUL_SCALAR, (double)s); }
  friend Tensor operator/(const Tensor& a, T s) { return a.unary(TRS_UN_DIV_SCALAR, (double)s); }
  Tensor operator-() const { return unary(TRS_UN_NEG); }

  // AddAssign / SubAssign / BitAndAssign (ops.rs:334-351, 393-410, 454-471):
  // the result replaces self (the reference rebinds storage, shape, strides).
  Tensor& operator+=(const Tensor& b) { return *this = *this + b; }
  Tensor& operator-=(const Tensor& b) { return *this = *this - b; }
  Tensor& operator&=(const Tensor& b) { return *this = *this & b; }

  // ---- named maps for the activations (Tensor::map call sites) ----

  Tensor relu() const { return unary(TRS_UN_RELU); }                       // relu.rs:32-42
  Tensor sigmoid() const { return unary(TRS_UN_SIGMOID); }                 // autodiff/ops.rs:585-594
  Tensor tanh() const { return unary(TRS_UN_TANH); }                       // autodiff/ops.rs:547-548
  Tensor elu(T alpha) const { return unary(TRS_UN_ELU, (double)alpha); }   // elu.rs:43-64
  Tensor leaky_relu(T alpha) const { return unary(TRS_UN_LEAKY_RELU, (double)alpha); }
  Tensor selu(T alpha, T lambda) const { return unary(TRS_UN_SELU, (double)alpha, (double)lambda); }
  Tensor ln() const { return unary(TRS_UN_LN); }
  Tensor abs() const { return unary(TRS_UN_ABS); }
  Tensor clamp(T lo, T hi) const { return unary(TRS_UN_CLAMP, (double)lo, (double)hi); }

  // SoftMax::forward over the last axis (activation/softmax.rs:42-68).
  Tensor softmax() const {
    Tensor out = empty(shape_);
    trs_view x = view(), o = out.view();
    check(trs_softmax_lastdim(&x, &o, nullptr));
    return out;
  }

  // The trs_view this tensor is.
  trs_view view() const {
    trs_view v;
    std::memset(&v, 0, sizeof(v));
    v.data = storage_->ptr;
    v.storage_len = storage_->len;
    v.dtype = DtypeOf<T>::value;
    v.ndim = (int32_t)shape_.size();
    for (size_t i = 0; i < shape_.size(); ++i) {
      v.shape[i] = shape_[i];
      v.strides[i] = strides_[i];
    }
    v.offset = offset_;
    return v;
  }

 private:
  std::shared_ptr<Storage> storage_;
  std::vector<int64_t> shape_;
  std::vector<int64_t> strides_;
  int64_t offset_ = 0;

  template <class U> friend class Tensor;

  bool is_packed() const { return is_contiguous() && !has_zero_stride_over_one(); }
  bool has_zero_stride_over_one() const {
    for (size_t i = 0; i < shape_.size(); ++i)
      if (shape_[i] > 1 && strides_[i] == 0) return true;
    return false;
  }

  static std::string shape_message(int32_t op) {
    switch (op) {
      case TRS_ADD: return "!!!Add: incompatible shapes!!!";
      case TRS_SUB: return "!!!Sub: incompatible shapes!!!";
      case TRS_MUL: return "!!!MulElems: incompatible shapes!!!";
      case TRS_DIV: return "!!!DIV: incompatible shapes!!!";
      default: return "!!!Powf: incompatible shapes!!!";
    }
  }

  // mode 0: sum, 1: mean, 2: max
  Tensor axis_op(int64_t axis, bool keepdim, int mode) const {
    if (axis < 0 || axis >= (int64_t)shape_.size()) throw Panic(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
    std::vector<int64_t> os = shape_;
    if (keepdim) os[axis] = 1; else os.erase(os.begin() + axis);
    Tensor out = empty(os);
    trs_view x = view(), o = out.view();
    if (mode == 0) check(trs_sum_axis(&x, (int32_t)axis, keepdim ? 1 : 0, &o, nullptr));
    else if (mode == 1) check(trs_mean_axis(&x, (int32_t)axis, keepdim ? 1 : 0, &o, nullptr));
    else check(trs_max_axis(&x, (int32_t)axis, &o, nullptr));
    return out;
  }
};

}  // namespace trs
