// abi.cpp -- the extern "C" entry points declared in include/trs.h.
//
// Each entry point validates its views on the host, maps the reference's
// shape/axis rules onto a launch plan and calls the launchers in ew.cu,
// reduce.cu and softmax.cu.  Failures never abort: they return a status and
// leave the message (the reference's panic text where it has one) for
// trs_last_error().
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "../../include/trs.h"
#include "launch.h"
#include "reduce.h"
#include "runtime.h"
#include "softmax.h"

using namespace trs;

namespace {

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

cudaStream_t as_stream(trs_stream s) { return static_cast<cudaStream_t>(s); }

Error check_axis(const trs_view* x, int32_t axis) {
  if (axis < 0 || axis >= x->ndim) return make_error(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
  return Error{};
}

// Output strides of `out` laid over the kept dimensions of `x` for a
// single-axis reduction (keepdim keeps the axis as size 1 in `out`).
Error map_axis_output(const trs_view* x, int axis, bool keepdim, const trs_view* out,
                      int64_t* out_strides) {
  const int on = keepdim ? x->ndim : x->ndim - 1;
  bool ok = out->ndim == on;
  for (int i = 0, j = 0; ok && i < x->ndim; ++i) {
    if (i == axis) {
      if (keepdim) ok = out->shape[j++] == 1;
      continue;
    }
    ok = out->shape[j] == x->shape[i];
    out_strides[i] = out->strides[j];
    ++j;
  }
  if (!ok) return make_error(TRS_ERR_SHAPE, "output shape does not match the reduced shape");
  return Error{};
}

Error axis_reduce(int mode, const trs_view* x, int32_t axis, bool keepdim, const trs_view* out,
                  cudaStream_t stream) {
  Error e = validate_view(x, "input");
  if (!e.ok()) return e;
  e = check_axis(x, axis);
  if (!e.ok()) return e;
  if ((mode == kRedMax || mode == kRedArgmax) && x->shape[axis] == 0)
    return make_error(TRS_ERR_EMPTY_AXIS, "!!!Cannot reduce an empty axis!!!");
  if (mode == kRedMean && !is_float(x->dtype))
    return make_error(TRS_ERR_DTYPE, "mean needs f32 or f64");
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  const int want_dt = mode == kRedArgmax ? (int)TRS_I64 : x->dtype;
  if (out->dtype != want_dt)
    return make_error(TRS_ERR_DTYPE, mode == kRedArgmax ? "argmax output must be i64"
                                                         : "output dtype differs from the input");
  RedRequest q;
  q.mode = mode;
  q.reduce_mask = 1u << axis;
  q.in[0] = x;
  for (int i = 0; i < x->ndim; ++i) q.op_strides[0][i] = x->strides[i];
  q.out[0] = out;
  e = map_axis_output(x, axis, mode == kRedMax || mode == kRedArgmax ? false : keepdim, out,
                      q.out_strides[0]);
  if (!e.ok()) return e;
  return run_reduce(q, stream);
}

// Whether two views can reach a common byte of memory.
bool views_overlap(const trs_view* a, const trs_view* b) {
  if (numel_of(a->shape, a->ndim) == 0 || numel_of(b->shape, b->ndim) == 0) return false;
  auto range = [](const trs_view* v, int64_t* lo, int64_t* hi) {
    const int es = dtype_size(v->dtype);
    int64_t l = v->offset, h = v->offset;
    for (int i = 0; i < v->ndim; ++i) {
      const int64_t span = (v->shape[i] - 1) * v->strides[i];
      if (span > 0) h += span; else l += span;
    }
    *lo = (int64_t)(uintptr_t)v->data + l * es;
    *hi = (int64_t)(uintptr_t)v->data + (h + 1) * es;
  };
  int64_t alo, ahi, blo, bhi;
  range(a, &alo, &ahi);
  range(b, &blo, &bhi);
  return alo < bhi && blo < ahi;
}

// Shared planning of reduce_broadcast_grad (base.rs:1651-1686): which
// dimensions of g are summed, or TRS_NONE where the reference returns None.
Error plan_to_shape(const trs_view* g, const int64_t* target, int tn, const trs_view* out,
                    uint32_t* mask, int64_t* out_strides) {
  const int lead = g->ndim - tn;
  *mask = 0;
  for (int i = 0; i < lead; ++i) *mask |= 1u << i;
  for (int i = 0; i < tn; ++i) {
    const int64_t s = g->shape[lead + i], t = target[i];
    if (s == t) continue;
    if (t == 1) { *mask |= 1u << (lead + i); continue; }
    return make_error(TRS_NONE, "cannot reduce the gradient to the target shape");
  }
  bool ok = out->ndim == tn;
  for (int i = 0; ok && i < tn; ++i) ok = out->shape[i] == target[i];
  if (!ok) return make_error(TRS_ERR_SHAPE, "output shape differs from the target shape");
  for (int i = 0; i < tn; ++i) out_strides[lead + i] = out->strides[i];
  return Error{};
}

}  // namespace

extern "C" {

int32_t trs_abi_version(void) { return TRS_ABI_VERSION; }

size_t trs_last_error(char* buf, size_t len) {
  const std::string& m = last_error();
  if (buf && len > 0) {
    const size_t n = m.size() < len - 1 ? m.size() : len - 1;
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return m.size();
}

const char* trs_status_string(int32_t status) {
  switch (status) {
    case TRS_OK: return "ok";
    case TRS_NONE: return "none (the reference returns None)";
    case TRS_ERR_SHAPE: return "incompatible shapes";
    case TRS_ERR_AXIS: return "axis out of range";
    case TRS_ERR_EMPTY_AXIS: return "empty axis";
    case TRS_ERR_VIEW: return "invalid view";
    case TRS_ERR_DTYPE: return "unsupported or mismatched dtype";
    case TRS_ERR_ALIAS: return "output aliases an input";
    case TRS_ERR_OOM: return "out of device memory";
    case TRS_ERR_CUDA: return "CUDA error";
    case TRS_ERR_NCCL: return "NCCL error";
    case TRS_ERR_TIMEOUT: return "timeout";
    case TRS_ERR_ARG: return "invalid argument";
    case TRS_ERR_DIV_ZERO: return "integer division by zero";
    case TRS_ERR_UNAVAILABLE: return "unavailable";
  }
  return "unknown status";
}

uint64_t trs_launch_count(void) { return g_launch_count.load(); }

uint64_t trs_scratch_alloc_count(void) { return g_scratch_alloc_count.load(); }

trs_status trs_async_error(int32_t* code) {
  int* word = async_error_word();
  if (!word) return finish(make_error(TRS_ERR_CUDA, "the async-error word is not available"));
  cudaError_t e = cudaDeviceSynchronize();
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost);
  const int zero = 0;
  if (e == cudaSuccess) e = cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return finish(cuda_error(e, "reading the async-error word"));
  if (code) *code = v;
  if (v)
    return finish(make_error(TRS_ERR_TIMEOUT, std::string("a kernel gave up waiting: ") +
                                                  ((v & 1) ? "for its own bulk copies " : "") +
                                                  ((v & 2) ? "for a peer rank's partial sum" : "")));
  return TRS_OK;
}

trs_status trs_broadcast_shape(const int64_t* a, int32_t a_ndim, const int64_t* b, int32_t b_ndim,
                               int64_t* out_shape, int32_t* out_ndim) {
  if (!a || !b || !out_shape || !out_ndim || a_ndim < 0 || b_ndim < 0 || a_ndim > TRS_MAX_DIMS ||
      b_ndim > TRS_MAX_DIMS)
    return finish(make_error(TRS_ERR_ARG, "bad broadcast_shape arguments"));
  int n = 0;
  if (!broadcast_shapes(a, a_ndim, b, b_ndim, out_shape, &n))
    return finish(make_error(TRS_ERR_SHAPE, "!!!Add: incompatible shapes!!!"));
  *out_ndim = n;
  return TRS_OK;
}

trs_status trs_plan_elementwise(const trs_ew_program* prog, const trs_view* in, const trs_view* out,
                                int32_t* variant, int32_t* folded_ndim, int64_t* folded_shape,
                                int64_t* strides_out, int32_t* vector_width) {
  if (!prog) return finish(make_error(TRS_ERR_ARG, "null program"));
  EwFold f;
  EwChoice c;
  Error e = plan_elementwise(*prog, in, out, &f, &c);
  if (!e.ok()) return finish(e);
  if (variant) *variant = c.variant;
  if (vector_width) *vector_width = c.vec;
  if (folded_ndim) *folded_ndim = f.nd;
  if (folded_shape)
    for (int i = 0; i < f.nd; ++i) folded_shape[i] = f.shape[i];
  if (strides_out)
    for (int k = 0; k < kMaxOperands; ++k)
      for (int i = 0; i < kMaxDims; ++i) strides_out[k * kMaxDims + i] = i < f.nd && k < f.n_ops ? f.st[k][i] : 0;
  return TRS_OK;
}

trs_status trs_binary(int32_t op, const trs_view* a, const trs_view* b, trs_view* out, trs_stream stream) {
  if (!a || !b) return finish(make_error(TRS_ERR_ARG, "null input"));
  if (!out) return finish(make_error(TRS_ERR_ARG, "null output"));
  trs_ew_program p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = 2;
  p.op1 = op;
  p.epilogue = TRS_UN_NONE;
  trs_view in[2] = {*a, *b};
  return finish(run_elementwise(p, in, out, nullptr, as_stream(stream)));
}

trs_status trs_unary(int32_t op, const trs_view* x, const trs_scalar* params, trs_view* out,
                     trs_stream stream) {
  if (!x) return finish(make_error(TRS_ERR_ARG, "null input"));
  if (!out) return finish(make_error(TRS_ERR_ARG, "null output"));
  trs_ew_program p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = 1;
  p.epilogue = op;
  if (params) {
    p.p0 = params[0];
    p.p1 = params[1];
  }
  return finish(run_elementwise(p, x, out, nullptr, as_stream(stream)));
}

trs_status trs_elementwise(const trs_ew_program* prog, const trs_view* in, trs_view* out,
                           trs_stream stream) {
  if (!prog) return finish(make_error(TRS_ERR_ARG, "null program"));
  if (!out) return finish(make_error(TRS_ERR_ARG, "null output"));
  return finish(run_elementwise(*prog, in, out, nullptr, as_stream(stream)));
}

trs_status trs_elementwise_sum(const trs_ew_program* prog, const trs_view* in, trs_view* out,
                               trs_view* sum_out, trs_stream stream) {
  if (!prog) return finish(make_error(TRS_ERR_ARG, "null program"));
  if (!sum_out) return finish(make_error(TRS_ERR_ARG, "null sum output"));
  SumTarget t;
  t.view = sum_out;
  return finish(run_elementwise(*prog, in, out, &t, as_stream(stream)));
}

trs_status trs_elementwise_row_sums(const trs_ew_program* prog, const trs_view* in, trs_view* out,
                                    trs_view* row_sums, trs_view* total, trs_stream stream) {
  if (!prog || !in || !out) return finish(make_error(TRS_ERR_ARG, "null argument"));
  if (!row_sums && !total) return finish(make_error(TRS_ERR_ARG, "neither row sums nor a total requested"));
  cudaStream_t s = as_stream(stream);
  EwFold fold;
  EwChoice choice;
  Error e = plan_elementwise(*prog, in, out, &fold, &choice);  // inputs, output, shapes, aliasing
  if (!e.ok()) return finish(e);
  const int axis = out->ndim - 1;
  e = check_axis(out, axis);
  if (!e.ok()) return finish(e);
  int64_t rs_strides[TRS_MAX_DIMS];
  bool keepdim = false;
  if (row_sums) {
    e = validate_view(row_sums, "row sums");
    if (!e.ok()) return finish(e);
    if (row_sums->dtype != out->dtype) return finish(make_error(TRS_ERR_DTYPE, "row sums dtype differs"));
    keepdim = row_sums->ndim == out->ndim;
    e = map_axis_output(out, axis, keepdim, row_sums, rs_strides);
    if (!e.ok()) return finish(e);
  }
  if (total) {
    e = validate_view(total, "total");
    if (!e.ok()) return finish(e);
    if (total->dtype != out->dtype) return finish(make_error(TRS_ERR_DTYPE, "total dtype differs"));
    if (numel_of(total->shape, total->ndim) != 1)
      return finish(make_error(TRS_ERR_SHAPE, "total must hold one element"));
  }
  // the sums are fresh tensors in the reference: they may overlap nothing
  const trs_view* sums[2] = {row_sums, total};
  for (int i = 0; i < 2; ++i) {
    if (!sums[i]) continue;
    bool clash = views_overlap(sums[i], out) || (i == 1 && row_sums && views_overlap(total, row_sums));
    for (int k = 0; k < prog->n_in && !clash; ++k) clash = views_overlap(sums[i], &in[k]);
    if (clash) return finish(make_error(TRS_ERR_ALIAS, "a sum output overlaps another operand"));
  }
  bool taken = false;
  e = run_row_sums_fused(*prog, in, out, row_sums, total, s, &taken);
  if (taken || !e.ok()) return finish(e);
  // the three passes: Y, then its sums along the last axis, then its total
  e = run_elementwise(*prog, in, out, nullptr, s);
  if (!e.ok()) return finish(e);
  if (row_sums) {
    e = axis_reduce(kRedSum, out, axis, keepdim, row_sums, s);
    if (!e.ok()) return finish(e);
  }
  if (total) {
    trs_ew_program p;
    std::memset(&p, 0, sizeof(p));
    p.n_in = 1;
    p.epilogue = TRS_UN_NONE;
    SumTarget t;
    t.view = total;
    e = run_elementwise(p, out, nullptr, &t, s);
  }
  return finish(e);
}

trs_status trs_pack(const trs_view* x, trs_view* out, trs_stream stream) {
  return trs_unary(TRS_UN_NONE, x, nullptr, out, stream);
}

trs_status trs_sum(const trs_view* x, trs_view* out, trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  trs_ew_program p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = 1;
  p.epilogue = TRS_UN_NONE;
  SumTarget t;
  t.view = out;
  return finish(run_elementwise(p, x, nullptr, &t, as_stream(stream)));
}

trs_status trs_sum_axis(const trs_view* x, int32_t axis, int32_t keepdim, trs_view* out,
                        trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(axis_reduce(kRedSum, x, axis, keepdim != 0, out, as_stream(stream)));
}

trs_status trs_mean_axis(const trs_view* x, int32_t axis, int32_t keepdim, trs_view* out,
                         trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(axis_reduce(kRedMean, x, axis, keepdim != 0, out, as_stream(stream)));
}

trs_status trs_max_axis(const trs_view* x, int32_t axis, trs_view* out, trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(axis_reduce(kRedMax, x, axis, false, out, as_stream(stream)));
}

trs_status trs_argmax_axis(const trs_view* x, int32_t axis, trs_view* out, trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(axis_reduce(kRedArgmax, x, axis, false, out, as_stream(stream)));
}

trs_status trs_reduce_broadcast_grad(const trs_view* g, const int64_t* target, int32_t target_ndim,
                                     trs_view* out, trs_stream stream) {
  if (!g || !out || (target_ndim > 0 && !target))
    return finish(make_error(TRS_ERR_ARG, "null argument"));
  if (target_ndim < 0 || target_ndim > TRS_MAX_DIMS)
    return finish(make_error(TRS_ERR_ARG, "target rank out of range"));
  Error e = validate_view(g, "gradient");
  if (!e.ok()) return finish(e);
  e = validate_view(out, "output");
  if (!e.ok()) return finish(e);
  if (out->dtype != g->dtype) return finish(make_error(TRS_ERR_DTYPE, "output dtype differs"));
  cudaStream_t s = as_stream(stream);
  trs_view gv = *g;
  if (gv.ndim < target_ndim) {
    if (numel_of(gv.shape, gv.ndim) == 1) {
      // a scalar broadcasts to any shape (Tensor::from_num(item, target))
      bool ok = out->ndim == target_ndim;
      for (int i = 0; ok && i < target_ndim; ++i) ok = out->shape[i] == target[i];
      if (!ok) return finish(make_error(TRS_ERR_SHAPE, "output shape differs from the target shape"));
      trs_ew_program p;
      std::memset(&p, 0, sizeof(p));
      p.n_in = 1;
      trs_view one = gv;  // the single element, seen with the target's shape
      one.ndim = target_ndim;
      for (int i = 0; i < target_ndim; ++i) {
        one.shape[i] = target[i];
        one.strides[i] = 0;
      }
      return finish(run_elementwise(p, &one, out, nullptr, s));
    }
    // prepend size-1 dimensions until the ranks match
    const int add = target_ndim - gv.ndim;
    for (int i = gv.ndim - 1; i >= 0; --i) {
      gv.shape[i + add] = gv.shape[i];
      gv.strides[i + add] = gv.strides[i];
    }
    for (int i = 0; i < add; ++i) { gv.shape[i] = 1; gv.strides[i] = 0; }
    gv.ndim = target_ndim;
  }
  RedRequest q;
  q.mode = kRedSum;
  q.in[0] = &gv;
  for (int i = 0; i < gv.ndim; ++i) q.op_strides[0][i] = gv.strides[i];
  q.out[0] = out;
  e = plan_to_shape(&gv, target, target_ndim, out, &q.reduce_mask, q.out_strides[0]);
  if (!e.ok()) return finish(e);
  if (q.reduce_mask == 0) {
    trs_ew_program p;
    std::memset(&p, 0, sizeof(p));
    p.n_in = 1;
    trs_view src = gv;
    src.ndim = target_ndim;
    const int lead = gv.ndim - target_ndim;
    for (int i = 0; i < target_ndim; ++i) {
      src.shape[i] = gv.shape[lead + i];
      src.strides[i] = gv.strides[lead + i];
    }
    return finish(run_elementwise(p, &src, out, nullptr, s));
  }
  return finish(run_reduce(q, s));
}

trs_status trs_sum_to_shape_fused(const trs_view* g, const trs_view* gate, const trs_view* mul,
                                  const int64_t* target, int32_t target_ndim, trs_view* out,
                                  trs_stream stream) {
  if (!g || !out || (target_ndim > 0 && !target))
    return finish(make_error(TRS_ERR_ARG, "null argument"));
  if (target_ndim < 0 || target_ndim > g->ndim)
    return finish(make_error(TRS_ERR_SHAPE, "target rank exceeds the gradient's rank"));
  Error e = validate_view(g, "gradient");
  if (!e.ok()) return finish(e);
  e = validate_view(out, "output");
  if (!e.ok()) return finish(e);
  if (out->dtype != g->dtype) return finish(make_error(TRS_ERR_DTYPE, "output dtype differs"));
  if (!is_float(g->dtype)) return finish(make_error(TRS_ERR_DTYPE, "fused sum-to-shape needs f32 or f64"));
  RedRequest q;
  q.mode = kRedSum3;
  q.in[0] = g;
  for (int i = 0; i < g->ndim; ++i) q.op_strides[0][i] = g->strides[i];
  const trs_view* aux[2] = {gate, mul};
  for (int k = 0; k < 2; ++k) {
    if (!aux[k]) continue;
    e = validate_view(aux[k], k == 0 ? "gate" : "mul");
    if (!e.ok()) return finish(e);
    if (aux[k]->dtype != g->dtype) return finish(make_error(TRS_ERR_DTYPE, "operand dtypes differ"));
    if (!broadcast_strides(aux[k], g->shape, g->ndim, q.op_strides[k + 1]))
      return finish(make_error(TRS_ERR_SHAPE, "!!!MulElems: incompatible shapes!!!"));
    q.in[k + 1] = aux[k];
  }
  q.out[0] = out;
  e = plan_to_shape(g, target, target_ndim, out, &q.reduce_mask, q.out_strides[0]);
  if (!e.ok()) return finish(e);
  return finish(run_reduce(q, as_stream(stream)));
}

trs_status trs_affine_relu_backward(const trs_view* g, const trs_view* x, const trs_view* scale,
                                    const trs_view* bias, trs_view* grad_scale, trs_view* grad_bias,
                                    trs_stream stream) {
  if (!g || !x || !scale || !bias) return finish(make_error(TRS_ERR_ARG, "null input"));
  if (!grad_scale && !grad_bias) return finish(make_error(TRS_ERR_ARG, "no output requested"));
  const trs_view* views[4] = {g, x, scale, bias};
  const char* names[4] = {"gradient", "x", "scale", "bias"};
  for (int k = 0; k < 4; ++k) {
    Error e = validate_view(views[k], names[k]);
    if (!e.ok()) return finish(e);
    if (views[k]->dtype != g->dtype) return finish(make_error(TRS_ERR_DTYPE, "operand dtypes differ"));
  }
  if (!is_float(g->dtype)) return finish(make_error(TRS_ERR_DTYPE, "needs f32 or f64"));
  bool same = x->ndim == g->ndim && scale->ndim == g->ndim && bias->ndim == g->ndim;
  for (int i = 0; same && i < g->ndim; ++i)
    same = x->shape[i] == g->shape[i] && bias->shape[i] == scale->shape[i];
  if (!same) return finish(make_error(TRS_ERR_SHAPE, "x must match the gradient and bias must match scale"));
  RedRequest q;
  q.mode = kRedAffineRelu;
  q.in[0] = g;
  q.in[1] = x;
  q.in[2] = scale;
  q.in[3] = bias;
  for (int i = 0; i < g->ndim; ++i) {
    q.op_strides[0][i] = g->strides[i];
    q.op_strides[1][i] = x->strides[i];
  }
  if (!broadcast_strides(scale, g->shape, g->ndim, q.op_strides[2]) ||
      !broadcast_strides(bias, g->shape, g->ndim, q.op_strides[3]))
    return finish(make_error(TRS_ERR_SHAPE, "!!!MulElems: incompatible shapes!!!"));
  trs_view* outs[2] = {grad_scale, grad_bias};
  uint32_t mask = 0;
  for (int m = 0; m < 2; ++m) {
    if (!outs[m]) continue;
    Error e = validate_view(outs[m], m == 0 ? "grad_scale" : "grad_bias");
    if (!e.ok()) return finish(e);
    if (outs[m]->dtype != g->dtype) return finish(make_error(TRS_ERR_DTYPE, "output dtype differs"));
    e = plan_to_shape(g, scale->shape, scale->ndim, outs[m], &mask, q.out_strides[m]);
    if (!e.ok()) return finish(e.status == TRS_NONE ? make_error(TRS_ERR_SHAPE, e.msg) : e);
    q.out[m] = outs[m];
  }
  q.reduce_mask = mask;
  // scale and bias must be constant along every reduced dimension
  for (int i = 0; i < g->ndim; ++i)
    if ((mask & (1u << i)) && (q.op_strides[2][i] != 0 || q.op_strides[3][i] != 0) && g->shape[i] != 1)
      return finish(make_error(TRS_ERR_SHAPE, "scale/bias must be broadcast along the reduced axes"));
  return finish(run_reduce(q, as_stream(stream)));
}

trs_status trs_softmax_lastdim(const trs_view* x, trs_view* out, trs_stream stream) {
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(run_softmax(x, out, as_stream(stream)));
}

trs_status trs_fill_uniform(trs_view* out, uint64_t seed, uint64_t first, double lo, double hi,
                            trs_stream stream) {
  if (!out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(run_fill(out, seed, first, lo, hi, false, as_stream(stream)));
}

trs_status trs_fill_normal(trs_view* out, uint64_t seed, uint64_t first, trs_stream stream) {
  if (!out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(run_fill(out, seed, first, 0.0, 1.0, true, as_stream(stream)));
}

trs_status trs_set_device(int32_t device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return finish(cuda_error(e, "cudaSetDevice"));
  return TRS_OK;
}

trs_status trs_malloc(void** ptr, size_t bytes) {
  if (!ptr) return finish(make_error(TRS_ERR_ARG, "null pointer"));
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return finish(make_error(e == cudaErrorMemoryAllocation ? TRS_ERR_OOM : TRS_ERR_CUDA,
                             std::string("cudaMalloc: ") + cudaGetErrorString(e)));
  }
  return TRS_OK;
}

trs_status trs_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return finish(cuda_error(e, "cudaFree"));
  return TRS_OK;
}

trs_status trs_memcpy_htod(void* dst, const void* src, size_t bytes, trs_stream stream) {
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream));
  if (e != cudaSuccess) return finish(cuda_error(e, "cudaMemcpyAsync (host to device)"));
  return TRS_OK;
}

trs_status trs_memcpy_dtoh(void* dst, const void* src, size_t bytes, trs_stream stream) {
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream));
  if (e != cudaSuccess) return finish(cuda_error(e, "cudaMemcpyAsync (device to host)"));
  return TRS_OK;
}

trs_status trs_stream_synchronize(trs_stream stream) {
  cudaError_t e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return finish(cuda_error(e, "cudaStreamSynchronize"));
  return TRS_OK;
}

}  // extern "C"
