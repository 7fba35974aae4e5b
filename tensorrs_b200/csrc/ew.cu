// ew.cu -- K-EW: N-ary broadcast element-wise kernels over folded strided
// views (binary_op, ops.rs:240-300; Tensor::map, base.rs:1708-1716; the
// activation compositions of src/activation), with an optional fused sum of
// the results (sum, base.rs:1024-1030).
//
// Three kernels, chosen on the host from the folded view layout:
//   ew_vec_kernel    every operand runs along the innermost folded dimension
//                    with unit stride or is broadcast there (stride 0): 16-byte
//                    vector loads/stores, persistent grid over 16-byte chunks.
//   ew_tile_kernel   some input runs along another dimension (a transposed
//                    view such as B^T): 32x32 tiles of it are staged through
//                    shared memory so both its reads and the output's writes
//                    are coalesced.
//   ew_generic_kernel anything else (reversed, gapped, mixed layouts): one
//                    element per thread with the index decomposed on the fly.
// The sum epilogue accumulates every output value in f64 (wrapping integers
// for i32/i64), reduces per block in a fixed order and writes one partial per
// block; sum_finalize_kernel adds the partials in a fixed order and rounds once.
#include <cmath>
#include <cstring>
#include <mutex>

#include "kernels.cuh"

namespace trs {

// Set by a kernel that gave up waiting for its own bulk copies (bulk.cuh).
__device__ int g_trs_async_error;

int* async_error_word() {
  static std::mutex mu;
  static int* words[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_trs_async_error) == cudaSuccess)
      words[dev] = static_cast<int*>(p);
    else
      cudaGetLastError();
  }
  return words[dev];
}

int program_code(const trs_ew_program& p, bool fl) {
  const int n = p.n_in, o1 = p.op1, o2 = p.op2, e = p.epilogue;
  if (n == 1 && e == TRS_UN_NONE) return kPack;
  if (n == 2 && e == TRS_UN_NONE) {
    if (o1 == TRS_ADD) return kAdd;
    if (o1 == TRS_SUB) return kSub;
    if (o1 == TRS_MUL) return kMul;
    if (o1 == TRS_DIV) return kDiv;
  }
  if (n == 3 && o1 == TRS_MUL && o2 == TRS_ADD && e == TRS_UN_NONE) return kMulAdd;
  if (fl) {
    if (n == 3 && o1 == TRS_MUL && o2 == TRS_ADD && e == TRS_UN_RELU) return kMulAddRelu;
    if (n == 2 && o1 == TRS_MUL && e == TRS_UN_SIGMOID) return kMulSigmoid;
    if (n == 1 && e == TRS_UN_SIGMOID) return kSigmoid;
    if (n == 1 && e == TRS_UN_TANH) return kTanh;
    if (n == 1 && e == TRS_UN_RELU) return kRelu;
  }
  const bool simple = is_simple_program(p) || !fl;
  return (simple ? kRunSimple1 : kRunFull1) + (n - 1);
}

FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d ? d : 1;
  uint32_t s = 0;
  while (s < 32 && (1ull << s) < f.d) ++s;
  f.s = s;
  f.m = (uint32_t)((((1ull << 32) * ((1ull << s) - f.d)) / f.d) + 1);
  return f;
}

namespace {

template <class T>
__global__ void acc_to_value_kernel(const typename Arith<T>::Acc* acc, T* out) {
  *out = Arith<T>::from_acc(*acc);
}

// Seeded synthetic inputs (trs_fill_uniform / trs_fill_normal).
__device__ __forceinline__ uint64_t splitmix64(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <class T>
__global__ void __launch_bounds__(kThreads)
fill_kernel(const EwDev d, uint64_t seed, uint64_t first, double lo, double hi, int normal) {
  T* out = static_cast<T*>(d.out);
  const double scale = 1.0 / 16777216.0;
  const uint64_t step = (uint64_t)gridDim.x * kThreads;
  for (uint64_t g = (uint64_t)blockIdx.x * kThreads + threadIdx.x; g < (uint64_t)d.n; g += step) {
    int64_t o = d.off[0];
    uint64_t r = g;
    for (int dd = d.nd - 1; dd > 0; --dd) {
      const uint64_t q = r / (uint64_t)d.shape[dd];
      o += (int64_t)(r - q * (uint64_t)d.shape[dd]) * d.st[0][dd];
      r = q;
    }
    o += (int64_t)r * d.st[0][0];
    double v;
    const uint64_t gi = first + g;
    if (normal) {
      const double u1 = (double)((splitmix64(seed, 2 * gi) >> 40) + 1) * scale;
      const double u2 = (double)(splitmix64(seed, 2 * gi + 1) >> 40) * scale;
      v = __dmul_rn(sqrt(__dmul_rn(-2.0, log(u1))), cospi(__dmul_rn(2.0, u2)));
    } else {
      const double u = (double)(splitmix64(seed, gi) >> 40) * scale;
      v = __dadd_rn(lo, __dmul_rn(__dsub_rn(hi, lo), u));
    }
    out[o] = (T)v;
  }
}

// ---- host side -------------------------------------------------------------

const char* shape_msg(int op) {
  switch (op) {
    case TRS_ADD: return "!!!Add: incompatible shapes!!!";
    case TRS_SUB: return "!!!Sub: incompatible shapes!!!";
    case TRS_MUL: return "!!!MulElems: incompatible shapes!!!";
    case TRS_DIV: return "!!!DIV: incompatible shapes!!!";
    default: return "!!!Powf: incompatible shapes!!!";
  }
}

bool unop_float_only(int op) {
  switch (op) {
    case TRS_UN_NONE: case TRS_UN_NEG: case TRS_UN_ABS: case TRS_UN_ADD_SCALAR:
    case TRS_UN_SUB_SCALAR: case TRS_UN_RSUB_SCALAR: case TRS_UN_MUL_SCALAR:
    case TRS_UN_DIV_SCALAR:
      return false;
  }
  return true;
}

Error prepare(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
              EwPrepared* pr) {
  if (!in) return make_error(TRS_ERR_ARG, "null input array");
  if (prog.n_in < 1 || prog.n_in > 3) return make_error(TRS_ERR_ARG, "n_in must be 1..3");
  if (prog.n_in >= 2 && (prog.op1 < TRS_ADD || prog.op1 > TRS_POW))
    return make_error(TRS_ERR_ARG, "unknown binary op");
  if (prog.n_in >= 3 && (prog.op2 < TRS_ADD || prog.op2 > TRS_POW))
    return make_error(TRS_ERR_ARG, "unknown binary op");
  if (prog.epilogue < TRS_UN_NONE || prog.epilogue > TRS_UN_RPOW_SCALAR)
    return make_error(TRS_ERR_ARG, "unknown unary op");
  const char* names[3] = {"input 0", "input 1", "input 2"};
  for (int k = 0; k < prog.n_in; ++k) {
    Error e = validate_view(&in[k], names[k]);
    if (!e.ok()) return e;
    if (in[k].dtype != in[0].dtype) return make_error(TRS_ERR_DTYPE, "inputs have different dtypes");
  }
  const int dt = in[0].dtype;
  const bool fl = is_float(dt);
  if (!fl) {
    if ((prog.n_in >= 2 && prog.op1 == TRS_POW) || (prog.n_in >= 3 && prog.op2 == TRS_POW) ||
        unop_float_only(prog.epilogue))
      return make_error(TRS_ERR_DTYPE, "op needs a floating-point dtype (the reference's Float)");
  }
  // broadcast shape, in the order the chained reference calls take
  int64_t shape[kMaxDims];
  int nd = in[0].ndim;
  for (int i = 0; i < nd; ++i) shape[i] = in[0].shape[i];
  for (int k = 1; k < prog.n_in; ++k) {
    int64_t ns[kMaxDims];
    int nn = 0;
    if (!broadcast_shapes(shape, nd, in[k].shape, in[k].ndim, ns, &nn))
      return make_error(TRS_ERR_SHAPE, shape_msg(k == 1 ? prog.op1 : prog.op2));
    nd = nn;
    for (int i = 0; i < nd; ++i) shape[i] = ns[i];
  }
  int64_t strides[kMaxOperands][kMaxDims] = {};
  int64_t offs[kMaxOperands] = {};
  const void* bases[kMaxOperands] = {nullptr, nullptr, nullptr, nullptr};
  for (int k = 0; k < prog.n_in; ++k) {
    // broadcast_shape maps a (0, 1) pair to 1, after which broadcast_to fails
    // and the reference panics with this message (ops.rs:271-272)
    if (!broadcast_strides(&in[k], shape, nd, strides[k + 1]))
      return make_error(TRS_ERR_SHAPE, "broadcast_to failed (bug)");
    offs[k + 1] = in[k].offset;
    bases[k + 1] = in[k].data;
  }
  if (out) {
    Error e = validate_view(out, "output");
    if (!e.ok()) return e;
    if (out->dtype != dt) return make_error(TRS_ERR_DTYPE, "output dtype differs from the inputs");
    bool same = out->ndim == nd;
    for (int i = 0; same && i < nd; ++i) same = out->shape[i] == shape[i];
    if (!same) return make_error(TRS_ERR_SHAPE, "output shape is not the broadcast shape");
    for (int i = 0; i < nd; ++i) strides[0][i] = out->strides[i];
    offs[0] = out->offset;
    bases[0] = out->data;
  } else {
    // no output: fold as if writing a contiguous tensor
    int64_t s = 1;
    for (int i = nd - 1; i >= 0; --i) { strides[0][i] = s; s *= shape[i]; }
  }
  const int64_t n = numel_of(shape, nd);
  // an output may be an input only through the identical layout
  if (out && n > 0) {
    const int es = dtype_size(dt);
    auto range = [&](const trs_view* v, const int64_t* st, int64_t* lo, int64_t* hi) {
      int64_t a = v->offset, b = v->offset;
      for (int i = 0; i < nd; ++i) {
        const int64_t span = (shape[i] - 1) * st[i];
        if (span > 0) b += span; else a += span;
      }
      *lo = (int64_t)(uintptr_t)v->data + a * es;
      *hi = (int64_t)(uintptr_t)v->data + (b + 1) * es;
    };
    int64_t olo, ohi;
    range(out, strides[0], &olo, &ohi);
    for (int k = 0; k < prog.n_in; ++k) {
      int64_t ilo, ihi;
      range(&in[k], strides[k + 1], &ilo, &ihi);
      if (ilo < ohi && olo < ihi) {
        bool identical = in[k].data == out->data && in[k].offset == out->offset;
        for (int i = 0; identical && i < nd; ++i) identical = strides[k + 1][i] == strides[0][i];
        if (!identical)
          return make_error(TRS_ERR_ALIAS, "output overlaps an input through a different layout");
      }
    }
  }
  fold_dims(shape, nd, strides, offs, prog.n_in + 1, &pr->fold);
  pr->choice = choose_ew(pr->fold, bases, dtype_size(dt));
  pr->dtype = dt;
  return Error{};
}

}  // namespace

Error plan_elementwise(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                       EwFold* fold, EwChoice* choice) {
  EwPrepared pr;
  Error e = prepare(prog, in, out, &pr);
  if (!e.ok()) return e;
  *fold = pr.fold;
  *choice = pr.choice;
  return Error{};
}

Error run_elementwise(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                      const SumTarget* sum, cudaStream_t stream) {
  EwPrepared pr;
  Error e = prepare(prog, in, out, &pr);
  if (!e.ok()) return e;
  if (sum && sum->view) {
    Error ev = validate_view(sum->view, "sum output");
    if (!ev.ok()) return ev;
    if (sum->view->dtype != pr.dtype) return make_error(TRS_ERR_DTYPE, "sum output dtype differs from the inputs");
    if (numel_of(sum->view->shape, sum->view->ndim) != 1)
      return make_error(TRS_ERR_SHAPE, "sum output must hold one element");
  }
  switch (pr.dtype) {
    case TRS_F32: return ew_launch<float>(prog, in, out, sum, pr, stream);
    case TRS_F64: return ew_launch<double>(prog, in, out, sum, pr, stream);
    case TRS_I32: return ew_launch<int32_t>(prog, in, out, sum, pr, stream);
    case TRS_I64: return ew_launch<int64_t>(prog, in, out, sum, pr, stream);
  }
  return make_error(TRS_ERR_DTYPE, "unknown dtype");
}

Error run_acc_to_value(int dtype, const void* acc, const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (out->dtype != dtype) return make_error(TRS_ERR_DTYPE, "output dtype differs from the input");
  switch (dtype) {
    case TRS_F32:
      acc_to_value_kernel<float><<<1, 1, 0, stream>>>(static_cast<const double*>(acc),
                                                      static_cast<float*>(out->data) + out->offset);
      break;
    case TRS_F64:
      acc_to_value_kernel<double><<<1, 1, 0, stream>>>(static_cast<const double*>(acc),
                                                       static_cast<double*>(out->data) + out->offset);
      break;
    case TRS_I32:
      acc_to_value_kernel<int32_t><<<1, 1, 0, stream>>>(static_cast<const uint32_t*>(acc),
                                                        static_cast<int32_t*>(out->data) + out->offset);
      break;
    case TRS_I64:
      acc_to_value_kernel<int64_t><<<1, 1, 0, stream>>>(static_cast<const uint64_t*>(acc),
                                                        static_cast<int64_t*>(out->data) + out->offset);
      break;
    default:
      return make_error(TRS_ERR_DTYPE, "unknown dtype");
  }
  return check_launch("accumulator conversion kernel");
}

Error run_fill(trs_view* out, uint64_t seed, uint64_t first, double lo, double hi, bool normal,
               cudaStream_t stream) {
  Error e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (!is_float(out->dtype)) return make_error(TRS_ERR_DTYPE, "fill needs f32 or f64");
  EwDev d;
  std::memset(&d, 0, sizeof(d));
  d.nd = out->ndim > 0 ? out->ndim : 1;
  if (out->ndim == 0) { d.shape[0] = 1; d.st[0][0] = 0; }
  for (int i = 0; i < out->ndim; ++i) { d.shape[i] = out->shape[i]; d.st[0][i] = out->strides[i]; }
  d.off[0] = out->offset;
  d.out = out->data;
  d.n = numel_of(out->shape, out->ndim);
  if (d.n == 0) return Error{};
  const DeviceInfo& dev = current_device_info();
  uint64_t wb = ((uint64_t)d.n + kThreads - 1) / kThreads;
  uint64_t cap = (uint64_t)dev.sm_count * 8;
  const int blocks = (int)(wb < cap ? wb : cap);
  if (out->dtype == TRS_F32)
    fill_kernel<float><<<blocks, kThreads, 0, stream>>>(d, seed, first, lo, hi, normal ? 1 : 0);
  else
    fill_kernel<double><<<blocks, kThreads, 0, stream>>>(d, seed, first, lo, hi, normal ? 1 : 0);
  return check_launch("fill kernel");
}

}  // namespace trs
