// callers.cu -- callers of the element-wise / reduction path fused into one
// kernel each: LayerNorm::forward (nn/layer_norm.rs:20-33) and the optimiser
// steps SGD (optim/sgd.rs:29-37), RMSprop (optim/rmsprop.rs:30-46) and Adam
// (optim/adam.rs:119-144).
//
// The reference runs each as a chain of separate tensor calls (Adam: nine
// passes over every parameter, each allocating a fresh tensor).  Here:
//   optim_kernel          one pass: reads param, grad and the moment tensors,
//                         writes param and the moments in place; every step
//                         of the chain is an explicitly rounded IEEE
//                         operation, so the result is the chain's, bit for bit
//                         (the bias corrections beta^t are powf on the host,
//                         as the reference computes them).
//   rows of 4 .. 96 KiB  the bulk-copy row pipeline of softmax.cu (LayerNorm
//                         mode): rows staged in shared memory, three passes
//                         (sum, sum of squares, normalise), one read and one
//                         write per element.
//   layernorm_rows_kernel other rows: a warp or a CTA per row holds the row
//                         in registers: mean, (x - mean), the sum of squares, the
//                         normalisation and gamma / beta in one read and one
//                         write; sums in f64, rounded once.
//   layernorm_long_kernel rows longer than a CTA holds: three passes.
#include <cmath>
#include <cstring>

#include "../../include/trs.h"
#include "kernels.cuh"
#include "softmax.h"

namespace trs {
namespace {

// ---- optimiser steps -------------------------------------------------------

enum OptKind { kOptSgd = 0, kOptRms = 1, kOptAdam = 2 };

template <class T>
struct OptParams {
  T lr, b1, omb1, b2, omb2, bc1, bc2, eps;
};

template <class T>
__device__ __forceinline__ T sqrt_rn(T x) {
  if constexpr (sizeof(T) == 4) return __fsqrt_rn(x);
  else return __dsqrt_rn(x);
}

// One element of the step, in the reference's order of operations.
template <class T, int KIND>
__device__ __forceinline__ void opt_elem(T& p, T g, T& m, T& v, const OptParams<T>& q) {
  using A = Arith<T>;
  if constexpr (KIND == kOptSgd) {
    p = A::sub(p, A::mul(g, q.lr));                                 // p - grad * lr
  } else if constexpr (KIND == kOptRms) {
    v = A::add(A::mul(v, q.b2), A::mul(A::mul(g, g), q.omb2));      // v*alpha + (g&g)*(1-alpha)
    const T vs = A::add(sqrt_rn(v), q.eps);                         // map(|x| x.sqrt() + eps)
    p = A::sub(p, A::div(A::mul(g, q.lr), vs, nullptr));            // p - (g*lr) / vs
  } else {
    m = A::add(A::mul(m, q.b1), A::mul(g, q.omb1));                 // m*b1 + g*(1-b1)
    v = A::add(A::mul(v, q.b2), A::mul(A::mul(g, g), q.omb2));      // v*b2 + (g&g)*(1-b2)
    const T mh = A::div(m, q.bc1, nullptr);                          // m / (1 - b1^t)
    const T vh = A::div(v, q.bc2, nullptr);                          // v / (1 - b2^t)
    const T vs = A::add(sqrt_rn(vh), q.eps);
    p = A::sub(p, A::div(A::mul(mh, q.lr), vs, nullptr));           // p - (mh*lr) / vs
  }
}

template <class T, int V>
struct alignas(16) OVec {
  T v[V];
};

template <class T, int V>
__device__ __forceinline__ OVec<T, V> oload(const T* p) {
  OVec<T, V> r;
  const int4 x = __ldcs(reinterpret_cast<const int4*>(p));
  memcpy(&r, &x, 16);
  return r;
}

template <class T, int V>
__device__ __forceinline__ void ostore(T* p, const OVec<T, V>& r) {
  int4 x;
  memcpy(&x, &r, 16);
  __stcs(reinterpret_cast<int4*>(p), x);
}

constexpr int kOptThreads = 256;

// Grid-stride over 16-byte chunks (two per thread per iteration, all loads
// issued first), then the scalar tail.
template <class T, int KIND>
__global__ void __launch_bounds__(kOptThreads) optim_kernel(T* p, const T* g, T* m, T* v, int64_t n,
                                                            OptParams<T> q) {
  constexpr int V = 16 / (int)sizeof(T);
  const uint64_t chunks = (uint64_t)n / V;
  const uint64_t stride = (uint64_t)gridDim.x * kOptThreads;
  uint64_t c = (uint64_t)blockIdx.x * kOptThreads + threadIdx.x;
  for (; c + stride < chunks; c += 2 * stride) {
    OVec<T, V> P[2], G[2], M[2], W[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint64_t e = (c + u * stride) * V;
      P[u] = oload<T, V>(p + e);
      G[u] = oload<T, V>(g + e);
      if constexpr (KIND == kOptAdam) M[u] = oload<T, V>(m + e);
      if constexpr (KIND != kOptSgd) W[u] = oload<T, V>(v + e);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint64_t e = (c + u * stride) * V;
#pragma unroll
      for (int i = 0; i < V; ++i) opt_elem<T, KIND>(P[u].v[i], G[u].v[i], M[u].v[i], W[u].v[i], q);
      ostore<T, V>(p + e, P[u]);
      if constexpr (KIND == kOptAdam) ostore<T, V>(m + e, M[u]);
      if constexpr (KIND != kOptSgd) ostore<T, V>(v + e, W[u]);
    }
  }
  for (; c < chunks; c += stride) {
    const uint64_t e = c * V;
    OVec<T, V> P = oload<T, V>(p + e), G = oload<T, V>(g + e), M, W;
    if constexpr (KIND == kOptAdam) M = oload<T, V>(m + e);
    if constexpr (KIND != kOptSgd) W = oload<T, V>(v + e);
#pragma unroll
    for (int i = 0; i < V; ++i) opt_elem<T, KIND>(P.v[i], G.v[i], M.v[i], W.v[i], q);
    ostore<T, V>(p + e, P);
    if constexpr (KIND == kOptAdam) ostore<T, V>(m + e, M);
    if constexpr (KIND != kOptSgd) ostore<T, V>(v + e, W);
  }
  // tail elements (n not a multiple of V)
  const uint64_t tail0 = chunks * V;
  for (uint64_t e = tail0 + (uint64_t)blockIdx.x * kOptThreads + threadIdx.x; e < (uint64_t)n; e += stride) {
    T P = p[e], M = KIND == kOptAdam ? m[e] : T(0), W = KIND != kOptSgd ? v[e] : T(0);
    opt_elem<T, KIND>(P, g[e], M, W, q);
    p[e] = P;
    if constexpr (KIND == kOptAdam) m[e] = M;
    if constexpr (KIND != kOptSgd) v[e] = W;
  }
}

// A view that covers its storage as one packed run starting at a 16-byte
// boundary.
bool packed(const trs_view* v) {
  int64_t step = 1;
  for (int i = v->ndim - 1; i >= 0; --i) {
    if (v->shape[i] != 1 && v->strides[i] != step) return false;
    step *= v->shape[i];
  }
  return true;
}

Error check_opt_view(const trs_view* v, const trs_view* ref, const char* what) {
  Error e = validate_view(v, what);
  if (!e.ok()) return e;
  if (v->dtype != ref->dtype) return make_error(TRS_ERR_DTYPE, std::string(what) + ": dtype differs from param");
  bool same = v->ndim == ref->ndim;
  for (int i = 0; same && i < v->ndim; ++i) same = v->shape[i] == ref->shape[i];
  if (!same) return make_error(TRS_ERR_SHAPE, std::string(what) + ": shape differs from param");
  if (!packed(v)) return make_error(TRS_ERR_VIEW, std::string(what) + ": optimiser steps need contiguous tensors");
  const int es = dtype_size(v->dtype);
  if (((uintptr_t)v->data + (uintptr_t)(v->offset * es)) % 16)
    return make_error(TRS_ERR_VIEW, std::string(what) + ": data must start on a 16-byte boundary");
  return Error{};
}

template <class T, int KIND>
Error launch_opt(const trs_view* p, const trs_view* g, const trs_view* m, const trs_view* v, const OptParams<T>& q,
                 cudaStream_t stream) {
  const int64_t n = numel_of(p->shape, p->ndim);
  if (n == 0) return Error{};
  auto at = [](const trs_view* w) -> T* { return w ? static_cast<T*>(w->data) + w->offset : nullptr; };
  auto k = optim_kernel<T, KIND>;
  const int per_sm = resident_blocks_smem((const void*)k, kOptThreads, 0);
  constexpr int V = 16 / sizeof(T);
  const uint64_t want = ((uint64_t)n / V + kOptThreads - 1) / kOptThreads + 1;
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)per_sm;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  k<<<grid, kOptThreads, 0, stream>>>(at(p), at(g), at(m), at(v), n, q);
  return check_launch("optimiser step kernel");
}

template <class T>
Error run_opt_typed(int kind, const trs_view* p, const trs_view* g, const trs_view* m, const trs_view* v,
                    double lr, double b1, double b2, double eps, int64_t t, cudaStream_t stream) {
  OptParams<T> q;
  std::memset(&q, 0, sizeof(q));
  // the reference's scalars, in its element type: T::from_f64(..), T::one() - b,
  // b.powf(T::from_usize(t))
  q.lr = (T)lr;
  q.eps = (T)eps;
  q.b1 = (T)b1;
  q.b2 = (T)b2;
  q.omb1 = (T)1 - q.b1;
  q.omb2 = (T)1 - q.b2;
  if (kind == kOptAdam) {
    if constexpr (sizeof(T) == 4) {
      q.bc1 = 1.0f - powf(q.b1, (float)t);
      q.bc2 = 1.0f - powf(q.b2, (float)t);
    } else {
      q.bc1 = 1.0 - std::pow(q.b1, (double)t);
      q.bc2 = 1.0 - std::pow(q.b2, (double)t);
    }
  }
  switch (kind) {
    case kOptSgd: return launch_opt<T, kOptSgd>(p, g, m, v, q, stream);
    case kOptRms: return launch_opt<T, kOptRms>(p, g, m, v, q, stream);
    default: return launch_opt<T, kOptAdam>(p, g, m, v, q, stream);
  }
}

Error run_opt(int kind, const trs_view* p, const trs_view* g, const trs_view* m, const trs_view* v, double lr,
              double b1, double b2, double eps, int64_t t, cudaStream_t stream) {
  if (!p || !g) return make_error(TRS_ERR_ARG, "null view");
  Error e = check_opt_view(p, p, "param");
  if (!e.ok()) return e;
  if (!is_float(p->dtype)) return make_error(TRS_ERR_DTYPE, "optimiser steps need f32 or f64 tensors");
  e = check_opt_view(g, p, "grad");
  if (!e.ok()) return e;
  if (kind == kOptAdam) {
    if (!m) return make_error(TRS_ERR_ARG, "null view");
    e = check_opt_view(m, p, "m");
    if (!e.ok()) return e;
    if (t < 1) return make_error(TRS_ERR_ARG, "the step number t starts at 1");
  }
  if (kind != kOptSgd) {
    if (!v) return make_error(TRS_ERR_ARG, "null view");
    e = check_opt_view(v, p, "v");
    if (!e.ok()) return e;
  }
  if (p->dtype == TRS_F32) return run_opt_typed<float>(kind, p, g, m, v, lr, b1, b2, eps, t, stream);
  return run_opt_typed<double>(kind, p, g, m, v, lr, b1, b2, eps, t, stream);
}

// ---- LayerNorm -------------------------------------------------------------

struct LnDev {
  const void* in;
  void* out;
  const void* gamma;
  const void* beta;
  int64_t in_off, out_off, g_off, b_off;
  int64_t g_st, b_st;        // strides of gamma / beta along the features
  int64_t C;                 // features (last axis)
  int64_t in_step, out_step; // strides along the last axis
  int64_t rows;
  int nouter;
  int64_t oshape[kMaxDims];
  int64_t ist[kMaxDims];
  int64_t ost[kMaxDims];
  double eps;
};

__device__ __forceinline__ void ln_row_bases(const LnDev& d, uint64_t row, int64_t* bi, int64_t* bo) {
  int64_t a = d.in_off, b = d.out_off;
  for (int q = d.nouter - 1; q >= 0; --q) {
    const uint64_t nq = q > 0 ? row / (uint64_t)d.oshape[q] : 0;
    const int64_t c = (int64_t)(q > 0 ? row - nq * (uint64_t)d.oshape[q] : row);
    row = nq;
    a += c * d.ist[q];
    b += c * d.ost[q];
  }
  *bi = a;
  *bo = b;
}

template <class T, int V>
struct alignas(sizeof(T) * V) LVec {
  T v[V];
};

// Sum over a group (a warp, or the whole CTA), returned to every thread.
template <class Acc, int GROUP>
__device__ __forceinline__ Acc group_sum(Acc s, Acc* red, Acc* bcast) {
  for (int o = 16; o > 0; o >>= 1) s = s + __shfl_xor_sync(0xffffffffu, s, o);
  if constexpr (GROUP == 32) {
    return s;
  } else {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      Acc t = red[0];
      for (int w = 1; w < GROUP / 32; ++w) t = t + red[w];
      *bcast = t;
    }
    __syncthreads();
    return *bcast;
  }
}

template <class T, int V, int CH, int GROUP, int THREADS>
__global__ void __launch_bounds__(THREADS) layernorm_rows_kernel(const LnDev d) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int kGroups = THREADS / GROUP;
  __shared__ Acc red[32];
  __shared__ Acc bcast;
  const T* x = static_cast<const T*>(d.in);
  T* out = static_cast<T*>(d.out);
  const T* gm = static_cast<const T*>(d.gamma);
  const T* bt = static_cast<const T*>(d.beta);
  const int g_lane = threadIdx.x % GROUP, g_id = threadIdx.x / GROUP;
  const int64_t C = d.C;
  const bool unit = d.in_step == 1 && d.out_step == 1;
  const T fc = (T)C, eps = (T)d.eps;
  for (uint64_t row0 = (uint64_t)blockIdx.x * kGroups; row0 < (uint64_t)d.rows;
       row0 += (uint64_t)gridDim.x * kGroups) {
    const uint64_t row = row0 + g_id;
    const bool live = row < (uint64_t)d.rows;
    int64_t bi = 0, bo = 0;
    if (live) ln_row_bases(d, row, &bi, &bo);
    LVec<T, V> v[CH];
    Acc s = Acc(0);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
        if (V > 1 && unit) {
          v[c] = *reinterpret_cast<const LVec<T, V>*>(x + bi + e);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) v[c].v[i] = e + i < C ? x[bi + (e + i) * d.in_step] : T(0);
        }
#pragma unroll
        for (int i = 0; i < V; ++i)
          if (e + i < C) s = s + A::to_acc(v[c].v[i]);
      }
    }
    // mean = sum_axis_keepdim(x) / F
    const T mean = A::div(A::from_acc(group_sum<Acc, GROUP>(s, red, &bcast)), fc, nullptr);
    // sq = (x - mean) ^ 2, var = sum_axis_keepdim(sq) / F
    Acc s2 = Acc(0);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (e + i < C) {
            const T xm = A::sub(v[c].v[i], mean);
            v[c].v[i] = xm;
            s2 = s2 + A::to_acc(A::mul(xm, xm));
          }
        }
      }
    }
    const T var = A::div(A::from_acc(group_sum<Acc, GROUP>(s2, red, &bcast)), fc, nullptr);
    // denom = (var + eps) ^ 0.5; out = ((x - mean) / denom) & gamma + beta
    const T denom = sqrt_rn(A::add(var, eps));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (e + i < C) {
            const T gj = __ldg(gm + d.g_off + (e + i) * d.g_st);
            const T bj = __ldg(bt + d.b_off + (e + i) * d.b_st);
            v[c].v[i] = A::add(A::mul(A::div(v[c].v[i], denom, nullptr), gj), bj);
          }
        }
        if (V > 1 && unit) {
          *reinterpret_cast<LVec<T, V>*>(out + bo + e) = v[c];
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i)
            if (e + i < C) out[bo + (e + i) * d.out_step] = v[c].v[i];
        }
      }
    }
  }
}

// Rows longer than a CTA holds in registers: a CTA per row, three passes.
template <class T>
__global__ void __launch_bounds__(1024) layernorm_long_kernel(const LnDev d) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  __shared__ Acc red[32];
  __shared__ Acc bcast;
  const T* x = static_cast<const T*>(d.in);
  T* out = static_cast<T*>(d.out);
  const T* gm = static_cast<const T*>(d.gamma);
  const T* bt = static_cast<const T*>(d.beta);
  const T fc = (T)d.C, eps = (T)d.eps;
  for (uint64_t row = blockIdx.x; row < (uint64_t)d.rows; row += gridDim.x) {
    int64_t bi, bo;
    ln_row_bases(d, row, &bi, &bo);
    Acc s = Acc(0);
    for (int64_t e = threadIdx.x; e < d.C; e += 1024) s = s + A::to_acc(x[bi + e * d.in_step]);
    const T mean = A::div(A::from_acc(group_sum<Acc, 1024>(s, red, &bcast)), fc, nullptr);
    Acc s2 = Acc(0);
    for (int64_t e = threadIdx.x; e < d.C; e += 1024) {
      const T xm = A::sub(x[bi + e * d.in_step], mean);
      s2 = s2 + A::to_acc(A::mul(xm, xm));
    }
    const T var = A::div(A::from_acc(group_sum<Acc, 1024>(s2, red, &bcast)), fc, nullptr);
    const T denom = sqrt_rn(A::add(var, eps));
    for (int64_t e = threadIdx.x; e < d.C; e += 1024) {
      const T xm = A::sub(x[bi + e * d.in_step], mean);
      out[bo + e * d.out_step] =
          A::add(A::mul(A::div(xm, denom, nullptr), gm[d.g_off + e * d.g_st]), bt[d.b_off + e * d.b_st]);
    }
    __syncthreads();
  }
}

template <class K>
unsigned ln_grid(K kernel, int threads, uint64_t work) {
  const int per_sm = resident_blocks_smem((const void*)kernel, threads, 0);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)per_sm;
  const uint64_t g = work < cap ? work : cap;
  return (unsigned)(g < 1 ? 1 : g);
}

template <class T>
Error launch_ln(const LnDev& d, bool vec, cudaStream_t stream) {
  constexpr int VW = 16 / sizeof(T);
  const int64_t C = d.C;
  if (C <= 32 * 32) {  // a warp per row
    constexpr int TH = 256, G = 32;
    const uint64_t work = ((uint64_t)d.rows + TH / G - 1) / (TH / G);
    if (C <= 32 * 4) {
      auto k = layernorm_rows_kernel<T, 1, 4, G, TH>;
      k<<<ln_grid(k, TH, work), TH, 0, stream>>>(d);
    } else if (vec) {
      auto k = layernorm_rows_kernel<T, VW, 32 / VW, G, TH>;
      k<<<ln_grid(k, TH, work), TH, 0, stream>>>(d);
    } else {
      auto k = layernorm_rows_kernel<T, 1, 32, G, TH>;
      k<<<ln_grid(k, TH, work), TH, 0, stream>>>(d);
    }
    return check_launch("layer norm kernel");
  }
  if (C <= 512 * 32) {  // a CTA per row
    constexpr int TH = 512;
    if (vec) {
      if (C <= 512 * 8) {
        auto k = layernorm_rows_kernel<T, VW, 8 / VW, TH, TH>;
        k<<<ln_grid(k, TH, (uint64_t)d.rows), TH, 0, stream>>>(d);
      } else {
        auto k = layernorm_rows_kernel<T, VW, 32 / VW, TH, TH>;
        k<<<ln_grid(k, TH, (uint64_t)d.rows), TH, 0, stream>>>(d);
      }
    } else {
      auto k = layernorm_rows_kernel<T, 1, 32, TH, TH>;
      k<<<ln_grid(k, TH, (uint64_t)d.rows), TH, 0, stream>>>(d);
    }
    return check_launch("layer norm kernel");
  }
  auto k = layernorm_long_kernel<T>;
  k<<<ln_grid(k, 1024, (uint64_t)d.rows), 1024, 0, stream>>>(d);
  return check_launch("layer norm kernel (long rows)");
}

// gamma / beta hold F values along their last axis (every other dim 1).
Error features_view(const trs_view* v, int64_t F, int dt, const char* what, int64_t* st) {
  Error e = validate_view(v, what);
  if (!e.ok()) return e;
  if (v->dtype != dt) return make_error(TRS_ERR_DTYPE, std::string(what) + ": dtype differs from x");
  if (v->ndim < 1 || v->shape[v->ndim - 1] != F || numel_of(v->shape, v->ndim) != F)
    return make_error(TRS_ERR_SHAPE, std::string(what) + ": must hold the F features along its last axis");
  *st = v->strides[v->ndim - 1];
  return Error{};
}

Error run_layer_norm(const trs_view* x, const trs_view* gamma, const trs_view* beta, double eps,
                     const trs_view* out, cudaStream_t stream) {
  if (!x || !gamma || !beta || !out) return make_error(TRS_ERR_ARG, "null view");
  Error e = validate_view(x, "x");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (!is_float(x->dtype)) return make_error(TRS_ERR_DTYPE, "layer norm needs f32 or f64");
  if (out->dtype != x->dtype) return make_error(TRS_ERR_DTYPE, "output dtype differs from x");
  if (x->ndim < 1) return make_error(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
  bool same = out->ndim == x->ndim;
  for (int i = 0; same && i < x->ndim; ++i) same = out->shape[i] == x->shape[i];
  if (!same) return make_error(TRS_ERR_SHAPE, "output shape differs from x");
  const int last = x->ndim - 1;
  LnDev d;
  std::memset(&d, 0, sizeof(d));
  d.C = x->shape[last];
  e = features_view(gamma, d.C, x->dtype, "gamma", &d.g_st);
  if (!e.ok()) return e;
  e = features_view(beta, d.C, x->dtype, "beta", &d.b_st);
  if (!e.ok()) return e;
  if (numel_of(x->shape, x->ndim) == 0) return Error{};
  d.in = x->data;
  d.out = out->data;
  d.gamma = gamma->data;
  d.beta = beta->data;
  d.in_off = x->offset;
  d.out_off = out->offset;
  d.g_off = gamma->offset;
  d.b_off = beta->offset;
  d.in_step = x->strides[last];
  d.out_step = out->strides[last];
  d.eps = eps;
  d.rows = 1;
  int q = 0;
  for (int i = 0; i < last; ++i) {
    d.rows *= x->shape[i];
    if (x->shape[i] == 1) continue;
    d.oshape[q] = x->shape[i];
    d.ist[q] = x->strides[i];
    d.ost[q] = out->strides[i];
    ++q;
  }
  d.nouter = q;
  const int es = dtype_size(x->dtype);
  const int VW = 16 / es;
  bool vec = d.in_step == 1 && d.out_step == 1 && d.C % VW == 0;
  if (((uintptr_t)x->data + (uintptr_t)(x->offset * es)) % 16) vec = false;
  if (((uintptr_t)out->data + (uintptr_t)(out->offset * es)) % 16) vec = false;
  for (int i = 0; i < q; ++i)
    if (d.ist[i] % VW || d.ost[i] % VW) vec = false;
  // rows of 4 KiB and more: the bulk-copy row pipeline
  SmDev sd;
  std::memset(&sd, 0, sizeof(sd));
  sd.in = d.in;
  sd.out = d.out;
  sd.in_off = d.in_off;
  sd.out_off = d.out_off;
  sd.C = d.C;
  sd.in_step = d.in_step;
  sd.out_step = d.out_step;
  sd.rows = d.rows;
  sd.nouter = d.nouter;
  for (int i = 0; i < q; ++i) {
    sd.oshape[i] = d.oshape[i];
    sd.ist[i] = d.ist[i];
    sd.ost[i] = d.ost[i];
  }
  sd.gamma = d.gamma;
  sd.beta = d.beta;
  sd.g_off = d.g_off;
  sd.b_off = d.b_off;
  sd.g_st = d.g_st;
  sd.b_st = d.b_st;
  sd.ln_eps = d.eps;
  e = run_layer_norm_stream(sd, x->dtype, stream);
  if (e.status != TRS_NONE) return e;
  if (x->dtype == TRS_F32) return launch_ln<float>(d, vec, stream);
  return launch_ln<double>(d, vec, stream);
}

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

cudaStream_t as_stream(trs_stream s) { return static_cast<cudaStream_t>(s); }

}  // namespace
}  // namespace trs

using namespace trs;

extern "C" {

trs_status trs_layer_norm_lastdim(const trs_view* x, const trs_view* gamma, const trs_view* beta, double eps,
                                  trs_view* out, trs_stream stream) {
  return finish(run_layer_norm(x, gamma, beta, eps, out, as_stream(stream)));
}

trs_status trs_sgd_step(trs_view* param, const trs_view* grad, double lr, trs_stream stream) {
  return finish(run_opt(kOptSgd, param, grad, nullptr, nullptr, lr, 0.0, 0.0, 0.0, 0, as_stream(stream)));
}

trs_status trs_rmsprop_step(trs_view* param, const trs_view* grad, trs_view* v, double lr, double alpha, double eps,
                            trs_stream stream) {
  return finish(run_opt(kOptRms, param, grad, nullptr, v, lr, 0.0, alpha, eps, 0, as_stream(stream)));
}

trs_status trs_adam_step(trs_view* param, const trs_view* grad, trs_view* m, trs_view* v, double lr, double beta1,
                         double beta2, double eps, int64_t t, trs_stream stream) {
  return finish(run_opt(kOptAdam, param, grad, m, v, lr, beta1, beta2, eps, t, as_stream(stream)));
}

}  // extern "C"
