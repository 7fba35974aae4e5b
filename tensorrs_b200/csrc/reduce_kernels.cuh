// reduce_kernels.cuh -- reduction kernel templates and their per-dtype
// launcher (instantiated in reduce_f32.cu, reduce_f64.cu, reduce_i32.cu and
// reduce_i64.cu).
//
// The reference walks each output's axis serially (and leaves outputs < 8192
// on one thread).  Here the reduced and kept dimensions are folded separately
// on the host and one of three kernels is chosen:
//   red_row_kernel  the innermost reduced dimension is contiguous: one warp
//                   per output for short reductions, otherwise one CTA -- or a
//                   thread-block cluster of up to 8 CTAs whose partials meet
//                   in distributed shared memory -- per output; 16-byte loads.
//   red_col_kernel  a kept dimension is contiguous (e.g. sum over axis 0):
//                   lanes run along the kept dimension, the 8 warps of a CTA
//                   and the CTAs of a cluster split the reduced rows, and the
//                   partials meet in shared / distributed shared memory.
//   red_generic_kernel one thread per output, any layout.
// Float sums accumulate in f64 and round once; integer sums wrap.  Max and
// argmax follow the reference's strict `>` scan exactly (see MaxState).
// Every combine happens in a fixed order, so results are deterministic.
#pragma once

#include <cooperative_groups.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kernels.cuh"
#include "reduce.h"

namespace cg = cooperative_groups;

namespace trs {
namespace rk {

constexpr int kRowThreads = 256;
constexpr int kWarpModeThreads = 128;

template <class T, int V>
struct alignas(sizeof(T) * V) RVec {
  T v[V];
};

template <class T, int V>
__device__ __forceinline__ RVec<T, V> rload(const T* p) {
  RVec<T, V> r;
  if constexpr (sizeof(T) * V == 16) {
    int4 x = __ldg(reinterpret_cast<const int4*>(p));
    memcpy(&r, &x, 16);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = __ldg(p + i);
  }
  return r;
}

// A value below every element of T (-inf, or the integer minimum): the start
// of the strict `>` scans, which then need no "empty" test per element.  An
// element equal to it never wins, so a scan that saw only such elements (and
// NaNs) stays empty, and red_write resolves that as the reference does: the
// element at index 0 (which is then that lowest value, or a NaN).
template <class T>
__device__ __forceinline__ T red_lowest() {
  if constexpr (IsFloat<T>::value) return T(-INFINITY);
  else return (T)((typename Arith<T>::Acc)1 << (sizeof(T) * 8 - 1));
}

// max(a, b) ignoring a NaN operand (fmax for floats).
template <class T>
__device__ __forceinline__ T red_fmax(T a, T b) {
  if constexpr (sizeof(T) == 4 && IsFloat<T>::value) return fmaxf(a, b);
  else if constexpr (IsFloat<T>::value) return fmax(a, b);
  else return a > b ? a : b;
}

// Accumulator state of one reduction, for every mode.
template <class T>
struct RedAcc {
  using Acc = typename Arith<T>::Acc;
  Acc s0, s1;         // sums (s1: the second output of the affine mode)
  MaxState<T> m;
};

template <class T>
__device__ __forceinline__ RedAcc<T> red_init() {
  RedAcc<T> a;
  a.s0 = 0;
  a.s1 = 0;
  a.m.val = T(0);
  a.m.idx = -1;
  return a;
}

template <class T>
__device__ __forceinline__ RedAcc<T> red_combine(int mode, RedAcc<T> a, const RedAcc<T>& b) {
  if (mode == kRedMax || mode == kRedArgmax) {
    a.m = max_combine(a.m, b.m);
  } else {
    a.s0 = a.s0 + b.s0;
    a.s1 = a.s1 + b.s1;
  }
  return a;
}

// Only the fields the mode uses move (a constant mode drops the others).
template <class T>
__device__ __forceinline__ RedAcc<T> red_shfl_down(int mode, const RedAcc<T>& a, int o) {
  RedAcc<T> r = a;
  if (mode == kRedMax || mode == kRedArgmax) {
    r.m = shfl_down_max(a.m, o);
  } else {
    r.s0 = __shfl_down_sync(0xffffffffu, a.s0, o);
    if (mode == kRedAffineRelu) r.s1 = __shfl_down_sync(0xffffffffu, a.s1, o);
  }
  return r;
}

template <class T>
__device__ __forceinline__ RedAcc<T> red_warp(int mode, RedAcc<T> a) {
  for (int o = 16; o > 0; o >>= 1) a = red_combine(mode, a, red_shfl_down(mode, a, o));
  return a;
}

// The first n (a power of two, <= 32) lanes' states combined as a tree in a
// fixed order; the result is valid in lane 0.
template <class T>
__device__ __forceinline__ RedAcc<T> red_lanes(int mode, RedAcc<T> a, int n) {
  for (int o = n >> 1; o > 0; o >>= 1) a = red_combine(mode, a, red_shfl_down(mode, a, o));
  return a;
}

// Block reduction of RedAcc; valid in thread 0.
template <class T>
__device__ __forceinline__ RedAcc<T> red_block(int mode, RedAcc<T> a, RedAcc<T>* smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = red_warp(mode, a);
  __syncthreads();
  if (lane == 0) smem[warp] = a;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (warp == 0) {
    a = lane < nw ? smem[lane] : red_init<T>();
    a = red_warp(mode, a);
  }
  return a;
}

// One element folded into the accumulator.  `k` is the position along the
// reduced axis (used by max/argmax, which reduce one axis only).
template <class T>
__device__ __forceinline__ void red_push(int mode, RedAcc<T>& a, T v, T g2, T g3, int64_t k) {
  using A = Arith<T>;
  switch (mode) {
    case kRedSum:
    case kRedMean:
      a.s0 = a.s0 + A::to_acc(v);
      break;
    case kRedMax:
    case kRedArgmax:
      max_push(a.m, v, k);
      break;
  }
  (void)g2;
  (void)g3;
}

// The fused modes evaluate the product the separate reference calls would
// have materialised, with the same roundings.
template <class T>
__device__ __forceinline__ void red_push_fused(const RedDev& d, RedAcc<T>& a, T g, T x1, T x2,
                                               T x3, T s_c, T b_c) {
  using A = Arith<T>;
  const T one = T(1), zero = T(0);
  if (d.mode == kRedSum3) {
    T v = g;
    if (d.has_gate) v = A::mul(v, x1 > zero ? one : zero);  // g & map(gate > 0 ? 1 : 0)
    if (d.has_mul) v = A::mul(v, x2);                        // ... & mul
    a.s0 = a.s0 + A::to_acc(v);
  } else {  // kRedAffineRelu: x1 = x, with scale s_c and bias b_c of this channel
    const T z = A::add(A::mul(x1, s_c), b_c);
    const T gm = A::mul(g, z > zero ? one : zero);           // grad of z
    a.s0 = a.s0 + A::to_acc(A::mul(gm, x1));                 // scale grad: (g & m) & x
    a.s1 = a.s1 + A::to_acc(gm);                             // bias grad:   g & m
  }
  (void)x3;
}

// Offsets of output number `o` for every operand and output.
__device__ __forceinline__ void kept_offsets(const RedDev& d, uint64_t o, int64_t* in_off,
                                             int64_t* out_off) {
#pragma unroll
  for (int k = 0; k < kRedOperands; ++k) in_off[k] = d.off[k];
  out_off[0] = d.out_off[0];
  out_off[1] = d.out_off[1];
  for (int q = d.nk - 1; q >= 0; --q) {
    const uint64_t nq = q > 0 ? o / (uint64_t)d.kshape[q] : 0;
    const int64_t c = (int64_t)(q > 0 ? o - nq * (uint64_t)d.kshape[q] : o);
    o = nq;
#pragma unroll
    for (int k = 0; k < kRedOperands; ++k) in_off[k] += c * d.kst[k][q];
    out_off[0] += c * d.kout[0][q];
    out_off[1] += c * d.kout[1][q];
  }
}

// Offsets of reduced index r (row-major over the reduced dimensions).
__device__ __forceinline__ void red_offsets(const RedDev& d, uint64_t r, int64_t* off) {
#pragma unroll
  for (int k = 0; k < kRedOperands; ++k) off[k] = 0;
  for (int q = d.nr - 1; q >= 0; --q) {
    const uint64_t nq = q > 0 ? r / (uint64_t)d.rshape[q] : 0;
    const int64_t c = (int64_t)(q > 0 ? r - nq * (uint64_t)d.rshape[q] : r);
    r = nq;
#pragma unroll
    for (int k = 0; k < kRedOperands; ++k) off[k] += c * d.rst[k][q];
  }
}

// Writes one output.  `first` is the output's element at reduced index 0,
// which the max modes need (callers read it ahead, off the critical path).
template <class T>
__device__ __forceinline__ void red_write_first(const RedDev& d, const RedAcc<T>& a, const int64_t* out_off,
                                                T first) {
  using A = Arith<T>;
  if (d.raw) {
    if (d.mode == kRedMax || d.mode == kRedArgmax) {
      MaxRecord<T> r;
      r.val = a.m.val;
      r.idx = a.m.idx < 0 ? -1 : a.m.idx + d.idx_base;
      r.first = d.total > 0 ? first : T(0);
      static_cast<MaxRecord<T>*>(d.out[0])[out_off[0]] = r;
    } else {
      static_cast<typename A::Acc*>(d.out[0])[out_off[0]] = a.s0;
    }
    return;
  }
  switch (d.mode) {
    case kRedSum:
    case kRedSum3:
      static_cast<T*>(d.out[0])[out_off[0]] = A::from_acc(a.s0);
      break;
    case kRedMean: {
      const T s = A::from_acc(a.s0);
      static_cast<T*>(d.out[0])[out_off[0]] = A::div(s, (T)d.total, nullptr);
      break;
    }
    case kRedAffineRelu:
      if (d.out[0]) static_cast<T*>(d.out[0])[out_off[0]] = A::from_acc(a.s0);
      if (d.out[1]) static_cast<T*>(d.out[1])[out_off[1]] = A::from_acc(a.s1);
      break;
    case kRedMax:
    case kRedArgmax: {
      // the reference keeps a NaN found at index 0 (base.rs:1404-1411)
      MaxState<T> m = a.m;
      if (is_nan_val(first) || m.idx < 0) { m.val = first; m.idx = 0; }
      if (d.mode == kRedMax)
        static_cast<T*>(d.out[0])[out_off[0]] = m.val;
      else
        static_cast<int64_t*>(d.out[0])[out_off[0]] = m.idx;
      break;
    }
  }
}

template <class T>
__device__ __forceinline__ void red_write(const RedDev& d, const RedAcc<T>& a, const int64_t* out_off,
                                          const T* x0, int64_t x_first) {
  const bool need = (d.mode == kRedMax || d.mode == kRedArgmax) && d.total > 0;
  red_write_first<T>(d, a, out_off, need ? x0[x_first] : T(0));
}

// --------------------------------------------------------------------------
// Row kernel.  Group = one warp (WARP) or one CTA of a cluster of CS CTAs.
// The reduced space of an output is [RO outer rows] x [L contiguous].
template <class T, int V, bool WARP>
__global__ void __launch_bounds__(WARP ? kWarpModeThreads : kRowThreads)
red_row_kernel(const RedDev d) {
  using A = Arith<T>;
  __shared__ RedAcc<T> smem[32];
  const T* x0 = static_cast<const T*>(d.in[0]);
  const T* x1 = static_cast<const T*>(d.in[1]);
  const T* x2 = static_cast<const T*>(d.in[2]);
  const T* x3 = static_cast<const T*>(d.in[3]);
  const bool fused = d.mode == kRedSum3 || d.mode == kRedAffineRelu;
  uint64_t o;
  uint32_t worker, n_workers;
  unsigned crank = 0, csize = 1;
  if constexpr (WARP) {
    o = (uint64_t)blockIdx.x * (kWarpModeThreads / 32) + (threadIdx.x >> 5);
    worker = threadIdx.x & 31;
    n_workers = 32;
  } else {
    cg::cluster_group cluster = cg::this_cluster();
    crank = cluster.block_rank();
    csize = cluster.num_blocks();
    o = blockIdx.x / csize;
    worker = crank * kRowThreads + threadIdx.x;
    n_workers = csize * kRowThreads;
  }
  const bool live = o < (uint64_t)d.n_out;
  int64_t koff[kRedOperands], ooff[2];
  kept_offsets(d, live ? o : 0, koff, ooff);
  RedAcc<T> acc = red_init<T>();
  T s_c = T(0), b_c = T(0);
  if (d.mode == kRedAffineRelu) {
    s_c = __ldg(x2 + koff[2]);
    b_c = __ldg(x3 + koff[3]);
  }
  if (live) {
    const uint64_t cpr = (uint64_t)(d.L / V);
    const uint64_t total = (uint64_t)d.RO * cpr;
    const int nr = d.nr;
    for (uint64_t idx = worker; idx < total; idx += n_workers) {
      const uint64_t ro = idx / cpr;
      const int64_t c = (int64_t)(idx - ro * cpr) * V;
      int64_t roff[kRedOperands];
#pragma unroll
      for (int k = 0; k < kRedOperands; ++k) roff[k] = 0;
      if (nr > 1) {
        uint64_t r = ro;
        for (int q = nr - 2; q >= 0; --q) {
          const uint64_t nq = q > 0 ? r / (uint64_t)d.rshape[q] : 0;
          const int64_t cc = (int64_t)(q > 0 ? r - nq * (uint64_t)d.rshape[q] : r);
          r = nq;
#pragma unroll
          for (int k = 0; k < kRedOperands; ++k) roff[k] += cc * d.rst[k][q];
        }
      }
      const RVec<T, V> g = rload<T, V>(x0 + koff[0] + roff[0] + c);
      if (!fused) {
#pragma unroll
        for (int i = 0; i < V; ++i) red_push<T>(d.mode, acc, g.v[i], T(0), T(0), c + i);
      } else {
        RVec<T, V> a1, a2;
        if (d.mode == kRedAffineRelu || d.has_gate) {
          if (d.inner_bcast[1]) { T s = __ldg(x1 + koff[1] + roff[1]);
#pragma unroll
            for (int i = 0; i < V; ++i) a1.v[i] = s; }
          else a1 = rload<T, V>(x1 + koff[1] + roff[1] + c);
        }
        if (d.mode == kRedSum3 && d.has_mul) {
          if (d.inner_bcast[2]) { T s = __ldg(x2 + koff[2] + roff[2]);
#pragma unroll
            for (int i = 0; i < V; ++i) a2.v[i] = s; }
          else a2 = rload<T, V>(x2 + koff[2] + roff[2] + c);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) red_push_fused<T>(d, acc, g.v[i], a1.v[i], a2.v[i], T(0), s_c, b_c);
      }
    }
  }
  if constexpr (WARP) {
    acc = red_warp(d.mode, acc);
    if (live && (threadIdx.x & 31) == 0) red_write<T>(d, acc, ooff, x0, koff[0]);
  } else {
    acc = red_block(d.mode, acc, smem);
    if (csize == 1) {
      if (threadIdx.x == 0 && live) red_write<T>(d, acc, ooff, x0, koff[0]);
      return;
    }
    // cluster: rank 0 combines the partials of ranks 0..csize-1 in order
    cg::cluster_group cluster = cg::this_cluster();
    if (threadIdx.x == 0) smem[0] = acc;
    cluster.sync();
    if (crank == 0 && threadIdx.x == 0) {
      RedAcc<T> tot = smem[0];
      for (unsigned r = 1; r < csize; ++r) {
        const RedAcc<T>* peer = cluster.map_shared_rank(&smem[0], r);
        tot = red_combine(d.mode, tot, *peer);
      }
      if (live) red_write<T>(d, tot, ooff, x0, koff[0]);
    }
    cluster.sync();
  }
}

// --------------------------------------------------------------------------
// Column kernel: lanes along the contiguous kept dimension w (32*V columns
// per CTA), warps and cluster ranks over the reduced rows.
template <class T, int V>
__global__ void __launch_bounds__(kRowThreads) red_col_kernel(const RedDev d) {
  using A = Arith<T>;
  __shared__ RedAcc<T> part[kRowThreads / 32][32 * V];
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank(), csize = cluster.num_blocks();
  const T* x0 = static_cast<const T*>(d.in[0]);
  const T* x1 = static_cast<const T*>(d.in[1]);
  const T* x2 = static_cast<const T*>(d.in[2]);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t cb = blockIdx.x / csize;         // column block (and outer kept index)
  const uint64_t col_blocks = (uint64_t)((d.W + 32 * V - 1) / (32 * V));
  const uint64_t outer = cb / col_blocks;
  const int64_t w0 = (int64_t)(cb - outer * col_blocks) * 32 * V + lane * V;
  // kept offsets of the outer kept dims (all kept dims except w)
  int64_t koff[kRedOperands], ooff[2];
  kept_offsets(d, outer, koff, ooff);
  RedAcc<T> acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = red_init<T>();
  const bool full = w0 + V <= d.W;
  const bool any = w0 < d.W;
  const uint64_t rows = (uint64_t)d.total;
  const bool fused = d.mode == kRedSum3;
  if (any) {
    for (uint64_t r = (uint64_t)crank * (kRowThreads / 32) + warp; r < rows;
         r += (uint64_t)csize * (kRowThreads / 32)) {
      int64_t roff[kRedOperands];
      red_offsets(d, r, roff);
      RVec<T, V> g, a1, a2;
      const int64_t b0 = koff[0] + roff[0] + w0 * d.wst[0];
      if (full && V > 1) {
        g = rload<T, V>(x0 + b0);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) g.v[i] = w0 + i < d.W ? __ldg(x0 + b0 + i * d.wst[0]) : T(0);
      }
      if (fused) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const bool in = w0 + i < d.W;
          a1.v[i] = (d.has_gate && in) ? __ldg(x1 + koff[1] + roff[1] + (w0 + i) * d.wst[1]) : T(0);
          a2.v[i] = (d.has_mul && in) ? __ldg(x2 + koff[2] + roff[2] + (w0 + i) * d.wst[2]) : T(0);
        }
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        if (w0 + i >= d.W) continue;
        if (fused)
          red_push_fused<T>(d, acc[i], g.v[i], a1.v[i], a2.v[i], T(0), T(0), T(0));
        else
          red_push<T>(d.mode, acc[i], g.v[i], T(0), T(0), (int64_t)r);
      }
    }
  }
  // warps -> shared memory, combined in warp order by warp 0
#pragma unroll
  for (int i = 0; i < V; ++i) part[warp][lane * V + i] = acc[i];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      RedAcc<T> t = part[0][lane * V + i];
      for (int w = 1; w < kRowThreads / 32; ++w) t = red_combine(d.mode, t, part[w][lane * V + i]);
      part[0][lane * V + i] = t;
    }
  }
  cluster.sync();
  if (crank == 0 && warp == 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      RedAcc<T> t = part[0][lane * V + i];
      for (unsigned r = 1; r < csize; ++r) {
        const RedAcc<T>* peer = cluster.map_shared_rank(&part[0][lane * V + i], r);
        t = red_combine(d.mode, t, *peer);
      }
      const int64_t w = w0 + i;
      if (w < d.W) {
        int64_t oo[2] = {ooff[0] + w * d.wout[0], ooff[1] + w * d.wout[1]};
        red_write<T>(d, t, oo, x0, koff[0] + w * d.wst[0]);
      }
    }
  }
  cluster.sync();
}

// --------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(kRowThreads) red_generic_kernel(const RedDev d) {
  const T* x0 = static_cast<const T*>(d.in[0]);
  const T* x1 = static_cast<const T*>(d.in[1]);
  const T* x2 = static_cast<const T*>(d.in[2]);
  const T* x3 = static_cast<const T*>(d.in[3]);
  const bool fused = d.mode == kRedSum3 || d.mode == kRedAffineRelu;
  for (uint64_t o = (uint64_t)blockIdx.x * kRowThreads + threadIdx.x; o < (uint64_t)d.n_out;
       o += (uint64_t)gridDim.x * kRowThreads) {
    int64_t koff[kRedOperands], ooff[2];
    kept_offsets(d, o, koff, ooff);
    RedAcc<T> acc = red_init<T>();
    T s_c = T(0), b_c = T(0);
    if (d.mode == kRedAffineRelu) {
      s_c = x2[koff[2]];
      b_c = x3[koff[3]];
    }
    for (uint64_t r = 0; r < (uint64_t)d.total; ++r) {
      int64_t roff[kRedOperands];
      red_offsets(d, r, roff);
      const T g = x0[koff[0] + roff[0]];
      if (!fused) {
        red_push<T>(d.mode, acc, g, T(0), T(0), (int64_t)r);
      } else {
        const T a1 = (d.mode == kRedAffineRelu || d.has_gate) ? x1[koff[1] + roff[1]] : T(0);
        const T a2 = (d.mode == kRedSum3 && d.has_mul) ? x2[koff[2] + roff[2]] : T(0);
        red_push_fused<T>(d, acc, g, a1, a2, T(0), s_c, b_c);
      }
    }
    red_write<T>(d, acc, ooff, x0, koff[0]);
  }
}

// ---- host ------------------------------------------------------------------

template <class K>
Error launch_cluster(K kernel, unsigned grid, unsigned threads, unsigned cluster,
                     cudaStream_t stream, const RedDev& d) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, d);
  if (e != cudaSuccess) return cuda_error(e, "cluster launch");
  return check_launch("reduction kernel");
}

// --------------------------------------------------------------------------
// red_stream_kernel: reductions whose innermost reduced dimension is
// contiguous, on the bulk-copy pipeline.  Output o reduces RO segments of L
// contiguous elements; every segment is cut into tiles of up to
// kRsTileBytes.  A work item is (output, part): with few outputs each one is
// split into P parts whose partials a second kernel combines in order.
// Warp 0 (lane 0) produces: per tile it waits for a free stage, arms the
// stage's `full` mbarrier and issues one cp.async.bulk per unit-stride
// operand.  Warps 1..8 consume: load the tile's per-segment scalars, wait,
// accumulate with the compile-time MODE, release the stage; at the end of an
// item they combine their states in a fixed order behind a named barrier (the
// producer takes no part in it) and write the output or the partial.
// A wait that runs out marks the CTA failed; the failed CTA keeps walking its
// schedule without waiting or computing, so every barrier is still met, then
// drains the copies it has in flight and reports through the error word.
constexpr int kRsConsumerWarps = 8;
constexpr int kRsThreads = 32 * (1 + kRsConsumerWarps);
constexpr int kRsTileBytes = 16384;
// Shared memory per CTA for the stages: 100 KiB (two CTAs per SM, up to 6
// stages of one input) in general; 64 KiB for max / argmax, whose consumers
// do more work per byte and gain more from a third CTA per SM (27 warps) than
// from deeper stages (measured on rows of 64 KiB: 0.83 -> 0.98 of the copy
// peak, where sum and the two-input gradients lose with it).
constexpr int kRsBudget = 100 * 1024;
constexpr int kRsBudgetMax = 64 * 1024;

__host__ __device__ constexpr int rs_stages(int nb, int mode) {
  const int budget = (mode == kRedMax || mode == kRedArgmax) ? kRsBudgetMax : kRsBudget;
  return budget / (nb * kRsTileBytes) > 8 ? 8 : (budget / (nb * kRsTileBytes) < 2 ? 2 : budget / (nb * kRsTileBytes));
}

__device__ __forceinline__ FastDiv fd3(const uint32_t* v) {
  FastDiv f;
  f.d = v[0];
  f.m = v[1];
  f.s = v[2];
  return f;
}

__device__ __forceinline__ void named_sync_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kRsConsumerWarps) : "memory");
}

// Kept-dimension offsets of output o (32-bit index arithmetic).
__device__ __forceinline__ void rs_kept(const RedDev& d, uint32_t o, int64_t* in_off, int64_t* out_off) {
#pragma unroll
  for (int k = 0; k < kRedOperands; ++k) in_off[k] = d.off[k];
  out_off[0] = d.out_off[0];
  out_off[1] = d.out_off[1];
  for (int q = d.nk - 1; q >= 0; --q) {
    uint32_t c = o;
    if (q > 0) {
      const FastDiv f = fd3(d.fk[q]);
      const uint32_t nq = fdiv(o, f);
      c = o - nq * f.d;
      o = nq;
    }
#pragma unroll
    for (int k = 0; k < kRedOperands; ++k) in_off[k] += (int64_t)c * d.kst[k][q];
    out_off[0] += (int64_t)c * d.kout[0][q];
    out_off[1] += (int64_t)c * d.kout[1][q];
  }
}

// Offsets of segment r over the reduced dimensions other than the innermost.
__device__ __forceinline__ void rs_seg(const RedDev& d, uint32_t r, int64_t* off) {
#pragma unroll
  for (int k = 0; k < kRedOperands; ++k) off[k] = 0;
  for (int q = d.nr - 2; q >= 0; --q) {
    uint32_t c = r;
    if (q > 0) {
      const FastDiv f = fd3(d.fr[q]);
      const uint32_t nq = fdiv(r, f);
      c = r - nq * f.d;
      r = nq;
    }
#pragma unroll
    for (int k = 0; k < kRedOperands; ++k) off[k] += (int64_t)c * d.rst[k][q];
  }
}

template <class T, int MODE, int NB>
__global__ void __launch_bounds__(kRsThreads) red_stream_kernel(const RedDev d) {
  // the partials' fold kernel, launched after this one, may be scheduled now
  pdl_launch_dependents();
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int TILE = kRsTileBytes / (int)sizeof(T);
  constexpr int S = rs_stages(NB, MODE);
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * NB * kRsTileBytes);
  uint64_t* empty = full + S;
  // per-warp states of an item, double-buffered by the item's parity (one
  // barrier per item: a buffer is rewritten two items later, after the next
  // barrier, which thread 0 reaches only once it has read this one)
  __shared__ RedAcc<T> wred[2][kRsConsumerWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n_items = (uint32_t)(d.n_out * d.P);
  const uint32_t P = (uint32_t)d.P, tpp = (uint32_t)d.tpp;
  const uint32_t tiles_out = (uint32_t)(d.RO * d.tps);
  const FastDiv ftps = fd3(d.f_tps);
  const T* x0 = static_cast<const T*>(d.in[0]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRsConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  uint32_t issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      uint32_t qn = 0;
      for (uint32_t it = blockIdx.x; it < n_items; it += gridDim.x) {
        const uint32_t o = it / P, part = it - o * P;
        int64_t koff[kRedOperands], ooff[2];
        rs_kept(d, o, koff, ooff);
        const uint32_t t0 = part * tpp;
        const uint32_t nt = part + 1 < P ? tpp : tiles_out - t0;
        for (uint32_t j = 0; j < nt; ++j, ++qn) {
          const int s = (int)(qn % S);
          if (!failed && qn >= (uint32_t)S && !mbar_wait(&empty[s], ((qn / S) - 1) & 1u)) failed = true;
          if (failed) continue;
          fence_proxy_async();
          const uint32_t u = t0 + j;
          const uint32_t r = fdiv(u, ftps);
          const int64_t col0 = (int64_t)(u - r * ftps.d) * TILE;
          const int64_t rem = d.L - col0;
          const uint32_t len = (uint32_t)(rem < TILE ? rem : TILE);
          int64_t roff[kRedOperands];
          rs_seg(d, r, roff);
          mbar_arrive_expect_tx(&full[s], len * (uint32_t)sizeof(T) * NB);
#pragma unroll
          for (int k = 0; k < kRedOperands; ++k) {
            const int slot = d.bulk_slot[k];
            if (slot >= 0)
              bulk_g2s(smem + (s * NB + slot) * kRsTileBytes,
                       static_cast<const T*>(d.in[k]) + koff[k] + roff[k] + col0, len * (uint32_t)sizeof(T),
                       &full[s]);
          }
          issued = qn + 1;
        }
      }
    }
  } else {
    const int ct = threadIdx.x - 32;
    uint32_t qn = 0, qi = 0;
    for (uint32_t it = blockIdx.x; it < n_items; it += gridDim.x, ++qi) {
      const uint32_t o = it / P, part = it - o * P;
      int64_t koff[kRedOperands], ooff[2];
      rs_kept(d, o, koff, ooff);
      const uint32_t t0 = part * tpp;
      const uint32_t nt = part + 1 < P ? tpp : tiles_out - t0;
      Acc acc0[V], acc1[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc0[i] = acc1[i] = Acc(0);
      MaxState<T> m;
      m.val = T(0);
      m.idx = -1;
      T s_c = T(0), b_c = T(0);
      if constexpr (MODE == kRedAffineRelu) {
        s_c = __ldg(static_cast<const T*>(d.in[2]) + koff[2]);
        b_c = __ldg(static_cast<const T*>(d.in[3]) + koff[3]);
      }
      // the element at index 0 for the max modes' rule, read ahead of the
      // item's end so the write does not wait on it
      T first_pref = T(0);
      if constexpr (MODE == kRedMax || MODE == kRedArgmax)
        if (ct == 0 && P == 1 && d.total > 0) first_pref = __ldg(x0 + koff[0]);
      for (uint32_t j = 0; j < nt; ++j, ++qn) {
        const int s = (int)(qn % S);
        const uint32_t u = t0 + j;
        const uint32_t r = fdiv(u, ftps);
        const int64_t col0 = (int64_t)(u - r * ftps.d) * TILE;
        const int64_t rem = d.L - col0;
        const uint32_t len = (uint32_t)(rem < TILE ? rem : TILE);
        // per-segment scalars of the fused modes (gate / mul constant along L)
        T sc1 = T(0), sc2 = T(0);
        if constexpr (MODE == kRedSum3) {
          int64_t roff[kRedOperands];
          rs_seg(d, r, roff);
          if (d.has_gate && d.bulk_slot[1] < 0) sc1 = __ldg(static_cast<const T*>(d.in[1]) + koff[1] + roff[1]);
          if (d.has_mul && d.bulk_slot[2] < 0) sc2 = __ldg(static_cast<const T*>(d.in[2]) + koff[2] + roff[2]);
        }
        if (!failed && !__all_sync(0xffffffffu, mbar_wait(&full[s], (qn / S) & 1u))) failed = true;
        if (!failed) {
          const unsigned char* stage = smem + s * NB * kRsTileBytes;
          const uint32_t chunks = len / V;
          // the first chunk of each thread rotates by three warps per tile
          // (leftover chunks of uneven tiles fall on a different warp each
          // time; chunks stay in increasing order within a thread)
          constexpr uint32_t kC = 32 * kRsConsumerWarps;
          const uint32_t c0 = ((uint32_t)ct + kC - (qn * 96u) % kC) % kC;
          if constexpr (MODE == kRedMax || MODE == kRedArgmax) {
            // Per chunk: its NaN-ignoring maximum, compared strictly with
            // the running best (so the earliest chunk holding the maximum
            // wins).  Once per tile the winning chunk is read again and its
            // first element equal to the best gives the index and the value
            // (a -0 before a +0 stays, as in the reference's scan).  Tiles
            // arrive in increasing order and fold into the item's state with
            // the same strict rule.
            T tb = red_lowest<T>();
            uint32_t tc = 0xffffffffu;
#pragma unroll 4
            for (uint32_t c = c0; c < chunks; c += kC) {
              const RVec<T, V> g = *reinterpret_cast<const RVec<T, V>*>(stage + c * 16);
              T cm = g.v[0];
#pragma unroll
              for (int i = 1; i < V; ++i) cm = red_fmax(cm, g.v[i]);
              const bool p = cm > tb;
              tb = p ? cm : tb;
              tc = p ? c : tc;
            }
            // the recovered value equals tb, so the strict test against the
            // running best comes first and most tiles skip the re-read
            if (tc != 0xffffffffu && (m.idx < 0 || tb > m.val)) {
              const RVec<T, V> g = *reinterpret_cast<const RVec<T, V>*>(stage + tc * 16);
              int first = V - 1;
              T val = g.v[V - 1];
#pragma unroll
              for (int i = V - 2; i >= 0; --i)
                if (g.v[i] == tb) {
                  first = i;
                  val = g.v[i];
                }
              m.val = val;
              m.idx = col0 + (int64_t)(tc * V + first);
            }
          }
#pragma unroll 4
          for (uint32_t c = c0; c < chunks && MODE != kRedMax && MODE != kRedArgmax; c += kC) {
            const RVec<T, V> g = *reinterpret_cast<const RVec<T, V>*>(stage + c * 16);
            if constexpr (MODE == kRedSum || MODE == kRedMean) {
#pragma unroll
              for (int i = 0; i < V; ++i) acc0[i] = acc0[i] + A::to_acc(g.v[i]);
            } else if constexpr (MODE == kRedMax || MODE == kRedArgmax) {
              // handled above
            } else if constexpr (MODE == kRedSum3) {
              RVec<T, V> a1, a2;
              const int s1 = d.bulk_slot[1], s2 = d.bulk_slot[2];
              if (d.has_gate && s1 >= 0) a1 = *reinterpret_cast<const RVec<T, V>*>(stage + s1 * kRsTileBytes + c * 16);
              if (d.has_mul && s2 >= 0) a2 = *reinterpret_cast<const RVec<T, V>*>(stage + s2 * kRsTileBytes + c * 16);
#pragma unroll
              for (int i = 0; i < V; ++i) {
                T v = g.v[i];
                if (d.has_gate) {
                  const T gt = s1 >= 0 ? a1.v[i] : sc1;
                  v = A::mul(v, gt > T(0) ? T(1) : T(0));
                }
                if (d.has_mul) v = A::mul(v, s2 >= 0 ? a2.v[i] : sc2);
                acc0[i] = acc0[i] + A::to_acc(v);
              }
            } else {  // kRedAffineRelu: slot 1 holds x
              const RVec<T, V> xv = *reinterpret_cast<const RVec<T, V>*>(stage + kRsTileBytes + c * 16);
#pragma unroll
              for (int i = 0; i < V; ++i) {
                const T z = A::add(A::mul(xv.v[i], s_c), b_c);
                const T gm = A::mul(g.v[i], z > T(0) ? T(1) : T(0));
                acc0[i] = acc0[i] + A::to_acc(A::mul(gm, xv.v[i]));
                acc1[i] = acc1[i] + A::to_acc(gm);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // combine the item across the consumer warps, in a fixed order
      RedAcc<T> a = red_init<T>();
#pragma unroll
      for (int i = 0; i < V; ++i) {
        a.s0 = a.s0 + acc0[i];
        a.s1 = a.s1 + acc1[i];
      }
      a.m = m;
      a = red_warp(MODE, a);
      RedAcc<T>* wb = wred[qi & 1u];
      if (lane == 0) wb[warp - 1] = a;
      named_sync_consumers();
      // the first consumer warp folds the warps' states as a lane tree
      if (warp == 1) {
        RedAcc<T> tot = lane < kRsConsumerWarps ? wb[lane] : red_init<T>();
        tot = red_lanes(MODE, tot, kRsConsumerWarps);
        if (ct == 0 && !failed) {
          if (P == 1)
            red_write_first<T>(d, tot, ooff, first_pref);
          else
            static_cast<RedAcc<T>*>(d.parts)[it] = tot;
        }
      }
    }
  }
  if (__syncthreads_or(failed)) {
    if (threadIdx.x == 0) {
      atomicOr(d.err, kAsyncWaitTimeout);
      const uint32_t start = issued > (uint32_t)S ? issued - S : 0;
      for (uint32_t k = start; k < issued; ++k) mbar_wait(&full[k % S], (k / S) & 1u);
    }
    __syncthreads();
  }
}

// Combines the P partials of every output in part order and writes it.
template <class T, int MODE>
__global__ void __launch_bounds__(256) red_parts_finalize(const RedDev d) {
  pdl_wait();  // the partials of the kernel before it
  const T* x0 = static_cast<const T*>(d.in[0]);
  const RedAcc<T>* parts = static_cast<const RedAcc<T>*>(d.parts);
  for (uint32_t o = blockIdx.x * 256 + threadIdx.x; o < (uint32_t)d.n_out; o += gridDim.x * 256) {
    // the parts in order, loaded eight at a time so their loads overlap
    const RedAcc<T>* po = parts + (uint64_t)o * d.P;
    RedAcc<T> tot = po[0];
    int64_t p = 1;
    for (; p + 8 <= d.P; p += 8) {
      RedAcc<T> v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = po[p + i];
#pragma unroll
      for (int i = 0; i < 8; ++i) tot = red_combine(MODE, tot, v[i]);
    }
    for (; p < d.P; ++p) tot = red_combine(MODE, tot, po[p]);
    int64_t koff[kRedOperands], ooff[2];
    rs_kept(d, o, koff, ooff);
    red_write<T>(d, tot, ooff, x0, koff[0]);
  }
}

// --------------------------------------------------------------------------
// red_cstream_kernel: reductions whose innermost KEPT dimension W is
// contiguous (sum/max/argmax over axis 0 of a row-major matrix, and the
// un-broadcast of a [rows, W] gradient), on the bulk-copy pipeline.
// W is cut into column blocks of cs_wt columns (<= 2 KiB of a row); the
// reduced rows of one (outer kept index, column block) are cut into parts of
// cs_rp rows.  A work item is (outer, part, block).  Per stage the producer
// warp arms the `full` mbarrier and its lanes issue one cp.async.bulk per
// staged row (up to cs_rt <= 32 rows of one block) and bulk operand.  The 8
// consumer warps own 16-byte column chunks (thread t: chunk t % cs_cpr_pad,
// row group t / cs_cpr_pad) and fold the rows of their group in increasing
// order; at the end of an item the row groups are combined in group order and
// the outputs (or, with several parts, per-part partials that
// red_cparts_finalize folds in part order) are written.  Failure handling is
// the row pipeline's: bounded waits, a failed CTA walks its schedule without
// waiting, drains its copies and sets the error word.

// Offsets of reduced row r over every reduced dimension.
__device__ __forceinline__ void cs_row(const RedDev& d, uint32_t r, int64_t* off) {
#pragma unroll
  for (int k = 0; k < kRedOperands; ++k) off[k] = 0;
  for (int q = d.nr - 1; q >= 0; --q) {
    uint32_t c = r;
    if (q > 0) {
      const FastDiv f = fd3(d.fr[q]);
      const uint32_t nq = fdiv(r, f);
      c = r - nq * f.d;
      r = nq;
    }
#pragma unroll
    for (int k = 0; k < kRedOperands; ++k) off[k] += (int64_t)c * d.rst[k][q];
  }
}

template <int MODE>
struct CsIsMax {
  static constexpr bool value = MODE == kRedMax || MODE == kRedArgmax;
};

// The partial of one output of one part.
template <class T, int MODE>
using CsPart = typename std::conditional<CsIsMax<MODE>::value, MaxState<T>, typename Arith<T>::Acc>::type;

template <class T, int MODE, int NB>
__global__ void __launch_bounds__(kRsThreads) red_cstream_kernel(const RedDev d) {
  // the partials' fold kernel, launched after this one, may be scheduled now
  pdl_launch_dependents();
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int S = cs_stages(NB);
  constexpr bool kMax = CsIsMax<MODE>::value;
  using Part = CsPart<T, MODE>;
  extern __shared__ __align__(128) unsigned char smem[];
  Part* comb = reinterpret_cast<Part*>(smem + S * NB * kCsStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * NB * kCsStageBytes + kCsCombBytes);
  uint64_t* empty = full + S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ncb = (uint32_t)d.cs_ncb;
  const uint32_t total = (uint32_t)d.total;
  const uint32_t rp = (uint32_t)d.cs_rp, rt = (uint32_t)d.cs_rt;
  const uint32_t P = (uint32_t)d.P;
  const uint32_t n_items = (uint32_t)d.n_out_outer * P * ncb;
  const int64_t W = d.W;
  const int wt = d.cs_wt, pitch = d.cs_pitch;
  const T* x0 = static_cast<const T*>(d.in[0]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRsConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  uint32_t issued = 0;
  if (warp == 0) {
    uint32_t qn = 0;
    for (uint32_t it = blockIdx.x; it < n_items; it += gridDim.x) {
      const uint32_t cb = it % ncb, op = it / ncb;
      const uint32_t part = op % P, o = op / P;
      int64_t koff[kRedOperands], ooff[2];
      rs_kept(d, o, koff, ooff);
      const int64_t col0 = (int64_t)cb * wt;
      const int64_t wl = W - col0 < wt ? W - col0 : wt;
      const uint32_t bytes = (uint32_t)wl * (uint32_t)sizeof(T);
      const uint32_t r_end = part * rp + rp < total ? part * rp + rp : total;
      for (uint32_t r0 = part * rp; r0 < r_end; r0 += rt, ++qn) {
        const int s = (int)(qn % S);
        if (!failed && qn >= (uint32_t)S) {
          bool ok = true;
          if (lane == 0) ok = mbar_wait(&empty[s], ((qn / S) - 1) & 1u);
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) failed = true;
        }
        if (failed) continue;
        const uint32_t nrows = r_end - r0 < rt ? r_end - r0 : rt;
        if (lane == 0) {
          fence_proxy_async();
          mbar_arrive_expect_tx(&full[s], nrows * bytes * NB);
        }
        __syncwarp();
        if ((uint32_t)lane < nrows) {
          int64_t roff[kRedOperands];
          cs_row(d, r0 + lane, roff);
#pragma unroll
          for (int k = 0; k < kRedOperands; ++k) {
            const int slot = d.bulk_slot[k];
            if (slot >= 0)
              bulk_g2s(smem + (s * NB + slot) * kCsStageBytes + lane * pitch,
                       static_cast<const T*>(d.in[k]) + koff[k] + roff[k] + col0, bytes, &full[s]);
          }
        }
        issued = qn + 1;
      }
    }
  } else {
    const int ct = threadIdx.x - 32;
    const int cpad = d.cs_cpr_pad;
    const int c = ct & (cpad - 1), g = ct / cpad, G = (32 * kRsConsumerWarps) / cpad;
    uint32_t qn = 0;
    for (uint32_t it = blockIdx.x; it < n_items; it += gridDim.x) {
      const uint32_t cb = it % ncb, op = it / ncb;
      const uint32_t part = op % P, o = op / P;
      int64_t koff[kRedOperands], ooff[2];
      rs_kept(d, o, koff, ooff);
      const int64_t col0 = (int64_t)cb * wt;
      const int64_t wl = W - col0 < wt ? W - col0 : wt;
      const bool mine = (int64_t)c * V < wl;
      const uint32_t r_end = part * rp + rp < total ? part * rp + rp : total;
      // the columns' elements at reduced index 0 (max modes' rule), read
      // ahead of the item's end
      RVec<T, V> fv;
      if constexpr (kMax)
        if (g == 0 && mine && P == 1) fv = rload<T, V>(x0 + koff[0] + col0 + (int64_t)c * V);
      Acc acc[V];
      T tb[V];          // strict `>` scan per column from red_lowest,
      uint32_t tr[V];   // with the row of the best (~0: none yet)
#pragma unroll
      for (int i = 0; i < V; ++i) {
        acc[i] = Acc(0);
        tb[i] = red_lowest<T>();
        tr[i] = 0xffffffffu;
      }
      for (uint32_t r0 = part * rp; r0 < r_end; r0 += rt, ++qn) {
        const int s = (int)(qn % S);
        const uint32_t nrows = r_end - r0 < rt ? r_end - r0 : rt;
        if (!failed && !__all_sync(0xffffffffu, mbar_wait(&full[s], (qn / S) & 1u))) failed = true;
        if (!failed && mine) {
          const unsigned char* stage = smem + s * NB * kCsStageBytes + c * 16;
#pragma unroll 4
          for (uint32_t j = g; j < nrows; j += G) {
            const RVec<T, V> v = *reinterpret_cast<const RVec<T, V>*>(stage + j * pitch);
            if constexpr (MODE == kRedSum || MODE == kRedMean) {
#pragma unroll
              for (int i = 0; i < V; ++i) acc[i] = acc[i] + A::to_acc(v.v[i]);
            } else if constexpr (kMax) {
#pragma unroll
              for (int i = 0; i < V; ++i) {
                const bool p = v.v[i] > tb[i];
                tb[i] = p ? v.v[i] : tb[i];
                tr[i] = p ? r0 + j : tr[i];
              }
            } else {  // kRedSum3: gate / mul staged (slot >= 0) or constant along W
              const int s1 = d.bulk_slot[1], s2 = d.bulk_slot[2];
              T sc1 = T(0), sc2 = T(0);
              RVec<T, V> a1, a2;
              if (d.has_gate) {
                if (s1 >= 0) a1 = *reinterpret_cast<const RVec<T, V>*>(stage + s1 * kCsStageBytes + j * pitch);
                else { int64_t ro[kRedOperands]; cs_row(d, r0 + j, ro); sc1 = __ldg(static_cast<const T*>(d.in[1]) + koff[1] + ro[1]); }
              }
              if (d.has_mul) {
                if (s2 >= 0) a2 = *reinterpret_cast<const RVec<T, V>*>(stage + s2 * kCsStageBytes + j * pitch);
                else { int64_t ro[kRedOperands]; cs_row(d, r0 + j, ro); sc2 = __ldg(static_cast<const T*>(d.in[2]) + koff[2] + ro[2]); }
              }
#pragma unroll
              for (int i = 0; i < V; ++i) {
                T x = v.v[i];
                if (d.has_gate) {
                  const T gt = s1 >= 0 ? a1.v[i] : sc1;
                  x = A::mul(x, gt > T(0) ? T(1) : T(0));
                }
                if (d.has_mul) x = A::mul(x, s2 >= 0 ? a2.v[i] : sc2);
                acc[i] = acc[i] + A::to_acc(x);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // row groups -> shared memory, folded in group order by group 0
#pragma unroll
      for (int i = 0; i < V; ++i) {
        if constexpr (kMax) {
          MaxState<T> m;
          m.val = tb[i];
          m.idx = tr[i] == 0xffffffffu ? -1 : (int64_t)tr[i];
          comb[ct * V + i] = m;
        } else {
          comb[ct * V + i] = acc[i];
        }
      }
      named_sync_consumers();
      if (g == 0 && mine && !failed) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int64_t w = col0 + (int64_t)c * V + i;
          if (w - col0 >= wl) break;
          Part t = comb[c * V + i];
          for (int gg = 1; gg < G; ++gg) {
            const Part u = comb[(gg * cpad + c) * V + i];
            if constexpr (kMax) t = max_combine(t, u);
            else t = t + u;
          }
          const uint64_t u_out = (uint64_t)o * (uint64_t)W + (uint64_t)w;
          if (P == 1) {
            RedAcc<T> ra = red_init<T>();
            if constexpr (kMax) ra.m = t;
            else ra.s0 = t;
            int64_t oo[2] = {ooff[0] + w * d.wout[0], ooff[1] + w * d.wout[1]};
            T first = T(0);
            if constexpr (kMax) first = fv.v[i];
            red_write_first<T>(d, ra, oo, first);
          } else {
            static_cast<Part*>(d.parts)[(uint64_t)part * (uint64_t)d.n_out + u_out] = t;
          }
        }
      }
      named_sync_consumers();
    }
  }
  if (__syncthreads_or(failed)) {
    if (threadIdx.x == 0) {
      atomicOr(d.err, kAsyncWaitTimeout);
      const uint32_t start = issued > (uint32_t)S ? issued - S : 0;
      for (uint32_t k = start; k < issued; ++k) mbar_wait(&full[k % S], (k / S) & 1u);
    }
    __syncthreads();
  }
}

// Folds the P per-part partials of every output in part order and writes it.
template <class T, int MODE>
__global__ void __launch_bounds__(256) red_cparts_finalize(const RedDev d) {
  pdl_wait();  // the partials of the kernel before it
  using Part = CsPart<T, MODE>;
  const T* x0 = static_cast<const T*>(d.in[0]);
  const Part* parts = static_cast<const Part*>(d.parts);
  const uint64_t n = (uint64_t)d.n_out;
  for (uint64_t u = (uint64_t)blockIdx.x * 256 + threadIdx.x; u < n; u += (uint64_t)gridDim.x * 256) {
    // the parts in order, loaded eight at a time so their loads overlap
    Part t = parts[u];
    int64_t p = 1;
    for (; p + 8 <= d.P; p += 8) {
      Part v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = parts[(uint64_t)(p + i) * n + u];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if constexpr (CsIsMax<MODE>::value) t = max_combine(t, v[i]);
        else t = t + v[i];
      }
    }
    for (; p < d.P; ++p) {
      const Part v = parts[(uint64_t)p * n + u];
      if constexpr (CsIsMax<MODE>::value) t = max_combine(t, v);
      else t = t + v;
    }
    const uint64_t o = u / (uint64_t)d.W;
    const int64_t w = (int64_t)(u - o * (uint64_t)d.W);
    int64_t koff[kRedOperands], ooff[2];
    kept_offsets(d, o, koff, ooff);
    RedAcc<T> ra = red_init<T>();
    if constexpr (CsIsMax<MODE>::value) ra.m = t;
    else ra.s0 = t;
    int64_t oo[2] = {ooff[0] + w * d.wout[0], ooff[1] + w * d.wout[1]};
    red_write<T>(d, ra, oo, x0, koff[0] + w * d.wst[0]);
  }
}

}  // namespace rk

namespace rk {

template <class T, int MODE, int NB>
const void* stream_kernel_nb() {
  return (const void*)red_stream_kernel<T, MODE, NB>;
}

// The stream kernel for (mode, bulk operands), or null when not instantiated.
template <class T>
const void* pick_red_stream(int mode, int nb) {
  if (mode == kRedSum && nb == 1) return stream_kernel_nb<T, kRedSum, 1>();
  if (mode == kRedMax && nb == 1) return stream_kernel_nb<T, kRedMax, 1>();
  if (mode == kRedArgmax && nb == 1) return stream_kernel_nb<T, kRedArgmax, 1>();
  if constexpr (IsFloat<T>::value) {
    if (mode == kRedMean && nb == 1) return stream_kernel_nb<T, kRedMean, 1>();
    if (mode == kRedSum3 && nb == 1) return stream_kernel_nb<T, kRedSum3, 1>();
    if (mode == kRedSum3 && nb == 2) return stream_kernel_nb<T, kRedSum3, 2>();
    if (mode == kRedSum3 && nb == 3) return stream_kernel_nb<T, kRedSum3, 3>();
    if (mode == kRedAffineRelu && nb == 2) return stream_kernel_nb<T, kRedAffineRelu, 2>();
  }
  return nullptr;
}

template <class T, int MODE, int NB>
const void* cstream_kernel_nb() {
  return (const void*)red_cstream_kernel<T, MODE, NB>;
}

// The column stream kernel for (mode, bulk operands), or null.
template <class T>
const void* pick_red_cstream(int mode, int nb) {
  if (mode == kRedSum && nb == 1) return cstream_kernel_nb<T, kRedSum, 1>();
  if (mode == kRedMax && nb == 1) return cstream_kernel_nb<T, kRedMax, 1>();
  if (mode == kRedArgmax && nb == 1) return cstream_kernel_nb<T, kRedArgmax, 1>();
  if constexpr (IsFloat<T>::value) {
    if (mode == kRedMean && nb == 1) return cstream_kernel_nb<T, kRedMean, 1>();
    if (mode == kRedSum3 && nb == 1) return cstream_kernel_nb<T, kRedSum3, 1>();
    if (mode == kRedSum3 && nb == 2) return cstream_kernel_nb<T, kRedSum3, 2>();
    if (mode == kRedSum3 && nb == 3) return cstream_kernel_nb<T, kRedSum3, 3>();
  }
  return nullptr;
}

template <class T>
const void* pick_red_cfinalize(int mode) {
  switch (mode) {
    case kRedSum: return (const void*)red_cparts_finalize<T, kRedSum>;
    case kRedMax: return (const void*)red_cparts_finalize<T, kRedMax>;
    case kRedArgmax: return (const void*)red_cparts_finalize<T, kRedArgmax>;
  }
  if constexpr (IsFloat<T>::value) {
    switch (mode) {
      case kRedMean: return (const void*)red_cparts_finalize<T, kRedMean>;
      case kRedSum3: return (const void*)red_cparts_finalize<T, kRedSum3>;
    }
  }
  return nullptr;
}

template <class T>
const void* pick_red_finalize(int mode) {
  switch (mode) {
    case kRedSum: return (const void*)red_parts_finalize<T, kRedSum>;
    case kRedMax: return (const void*)red_parts_finalize<T, kRedMax>;
    case kRedArgmax: return (const void*)red_parts_finalize<T, kRedArgmax>;
  }
  if constexpr (IsFloat<T>::value) {
    switch (mode) {
      case kRedMean: return (const void*)red_parts_finalize<T, kRedMean>;
      case kRedSum3: return (const void*)red_parts_finalize<T, kRedSum3>;
      case kRedAffineRelu: return (const void*)red_parts_finalize<T, kRedAffineRelu>;
    }
  }
  return nullptr;
}

}  // namespace rk

template <class T>
bool red_stream_available(int mode, int nb) {
  return rk::pick_red_stream<T>(mode, nb) != nullptr;
}

template <class T>
bool red_cstream_available(int mode, int nb) {
  return rk::pick_red_cstream<T>(mode, nb) != nullptr;
}

// A fold kernel launched with programmatic stream serialization: it is
// scheduled while the reduction before it finishes and waits (pdl_wait) for
// that grid's completion, which removes the gap between the two launches.
inline cudaError_t launch_fold(const void* k, unsigned grid, void** args, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, k, args);
}

template <class T>
Error red_launch(RedDev& d, const RedChoice& c, cudaStream_t stream) {
  using namespace rk;
  const DeviceInfo& dev = current_device_info();
  if (d.n_out == 0) return Error{};
  constexpr int VW = 16 / sizeof(T);
  if (c.variant == kRedRowStream) {
    const void* k = pick_red_stream<T>(d.mode, c.nb);
    if (!k) return make_error(TRS_ERR_ARG, "no stream reduction kernel for this mode");
    const int S = rs_stages(c.nb, d.mode);
    const int smem = S * c.nb * kRsTileBytes + 2 * S * 8;
    allow_smem(k, smem);  // once per kernel
    const int per_sm = resident_blocks_smem(k, kRsThreads, smem);
    const uint64_t items = (uint64_t)d.n_out * (uint64_t)d.P;
    const uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
    const unsigned grid = (unsigned)(items < cap ? items : cap);
    Scratch parts;
    if (d.P > 1) {
      Error e = parts.alloc(sizeof(RedAcc<T>) * items, stream);
      if (!e.ok()) return e;
      d.parts = parts.get();
    }
    void* args[] = {(void*)&d};
    cudaError_t ce = cudaLaunchKernel(k, dim3(grid), dim3(kRsThreads), args, (size_t)smem, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "stream reduction launch");
    Error e = check_launch("stream reduction kernel");
    if (!e.ok()) return e;
    if (d.P > 1) {
      const void* fk = pick_red_finalize<T>(d.mode);
      const uint64_t fb = ((uint64_t)d.n_out + 255) / 256;
      const unsigned fg = (unsigned)(fb < (uint64_t)dev.sm_count * 8 ? fb : (uint64_t)dev.sm_count * 8);
      ce = launch_fold(fk, fg, args, stream);
      if (ce != cudaSuccess) return cuda_error(ce, "partials finalize launch");
      return check_launch("reduction finalize kernel");
    }
    return Error{};
  }
  if (c.variant == kRedColStream) {
    const void* k = pick_red_cstream<T>(d.mode, c.nb);
    if (!k) return make_error(TRS_ERR_ARG, "no column stream reduction kernel for this mode");
    const int smem = cs_smem_bytes(c.nb);
    allow_smem(k, smem);  // once per kernel
    const uint64_t items = (uint64_t)d.n_out_outer * (uint64_t)d.P * (uint64_t)d.cs_ncb;
    const uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)c.per_sm;
    const unsigned grid = (unsigned)(items < cap ? items : cap);
    Scratch parts;
    if (d.P > 1) {
      const size_t psz = (d.mode == kRedMax || d.mode == kRedArgmax) ? sizeof(MaxState<T>)
                                                                      : sizeof(typename Arith<T>::Acc);
      Error e = parts.alloc(psz * (size_t)d.n_out * (size_t)d.P, stream);
      if (!e.ok()) return e;
      d.parts = parts.get();
    }
    void* args[] = {(void*)&d};
    cudaError_t ce = cudaLaunchKernel(k, dim3(grid), dim3(kRsThreads), args, (size_t)smem, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "column stream reduction launch");
    Error e = check_launch("column stream reduction kernel");
    if (!e.ok()) return e;
    if (d.P > 1) {
      const void* fk = pick_red_cfinalize<T>(d.mode);
      const uint64_t fb = ((uint64_t)d.n_out + 255) / 256;
      const unsigned fg = (unsigned)(fb < (uint64_t)dev.sm_count * 8 ? fb : (uint64_t)dev.sm_count * 8);
      ce = launch_fold(fk, fg, args, stream);
      if (ce != cudaSuccess) return cuda_error(ce, "column partials finalize launch");
      return check_launch("column reduction finalize kernel");
    }
    return Error{};
  }
  if (c.variant == kRedRow) {
    if (c.warp_mode) {
      const unsigned grid = (unsigned)((d.n_out + kWarpModeThreads / 32 - 1) / (kWarpModeThreads / 32));
      if (c.vec == VW) red_row_kernel<T, VW, true><<<grid, kWarpModeThreads, 0, stream>>>(d);
      else red_row_kernel<T, 1, true><<<grid, kWarpModeThreads, 0, stream>>>(d);
      return check_launch("row reduction kernel");
    }
    const unsigned grid = (unsigned)(d.n_out * c.cluster);
    if (c.vec == VW) return launch_cluster(red_row_kernel<T, VW, false>, grid, kRowThreads, c.cluster, stream, d);
    return launch_cluster(red_row_kernel<T, 1, false>, grid, kRowThreads, c.cluster, stream, d);
  }
  if (c.variant == kRedCol) {
    const int V = c.vec;
    const uint64_t col_blocks = (uint64_t)((d.W + 32 * V - 1) / (32 * V));
    const unsigned grid = (unsigned)(col_blocks * (uint64_t)d.n_out_outer * c.cluster);
    if (V == VW) return launch_cluster(red_col_kernel<T, VW>, grid, kRowThreads, c.cluster, stream, d);
    return launch_cluster(red_col_kernel<T, 1>, grid, kRowThreads, c.cluster, stream, d);
  }
  uint64_t blocks = ((uint64_t)d.n_out + kRowThreads - 1) / kRowThreads;
  const uint64_t cap = (uint64_t)dev.sm_count * 16;
  if (blocks > cap) blocks = cap;
  red_generic_kernel<T><<<(unsigned)blocks, kRowThreads, 0, stream>>>(d);
  return check_launch("generic reduction kernel");
}


}  // namespace trs
