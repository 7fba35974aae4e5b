// softmax.cu -- K-SOFTMAX: SoftMax::forward over the last axis
// (activation/softmax.rs:42-68).  The reference takes five passes over the
// data (max_axis, x - max, powf(E, .), sum_axis_keepdim, e / sum); here one
// warp or one CTA holds a row in registers and reads and writes it once:
//   m = max_axis(row)          strict `>` scan semantics (MaxState)
//   e = powf(E, x - m)         x - m rounded to T, then E^(x-m) rounded to T
//   s = sum of e               accumulated in f64, rounded once to T
//   out = e / s                IEEE division in T
// Rows longer than a CTA can hold in registers take three passes over global
// memory instead (max, sum, write).
#include <cmath>
#include <cstring>

#include "kernels.cuh"
#include "softmax.h"

namespace trs {
namespace {

template <class T, int V>
struct alignas(sizeof(T) * V) SVec {
  T v[V];
};

template <class T, int V>
__device__ __forceinline__ SVec<T, V> sload(const T* p) {
  SVec<T, V> r;
  if constexpr (sizeof(T) * V == 16) {
    int4 x = __ldg(reinterpret_cast<const int4*>(p));
    memcpy(&r, &x, 16);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = __ldg(p + i);
  }
  return r;
}

template <class T, int V>
__device__ __forceinline__ void sstore(T* p, const SVec<T, V>& r) {
  if constexpr (sizeof(T) * V == 16) {
    int4 x;
    memcpy(&x, &r, 16);
    *reinterpret_cast<int4*>(p) = x;
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = r.v[i];
  }
}

__device__ __forceinline__ void row_bases(const SmDev& d, uint64_t row, int64_t* bi, int64_t* bo) {
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

// GROUP threads (a warp, or a whole CTA) per row; each holds up to CH chunks
// of V elements in registers.
template <class T, int V, int CH, int GROUP, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_rows_kernel(const SmDev d) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int kGroups = THREADS / GROUP;
  __shared__ MaxState<T> red_m[32];
  __shared__ Acc red_s[32];
  __shared__ T bcast[2];
  const T* x = static_cast<const T*>(d.in);
  T* out = static_cast<T*>(d.out);
  const int g_lane = threadIdx.x % GROUP;
  const int g_id = threadIdx.x / GROUP;
  const int64_t C = d.C;
  const bool unit = d.in_step == 1 && d.out_step == 1;
  for (uint64_t row0 = (uint64_t)blockIdx.x * kGroups; row0 < (uint64_t)d.rows;
       row0 += (uint64_t)gridDim.x * kGroups) {
    const uint64_t row = row0 + g_id;
    const bool live = row < (uint64_t)d.rows;
    int64_t bi = 0, bo = 0;
    if (live) row_bases(d, row, &bi, &bo);
    SVec<T, V> v[CH];
    MaxState<T> m;
    m.val = T(0);
    m.idx = -1;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
        if (V > 1 && unit) {
          v[c] = sload<T, V>(x + bi + e);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i)
            v[c].v[i] = e + i < C ? __ldg(x + bi + (e + i) * d.in_step) : T(0);
        }
#pragma unroll
        for (int i = 0; i < V; ++i)
          if (e + i < C) max_push(m, v[c].v[i], e + i);
      }
    }
    // row maximum, with a NaN at index 0 kept as the reference keeps it
    T mx;
    if constexpr (GROUP == 32) {
      m = warp_max(m);
      mx = __shfl_sync(0xffffffffu, m.val, 0);
      const int64_t mi = __shfl_sync(0xffffffffu, m.idx, 0);
      const T first = live ? __ldg(x + bi) : T(0);
      if (is_nan_val(first) || mi < 0) mx = first;
    } else {
      m = block_max(m, red_m);
      if (threadIdx.x == 0) {
        const T first = live ? __ldg(x + bi) : T(0);
        bcast[0] = (is_nan_val(first) || m.idx < 0) ? first : m.val;
      }
      __syncthreads();
      mx = bcast[0];
    }
    // e = powf(E, x - m); sum in f64
    Acc s = Acc(0);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (e + i < C) {
            const T p = A::pow_e_inline(A::sub(v[c].v[i], mx), d.e_const);
            v[c].v[i] = p;
            s = s + A::to_acc(p);
          }
        }
      }
    }
    T sum;
    if constexpr (GROUP == 32) {
      for (int o = 16; o > 0; o >>= 1) s = s + __shfl_down_sync(0xffffffffu, s, o);
      sum = A::from_acc(__shfl_sync(0xffffffffu, s, 0));
    } else {
      s = block_sum<Acc>(s, red_s);
      if (threadIdx.x == 0) bcast[1] = A::from_acc(s);
      __syncthreads();
      sum = bcast[1];
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t e = ((int64_t)c * GROUP + g_lane) * V;
      if (live && e < C) {
        SVec<T, V> r;
#pragma unroll
        for (int i = 0; i < V; ++i) r.v[i] = A::div(v[c].v[i], sum, nullptr);
        if (V > 1 && unit) {
          sstore<T, V>(out + bo + e, r);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i)
            if (e + i < C) out[bo + (e + i) * d.out_step] = r.v[i];
        }
      }
    }
    if constexpr (GROUP != 32) __syncthreads();
  }
}

// Long rows: one CTA per row, three passes over global memory.
template <class T>
__global__ void __launch_bounds__(1024) softmax_long_kernel(const SmDev d) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  __shared__ MaxState<T> red_m[32];
  __shared__ Acc red_s[32];
  __shared__ T bcast[2];
  const T* x = static_cast<const T*>(d.in);
  T* out = static_cast<T*>(d.out);
  for (uint64_t row = blockIdx.x; row < (uint64_t)d.rows; row += gridDim.x) {
    int64_t bi, bo;
    row_bases(d, row, &bi, &bo);
    MaxState<T> m;
    m.val = T(0);
    m.idx = -1;
    for (int64_t e = threadIdx.x; e < d.C; e += blockDim.x) max_push(m, __ldg(x + bi + e * d.in_step), e);
    m = block_max(m, red_m);
    if (threadIdx.x == 0) {
      const T first = __ldg(x + bi);
      bcast[0] = (is_nan_val(first) || m.idx < 0) ? first : m.val;
    }
    __syncthreads();
    const T mx = bcast[0];
    Acc s = Acc(0);
    for (int64_t e = threadIdx.x; e < d.C; e += blockDim.x)
      s = s + A::to_acc(A::pow_e_inline(A::sub(__ldg(x + bi + e * d.in_step), mx), d.e_const));
    s = block_sum<Acc>(s, red_s);
    if (threadIdx.x == 0) bcast[1] = A::from_acc(s);
    __syncthreads();
    const T sum = bcast[1];
    for (int64_t e = threadIdx.x; e < d.C; e += blockDim.x) {
      const T p = A::pow_e_inline(A::sub(__ldg(x + bi + e * d.in_step), mx), d.e_const);
      out[bo + e * d.out_step] = A::div(p, sum, nullptr);
    }
    __syncthreads();
  }
}

template <class K>
unsigned grid_of(K kernel, int threads, uint64_t work) {
  const DeviceInfo& dev = current_device_info();
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
  const uint64_t g = work < cap ? work : cap;
  return (unsigned)(g < 1 ? 1 : g);
}

template <class T>
Error launch_softmax_typed(const SmDev& d, int vec, cudaStream_t stream) {
  if (d.rows == 0 || d.C == 0) return Error{};
  constexpr int VW = 16 / sizeof(T);
  const int64_t C = d.C;
  // warp per row
  if (C <= 32 * 32) {
    constexpr int TH = 256, G = 32, kG = TH / G;
    const uint64_t work = ((uint64_t)d.rows + kG - 1) / kG;
    if (C <= 32 * 4) {
      auto k = softmax_rows_kernel<T, 1, 4, G, TH>;
      k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
    } else if (C <= 32 * 8) {
      auto k = softmax_rows_kernel<T, 1, 8, G, TH>;
      k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
    } else if (vec == VW) {
      auto k = softmax_rows_kernel<T, VW, 32 / VW, G, TH>;
      k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
    } else {
      auto k = softmax_rows_kernel<T, 1, 32, G, TH>;
      k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
    }
    return check_launch("softmax kernel");
  }
  // CTA per row, row in registers
  if (C <= 512 * 32) {
    constexpr int TH = 512;
    const uint64_t work = (uint64_t)d.rows;
    if (vec == VW) {
      if (C <= 512 * 8) {
        auto k = softmax_rows_kernel<T, VW, 8 / VW, TH, TH>;
        k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
      } else if (C <= 512 * 16) {
        auto k = softmax_rows_kernel<T, VW, 16 / VW, TH, TH>;
        k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
      } else {
        auto k = softmax_rows_kernel<T, VW, 32 / VW, TH, TH>;
        k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
      }
    } else {
      auto k = softmax_rows_kernel<T, 1, 32, TH, TH>;
      k<<<grid_of(k, TH, work), TH, 0, stream>>>(d);
    }
    return check_launch("softmax kernel");
  }
  auto k = softmax_long_kernel<T>;
  k<<<grid_of(k, 1024, (uint64_t)d.rows), 1024, 0, stream>>>(d);
  return check_launch("softmax kernel (long rows)");
}

}  // namespace

Error run_softmax(const trs_view* x, const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(x, "input");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (!is_float(x->dtype)) return make_error(TRS_ERR_DTYPE, "softmax needs f32 or f64");
  if (out->dtype != x->dtype) return make_error(TRS_ERR_DTYPE, "output dtype differs from the input");
  if (x->ndim < 1) return make_error(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
  bool same = out->ndim == x->ndim;
  for (int i = 0; same && i < x->ndim; ++i) same = out->shape[i] == x->shape[i];
  if (!same) return make_error(TRS_ERR_SHAPE, "output shape differs from the input");
  const int last = x->ndim - 1;
  if (x->shape[last] == 0 && numel_of(x->shape, x->ndim) > 0)
    return make_error(TRS_ERR_EMPTY_AXIS, "!!!Cannot reduce an empty axis!!!");
  SmDev d;
  std::memset(&d, 0, sizeof(d));
  d.in = x->data;
  d.out = out->data;
  d.in_off = x->offset;
  d.out_off = out->offset;
  d.C = x->shape[last];
  d.in_step = x->strides[last];
  d.out_step = out->strides[last];
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
  if (x->dtype == TRS_F32) {
    d.e_const = std::log((double)2.7182817f);
    return launch_softmax_typed<float>(d, vec ? VW : 1, stream);
  }
  d.e_const = 2.718281828459045;
  return launch_softmax_typed<double>(d, vec ? VW : 1, stream);
}

}  // namespace trs
