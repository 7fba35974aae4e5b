// softmax.cu -- K-SOFTMAX: SoftMax::forward over the last axis
// (activation/softmax.rs:42-68).  The reference takes five passes over the
// data (max_axis, x - max, powf(E, .), sum_axis_keepdim, e / sum); here each
// row is read and written once:
//   m = max_axis(row)          the reference's max (a NaN at index 0 is kept)
//   e = powf(E, x - m)         x - m rounded to T, then E^(x-m) rounded to T
//   s = sum of e               accumulated in f64, rounded once to T
//   out = e / s                IEEE division in T
// Kernels:
//   softmax_stream_kernel  rows of 4 KiB .. 96 KiB with 16-byte aligned rows:
//                          one CTA per SM; a producer warp streams whole rows
//                          into a ring of shared-memory stages with
//                          cp.async.bulk; the consumer warps take the max, the
//                          exponentials (in place) with the f64 sum, and e / s
//                          from the staged row, reduce across the CTA with two
//                          named barriers, and store with 16-byte stores.
//   softmax_rows_kernel    other rows up to 16384: a warp or a CTA holds the
//                          row in registers.
//   softmax_long_kernel    longer rows: three passes over global memory.
// The max only feeds x - m, where a -0 / +0 maximum gives the same
// difference's exponential (E^0 = 1), so the stream kernel takes it with the
// NaN-ignoring fmax and then applies the reference's NaN-at-index-0 rule.
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

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
            const T p = A::pow_e_nonpos(A::sub(v[c].v[i], mx), d.e_const);
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
      s = s + A::to_acc(A::pow_e_nonpos(A::sub(__ldg(x + bi + e * d.in_step), mx), d.e_const));
    s = block_sum<Acc>(s, red_s);
    if (threadIdx.x == 0) bcast[1] = A::from_acc(s);
    __syncthreads();
    const T sum = bcast[1];
    for (int64_t e = threadIdx.x; e < d.C; e += blockDim.x) {
      const T p = A::pow_e_nonpos(A::sub(__ldg(x + bi + e * d.in_step), mx), d.e_const);
      out[bo + e * d.out_step] = A::div(p, sum, nullptr);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// softmax_stream_kernel: the bulk-copy row pipeline (see the file comment).
// Consumers work on the staged row in shared memory in three passes: the max;
// e = E^(x - m) written back over x, with the f64 sum; e / sum streamed out.
// Each thread reads back only the chunks it wrote, so the passes need no
// barrier beyond the two CTA-wide reductions, and few registers stay live
// per thread, which leaves room for many exponentials in flight.
#ifndef TRS_SM_CONSUMER_WARPS
#define TRS_SM_CONSUMER_WARPS 16
#endif
constexpr int kSmConsumerWarps = TRS_SM_CONSUMER_WARPS;
constexpr int kSmConsumers = 32 * kSmConsumerWarps;
constexpr int kSmThreads = 32 + kSmConsumers;
constexpr int kSmStageBudget = 192 * 1024;
constexpr int kSmMaxStages = 8;
constexpr uint32_t kSmCopyBytes = 16384;  // one bulk copy per 16 KiB of a row

// The consumer warps form kSmGroups groups that take alternate rows, so one
// group computes while the other waits at a barrier of its row.
#ifndef TRS_SM_GROUPS
#define TRS_SM_GROUPS 2
#endif
constexpr int kSmGroups = TRS_SM_GROUPS;
constexpr int kSmGroupWarps = kSmConsumerWarps / kSmGroups;
constexpr int kSmGroupThreads = 32 * kSmGroupWarps;

__device__ __forceinline__ void sm_group_sync(int grp) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "n"(kSmGroupThreads) : "memory");
}

template <class T>
__device__ __forceinline__ T fmax_t(T a, T b) {
  if constexpr (sizeof(T) == 4) return fmaxf(a, b);
  else return fmax(a, b);
}

template <class T, int V>
__device__ __forceinline__ void sstore_stream(T* p, const SVec<T, V>& r) {
  int4 x;
  memcpy(&x, &r, 16);
  __stcs(reinterpret_cast<int4*>(p), x);
}

// The V per-lane accumulators of a thread, added in a fixed order.
template <class Acc, int V>
__device__ __forceinline__ Acc lanes_sum(const Acc (&a)[V]) {
  Acc t = a[0];
#pragma unroll
  for (int i = 1; i < V; ++i) t = t + a[i];
  return t;
}

// Sum over the consumer warps (fixed order), returned to every consumer.
// `red` is the group's slice of kSmGroupWarps entries.
template <class Acc>
__device__ __forceinline__ Acc consumer_sum(Acc acc, Acc* red, int cw, int lane, int grp) {
  for (int o = 16; o > 0; o >>= 1) acc = acc + __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) red[cw] = acc;
  sm_group_sync(grp);
  Acc tot = red[0];
#pragma unroll
  for (int w = 1; w < kSmGroupWarps; ++w) tot = tot + red[w];
  sm_group_sync(grp);  // red is reused by the next sum
  return tot;
}

// Tuning knob: independent f64 accumulators per thread in LayerNorm's two
// sums (1: one chain of additions).
#ifndef TRS_LN_NACC
#define TRS_LN_NACC 1
#endif
// Tuning knob: chunks of the normalising pass unrolled (their gamma and beta
// loads in flight together; 8 against 4: 2.5 % at [8192, 16384] in f32, where
// 4 spilled 20 bytes of registers and 8 spills none).
#ifndef TRS_LN_U3
#define TRS_LN_U3 8
#endif

// LayerNorm::forward (nn/layer_norm.rs:20-33) of one staged row: mean =
// sum / F; var = sum((x - mean)^2) / F with the square rounded once (the
// correctly rounded powf(., 2)); denom = sqrt(var + eps) (the correctly
// rounded powf(., 0.5)); out = ((x - mean) / denom) * gamma + beta.  Sums in
// f64, rounded once.  f32 divides by denom through its reciprocal pair and
// the correction step (results below 2^-125: IEEE division).
template <class T>
__device__ __forceinline__ void layer_norm_row(const SmDev& d, const unsigned char* stage, uint32_t nchunk,
                                               uint64_t row, int ct, int cw, int lane, int grp, bool failed,
                                               typename Arith<T>::Acc* red) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int V = 16 / (int)sizeof(T);
  constexpr bool kF32 = std::is_same<T, float>::value;
  const T fc = (T)d.C;
  // one accumulator per lane of the 16-byte chunk (TRS_LN_NACC > 1): V
  // independent chains of additions instead of one, combined pairwise at the end
  constexpr int NA = TRS_LN_NACC > 1 ? V : 1;
  Acc acc[NA];
#pragma unroll
  for (int a = 0; a < NA; ++a) acc[a] = Acc(0);
  if (!failed) {
#pragma unroll 4
    for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
      const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i % NA] = acc[i % NA] + A::to_acc(v.v[i]);
    }
  }
  Acc tot = acc[0];
  if constexpr (NA == 4) tot = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  if constexpr (NA == 2) tot = acc[0] + acc[1];
  const T mean = A::div(A::from_acc(consumer_sum<Acc>(tot, red, cw, lane, grp)), fc, nullptr);
#pragma unroll
  for (int a = 0; a < NA; ++a) acc[a] = Acc(0);
  if (!failed) {
#pragma unroll 4
    for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
      const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const T xm = A::sub(v.v[i], mean);
        acc[i % NA] = acc[i % NA] + A::to_acc(A::mul(xm, xm));
      }
    }
  }
  tot = acc[0];
  if constexpr (NA == 4) tot = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  if constexpr (NA == 2) tot = acc[0] + acc[1];
  const T var = A::div(A::from_acc(consumer_sum<Acc>(tot, red, cw, lane, grp)), fc, nullptr);
  if (failed) return;
  T denom;
  if constexpr (kF32) denom = __fsqrt_rn(A::add(var, (T)d.ln_eps));
  else denom = __dsqrt_rn(A::add(var, (T)d.ln_eps));
  float yh = 0.0f, yl = 0.0f;
  if constexpr (kF32) {
    yh = __frcp_rn(denom);
    yl = (float)__dsub_rn(__drcp_rn((double)denom), (double)yh);
  }
  int64_t bi, bo;
  row_bases(d, row, &bi, &bo);
  T* orow = static_cast<T*>(d.out) + bo;
  const T* gm = static_cast<const T*>(d.gamma) + d.g_off;
  const T* bt = static_cast<const T*>(d.beta) + d.b_off;
  constexpr int kU3 = TRS_LN_U3;
#pragma unroll kU3
  for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
    const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
    SVec<T, V> gv, bv, r;
    if (d.gb_vec) {
      gv = sload<T, V>(gm + (int64_t)k * V);
      bv = sload<T, V>(bt + (int64_t)k * V);
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        gv.v[i] = __ldg(gm + ((int64_t)k * V + i) * d.g_st);
        bv.v[i] = __ldg(bt + ((int64_t)k * V + i) * d.b_st);
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const T xm = A::sub(v.v[i], mean);
      T q;
      if constexpr (kF32) {
        const float q0 = __fmaf_rn(xm, yh, __fmul_rn(xm, yl));
        const float rem = __fmaf_rn(-q0, denom, xm);
        q = __fmaf_rn(rem, yh, q0);
        if (fabsf(q) < 0x1p-125f) q = __fdiv_rn(xm, denom);
      } else {
        q = A::div(xm, denom, nullptr);
      }
      r.v[i] = A::add(A::mul(q, gv.v[i]), bv.v[i]);
    }
    sstore_stream<T, V>(orow + (size_t)k * V, r);
  }
}

enum RowMode { kRowSoftmax = 0, kRowLayerNorm = 1 };

template <class T, int MODE>
__global__ void __launch_bounds__(kSmThreads, 1) softmax_stream_kernel(const SmDev d) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int V = 16 / (int)sizeof(T);
  constexpr bool kF32 = std::is_same<T, float>::value;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full[kSmMaxStages], empty[kSmMaxStages];
  __shared__ T red_max[kSmConsumerWarps];
  __shared__ Acc red_sum[kSmConsumerWarps];
  const int S = d.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row_bytes = (uint32_t)d.C * (uint32_t)sizeof(T);
  const uint32_t nchunk = row_bytes / 16;
  const T* x = static_cast<const T*>(d.in);
  T* out = static_cast<T*>(d.out);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSmGroupWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  uint32_t issued = 0;
  if (warp == 0) {
    if (lane == 0) {
      uint32_t qn = 0;
      for (uint64_t row = blockIdx.x; row < (uint64_t)d.rows; row += gridDim.x, ++qn) {
        const int s = (int)(qn % (uint32_t)S);
        if (!failed && qn >= (uint32_t)S && !mbar_wait(&empty[s], ((qn / S) - 1) & 1u)) failed = true;
        if (failed) continue;
        int64_t bi, bo;
        row_bases(d, row, &bi, &bo);
        fence_proxy_async();
        mbar_arrive_expect_tx(&full[s], row_bytes);
        const unsigned char* src = reinterpret_cast<const unsigned char*>(x + bi);
        unsigned char* dst = smem + (size_t)s * row_bytes;
        for (uint32_t o = 0; o < row_bytes; o += kSmCopyBytes)
          bulk_g2s(dst + o, src + o, row_bytes - o < kSmCopyBytes ? row_bytes - o : kSmCopyBytes, &full[s]);
        issued = qn + 1;
      }
    }
  } else {
    const int grp = (warp - 1) / kSmGroupWarps;
    const int cw = (warp - 1) % kSmGroupWarps;
    const int ct = (threadIdx.x - 32) % kSmGroupThreads;
    T* gred_max = red_max + grp * kSmGroupWarps;
    Acc* gred_sum = red_sum + grp * kSmGroupWarps;
    uint32_t qn = (uint32_t)grp;
    for (uint64_t row = blockIdx.x + (uint64_t)grp * gridDim.x; row < (uint64_t)d.rows;
         row += (uint64_t)kSmGroups * gridDim.x, qn += kSmGroups) {
      const int s = (int)(qn % (uint32_t)S);
      if (!failed && !__all_sync(0xffffffffu, mbar_wait(&full[s], (qn / S) & 1u))) failed = true;
      unsigned char* stage = smem + (size_t)s * row_bytes;
      if constexpr (MODE == kRowLayerNorm) {
        layer_norm_row<T>(d, stage, nchunk, row, ct, cw, lane, grp, failed, gred_sum);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        continue;
      }
      // pass 1: the row maximum (NaN-ignoring), then the reference's rule:
      // a NaN at index 0 is the maximum
      T mx = -INFINITY;
      if (!failed) {
#pragma unroll 4
        for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
          const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
#pragma unroll
          for (int i = 0; i < V; ++i) mx = fmax_t(mx, v.v[i]);
        }
      }
      for (int o = 16; o > 0; o >>= 1) mx = fmax_t(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) gred_max[cw] = mx;
      sm_group_sync(grp);
      T m = gred_max[0];
#pragma unroll
      for (int w = 1; w < kSmGroupWarps; ++w) m = fmax_t(m, gred_max[w]);
      if (!failed) {
        const T first = *reinterpret_cast<const T*>(stage);
        if (is_nan_val(first)) m = first;
      }
      // pass 2: e = powf(E, x - m) over x in place, summed in f64; each
      // thread keeps the least e it produced (f32)
      Acc accs[V];  // one per vector lane: V independent add chains
#pragma unroll
      for (int i = 0; i < V; ++i) accs[i] = Acc(0);
      float emin = INFINITY;
      if (!failed) {
#pragma unroll 4
        for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
          SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            if constexpr (kF32) {
              // two lanes at a time on the packed units (exp_nonpos2 is
              // exp_nonpos lane by lane; x - m is the packed add of -m)
              if (i % 2 == 0) {
                const float2 e2 = expf32::exp_nonpos2(
                    __fadd2_rn(make_float2(v.v[i], v.v[i + 1]), make_float2(-m, -m)), expf32::kBaseEf32);
                v.v[i] = e2.x;
                v.v[i + 1] = e2.y;
              }
              const float e = v.v[i];
              emin = fminf(emin, e);
              accs[i] = accs[i] + (double)e;
            } else {
              const T e = A::pow_e_nonpos(A::sub(v.v[i], m), d.e_const);
              v.v[i] = e;
              accs[i] = accs[i] + A::to_acc(e);
            }
          }
          *reinterpret_cast<SVec<T, V>*>(stage + k * 16) = v;
        }
      }
      Acc acc = lanes_sum<Acc, V>(accs);
      for (int o = 16; o > 0; o >>= 1) acc = acc + __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) gred_sum[cw] = acc;
      sm_group_sync(grp);
      Acc tot = gred_sum[0];
#pragma unroll
      for (int w = 1; w < kSmGroupWarps; ++w) tot = tot + gred_sum[w];
      const T sum = A::from_acc(tot);
      // pass 3: e / sum.  f32: with the reciprocal of the row sum as a pair
      // yh + yl (yh = 1/sum rounded, yl the rounded rest), q0 = e*yh + e*yl
      // is within one ulp of e/sum, so the remainder e - q0*sum is exact (one
      // fused multiply-add) and q0 + rem*yh, rounded once, is the correctly
      // rounded quotient (P. Markstein's correction step).  Results below
      // 2^-125 take the IEEE division itself; a thread whose least e is at
      // least sum * 2^-124 has none (every quotient is above 2^-125), so
      // only the other threads test each result.
      if (!failed) {
        int64_t bi, bo;
        row_bases(d, row, &bi, &bo);
        T* orow = out + bo;
        float yh = 0.0f, yl = 0.0f;
        bool careful = true;
        if constexpr (kF32) {
          yh = __frcp_rn(sum);
          yl = (float)__dsub_rn(__drcp_rn((double)sum), (double)yh);
          careful = !(emin >= __fmul_rn(sum, 0x1p-124f));
        }
        if (kF32 && !careful) {
#pragma unroll 4
          for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
            const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
            SVec<T, V> r;
#pragma unroll
            for (int i = 0; i < V; i += 2) {  // the same steps, two lanes at a time
              const float2 e = make_float2(v.v[i], v.v[i + 1]);
              const float2 yh2 = make_float2(yh, yh), yl2 = make_float2(yl, yl);
              const float2 q0 = __ffma2_rn(e, yh2, __fmul2_rn(e, yl2));
              const float2 rem = __ffma2_rn(make_float2(-q0.x, -q0.y), make_float2(sum, sum), e);
              const float2 q = __ffma2_rn(rem, yh2, q0);
              r.v[i] = q.x;
              r.v[i + 1] = q.y;
            }
            sstore_stream<T, V>(orow + (size_t)k * V, r);
          }
        } else {
#pragma unroll 4
          for (uint32_t k = (uint32_t)ct; k < nchunk; k += kSmGroupThreads) {
            const SVec<T, V> v = *reinterpret_cast<const SVec<T, V>*>(stage + k * 16);
            SVec<T, V> r;
#pragma unroll
            for (int i = 0; i < V; ++i) {
              if constexpr (kF32) {
                const float e = v.v[i];
                const float q0 = __fmaf_rn(e, yh, __fmul_rn(e, yl));
                const float rem = __fmaf_rn(-q0, sum, e);
                float q = __fmaf_rn(rem, yh, q0);
                if (fabsf(q) < 0x1p-125f) q = __fdiv_rn(e, sum);
                r.v[i] = q;
              } else {
                r.v[i] = A::div(v.v[i], sum, nullptr);
              }
            }
            sstore_stream<T, V>(orow + (size_t)k * V, r);
          }
        }
      }
      // the consumers wrote this stage; order those writes before the next
      // bulk copy into it, then release it
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (__syncthreads_or(failed)) {
    if (threadIdx.x == 0) {
      atomicOr(d.err, kAsyncWaitTimeout);
      const uint32_t start = issued > (uint32_t)S ? issued - (uint32_t)S : 0;
      for (uint32_t k = start; k < issued; ++k) mbar_wait(&full[k % S], (k / S) & 1u);
    }
    __syncthreads();
  }
}

template <class T, int MODE = kRowSoftmax>
Error launch_softmax_stream(const SmDev& d, cudaStream_t stream) {
  auto k = softmax_stream_kernel<T, MODE>;
  const int smem = d.stages * (int)(d.C * (int64_t)sizeof(T));
  allow_smem((const void*)k, kSmStageBudget);  // once per kernel
  const uint64_t sms = (uint64_t)current_device_info().sm_count;
  const unsigned grid = (unsigned)((uint64_t)d.rows < sms ? (uint64_t)d.rows : sms);
  k<<<grid, kSmThreads, smem, stream>>>(d);
  return check_launch("softmax stream kernel");
}

// Whether the stream kernel takes these rows (else the register kernels run).
template <class T>
bool softmax_stream_fits(const SmDev& d, bool aligned) {
  const int64_t row_bytes = d.C * (int64_t)sizeof(T);
  return aligned && d.in_step == 1 && d.out_step == 1 && row_bytes % 16 == 0 && row_bytes >= 4096 &&
         row_bytes * 2 <= kSmStageBudget && d.err != nullptr;
}

template <class T>
Error launch_softmax_stream_typed(SmDev d, cudaStream_t stream) {
  const int64_t row_bytes = d.C * (int64_t)sizeof(T);
  int64_t st = kSmStageBudget / row_bytes;
  d.stages = (int)(st > kSmMaxStages ? kSmMaxStages : st);
  return launch_softmax_stream<T>(d, stream);
}

template <class K>
unsigned grid_of(K kernel, int threads, uint64_t work) {
  const DeviceInfo& dev = current_device_info();
  const int per_sm = resident_blocks_smem((const void*)kernel, threads, 0);
  const uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
  const uint64_t g = work < cap ? work : cap;
  return (unsigned)(g < 1 ? 1 : g);
}

template <class T>
Error launch_softmax_typed(const SmDev& d, int vec, cudaStream_t stream) {
  if (d.rows == 0 || d.C == 0) return Error{};
  constexpr int VW = 16 / sizeof(T);
  if (softmax_stream_fits<T>(d, vec == VW)) return launch_softmax_stream_typed<T>(d, stream);
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

Error run_layer_norm_stream(SmDev d, int dtype, cudaStream_t stream) {
  const int es = dtype_size(dtype);
  const int64_t row_bytes = d.C * es;
  bool ok = d.in_step == 1 && d.out_step == 1 && row_bytes % 16 == 0 && row_bytes >= 4096 &&
            row_bytes * 2 <= kSmStageBudget;
  if (((uintptr_t)d.in + (uintptr_t)(d.in_off * es)) % 16) ok = false;
  if (((uintptr_t)d.out + (uintptr_t)(d.out_off * es)) % 16) ok = false;
  for (int i = 0; i < d.nouter; ++i)
    if ((d.ist[i] * es) % 16 || (d.ost[i] * es) % 16) ok = false;
  d.err = async_error_word();
  if (!ok || !d.err || d.rows == 0) return make_error(TRS_NONE, "rows do not suit the row pipeline");
  d.gb_vec = d.g_st == 1 && d.b_st == 1 &&
             ((uintptr_t)d.gamma + (uintptr_t)(d.g_off * es)) % 16 == 0 &&
             ((uintptr_t)d.beta + (uintptr_t)(d.b_off * es)) % 16 == 0;
  int64_t st = kSmStageBudget / row_bytes;
  d.stages = (int)(st > kSmMaxStages ? kSmMaxStages : st);
  if (dtype == TRS_F32) return launch_softmax_stream<float, kRowLayerNorm>(d, stream);
  return launch_softmax_stream<double, kRowLayerNorm>(d, stream);
}

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
  d.err = async_error_word();
  if (x->dtype == TRS_F32) {
    d.e_const = std::log2((double)2.7182817f);
    return launch_softmax_typed<float>(d, vec ? VW : 1, stream);
  }
  d.e_const = 2.718281828459045;
  return launch_softmax_typed<double>(d, vec ? VW : 1, stream);
}

}  // namespace trs
