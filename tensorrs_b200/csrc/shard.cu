// shard.cu -- the device side of combining per-rank partials of a tensor
// split on axis 0: rounding all-reduced f64 sums into the output view, and
// folding the gathered max/argmax records of every rank in rank order.
#include <cstring>

#include "kernels.cuh"
#include "reduce.h"

namespace trs {
namespace {

struct OutDesc {
  int nd;
  int64_t shape[kMaxDims];
  int64_t st[kMaxDims];
  int64_t off;
  int64_t n;
};

__device__ __forceinline__ int64_t out_offset(const OutDesc& o, uint64_t i) {
  int64_t at = o.off;
  for (int d = o.nd - 1; d > 0; --d) {
    const uint64_t q = i / (uint64_t)o.shape[d];
    at += (int64_t)(i - q * (uint64_t)o.shape[d]) * o.st[d];
    i = q;
  }
  if (o.nd > 0) at += (int64_t)i * o.st[0];
  return at;
}

template <class T>
__global__ void __launch_bounds__(kThreads)
accs_to_view_kernel(const typename Arith<T>::Acc* acc, OutDesc o, T* out) {
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < (uint64_t)o.n;
       i += (uint64_t)gridDim.x * kThreads)
    out[out_offset(o, i)] = Arith<T>::from_acc(acc[i]);
}

// records: [nranks][n]; the `first` of rank `first_rank` (the lowest rank
// holding rows) is the element at global index 0.
template <class T>
__global__ void __launch_bounds__(kThreads)
max_records_kernel(const MaxRecord<T>* rec, int nranks, int first_rank, OutDesc o, void* out, int argmax) {
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < (uint64_t)o.n;
       i += (uint64_t)gridDim.x * kThreads) {
    MaxState<T> s;
    s.val = T(0);
    s.idx = -1;
    for (int r = 0; r < nranks; ++r) {
      const MaxRecord<T> p = rec[(uint64_t)r * (uint64_t)o.n + i];
      MaxState<T> t;
      t.val = p.val;
      t.idx = p.idx;
      s = max_combine(s, t);
    }
    const T first = rec[(uint64_t)first_rank * (uint64_t)o.n + i].first;
    if (is_nan_val(first) || s.idx < 0) { s.val = first; s.idx = 0; }
    if (argmax)
      static_cast<int64_t*>(out)[out_offset(o, i)] = s.idx;
    else
      static_cast<T*>(out)[out_offset(o, i)] = s.val;
  }
}

OutDesc describe(const trs_view* v) {
  OutDesc o;
  std::memset(&o, 0, sizeof(o));
  o.nd = v->ndim;
  for (int i = 0; i < v->ndim; ++i) {
    o.shape[i] = v->shape[i];
    o.st[i] = v->strides[i];
  }
  o.off = v->offset;
  o.n = numel_of(v->shape, v->ndim);
  return o;
}

unsigned blocks_for(int64_t n) {
  const uint64_t b = ((uint64_t)n + kThreads - 1) / kThreads;
  const uint64_t cap = (uint64_t)current_device_info().sm_count * 8;
  return (unsigned)(b < 1 ? 1 : (b < cap ? b : cap));
}

// ---- the axis-0 exchange over peer memory ------------------------------------

// Each wait polls at most kAxis0Polls times, 256 ns apart (about 2 s).
constexpr unsigned kAxis0Polls = 1u << 23;

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long* x_flag(const Axis0Exchange& x, int owner, int from) {
  return reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(x.peers[owner]) + x.flags_off) +
         (size_t)x.parity * x.world + from;
}
template <class P>
__device__ __forceinline__ const P* x_arena(const Axis0Exchange& x, int r) {
  return reinterpret_cast<const P*>(reinterpret_cast<const char*>(x.peers[r]) + x.arena_off +
                                    (size_t)x.parity * kAxis0Arena);
}

// After this rank's partials are in its arena (the reduction kernel before it
// on the stream): a system-scope fence, then the call's number into every
// rank's flag of (parity, this rank), with release semantics.
__global__ void axis0_publish_kernel(const Axis0Exchange x) {
  __threadfence_system();
  for (int t = threadIdx.x; t < x.world; t += blockDim.x) st_release_sys_u64(x_flag(x, t, x.rank), x.seq);
}

// Every CTA: threads t < world wait for rank t's flag (acquire), then the
// CTA's columns are combined from every rank's arena in rank order.  Loads of
// the arenas bypass L1 (a slot is rewritten every second call).  Returns
// false when a wait ran out (the error bit is set).
__device__ __forceinline__ bool axis0_wait(const Axis0Exchange& x) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < x.world) {
    const unsigned long long* f = x_flag(x, x.rank, threadIdx.x);
    unsigned polls = 0;
    while (ld_acquire_sys_u64(f) < x.seq) {
      if (++polls > kAxis0Polls) {
        atomicOr(&failed, 1);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncthreads();
  const bool ok = failed == 0;
  if (!ok && threadIdx.x == 0 && x.err) atomicOr(x.err, kAsyncPeerTimeout);
  return ok;
}

template <class T>
__global__ void __launch_bounds__(kThreads) axis0_sum_combine_kernel(const Axis0Exchange x, OutDesc o, T* out) {
  using Acc = typename Arith<T>::Acc;
  const bool ok = axis0_wait(x);
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < (uint64_t)o.n;
       i += (uint64_t)gridDim.x * kThreads) {
    T v;
    if (ok) {
      Acc acc = Acc(0);
      for (int r = 0; r < x.world; ++r) acc = acc + __ldcv(x_arena<Acc>(x, r) + i);
      v = Arith<T>::from_acc(acc);
    } else {
      v = IsFloat<T>::value ? (T)NAN : T(0);
    }
    out[out_offset(o, i)] = v;
  }
}

template <class T>
__global__ void __launch_bounds__(kThreads)
axis0_max_combine_kernel(const Axis0Exchange x, int first_rank, OutDesc o, void* out, int argmax) {
  const bool ok = axis0_wait(x);
  for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < (uint64_t)o.n;
       i += (uint64_t)gridDim.x * kThreads) {
    MaxState<T> s;
    s.val = T(0);
    s.idx = -1;
    if (ok) {
      for (int r = 0; r < x.world; ++r) {
        const MaxRecord<T>* p = x_arena<MaxRecord<T>>(x, r) + i;
        MaxState<T> t;
        t.val = __ldcv(&p->val);
        t.idx = __ldcv(&p->idx);
        s = max_combine(s, t);
      }
      const T first = __ldcv(&(x_arena<MaxRecord<T>>(x, first_rank) + i)->first);
      if (is_nan_val(first) || s.idx < 0) { s.val = first; s.idx = 0; }
    } else {
      s.val = IsFloat<T>::value ? (T)NAN : T(0);
      s.idx = -1;
    }
    if (argmax)
      static_cast<int64_t*>(out)[out_offset(o, i)] = s.idx;
    else
      static_cast<T*>(out)[out_offset(o, i)] = s.val;
  }
}

// A grid whose CTAs all fit on the device at once (each waits for the peers).
template <class K>
unsigned resident_grid(K kernel, int64_t n) {
  const uint64_t b = ((uint64_t)n + kThreads - 1) / kThreads;
  const uint64_t cap = (uint64_t)current_device_info().sm_count *
                       (uint64_t)resident_blocks_smem((const void*)kernel, kThreads, 0);
  return (unsigned)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace

Error run_axis0_publish(const Axis0Exchange& x, cudaStream_t stream) {
  axis0_publish_kernel<<<1, 64, 0, stream>>>(x);
  return check_launch("axis-0 exchange publish kernel");
}

Error run_axis0_sum_combine(int dtype, const Axis0Exchange& x, const trs_view* out, cudaStream_t stream) {
  const OutDesc o = describe(out);
  switch (dtype) {
    case TRS_F32: { auto k = axis0_sum_combine_kernel<float>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, o, static_cast<float*>(out->data)); break; }
    case TRS_F64: { auto k = axis0_sum_combine_kernel<double>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, o, static_cast<double*>(out->data)); break; }
    case TRS_I32: { auto k = axis0_sum_combine_kernel<int32_t>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, o, static_cast<int32_t*>(out->data)); break; }
    case TRS_I64: { auto k = axis0_sum_combine_kernel<int64_t>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, o, static_cast<int64_t*>(out->data)); break; }
    default: return make_error(TRS_ERR_DTYPE, "unknown dtype");
  }
  return check_launch("axis-0 exchange sum kernel");
}

Error run_axis0_max_combine(int dtype, const Axis0Exchange& x, int first_rank, const trs_view* out, bool argmax,
                            cudaStream_t stream) {
  const OutDesc o = describe(out);
  const int am = argmax ? 1 : 0;
  switch (dtype) {
    case TRS_F32: { auto k = axis0_max_combine_kernel<float>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, first_rank, o, out->data, am); break; }
    case TRS_F64: { auto k = axis0_max_combine_kernel<double>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, first_rank, o, out->data, am); break; }
    case TRS_I32: { auto k = axis0_max_combine_kernel<int32_t>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, first_rank, o, out->data, am); break; }
    case TRS_I64: { auto k = axis0_max_combine_kernel<int64_t>; k<<<resident_grid(k, o.n), kThreads, 0, stream>>>(x, first_rank, o, out->data, am); break; }
    default: return make_error(TRS_ERR_DTYPE, "unknown dtype");
  }
  return check_launch("axis-0 exchange max kernel");
}

Error run_accs_to_view(int dtype, const void* acc, const trs_view* out, cudaStream_t stream) {
  const OutDesc o = describe(out);
  if (o.n == 0) return Error{};
  const unsigned g = blocks_for(o.n);
  switch (dtype) {
    case TRS_F32: accs_to_view_kernel<float><<<g, kThreads, 0, stream>>>(static_cast<const double*>(acc), o, static_cast<float*>(out->data)); break;
    case TRS_F64: accs_to_view_kernel<double><<<g, kThreads, 0, stream>>>(static_cast<const double*>(acc), o, static_cast<double*>(out->data)); break;
    case TRS_I32: accs_to_view_kernel<int32_t><<<g, kThreads, 0, stream>>>(static_cast<const uint32_t*>(acc), o, static_cast<int32_t*>(out->data)); break;
    case TRS_I64: accs_to_view_kernel<int64_t><<<g, kThreads, 0, stream>>>(static_cast<const uint64_t*>(acc), o, static_cast<int64_t*>(out->data)); break;
    default: return make_error(TRS_ERR_DTYPE, "unknown dtype");
  }
  return check_launch("accumulator conversion kernel");
}

Error run_max_records(int dtype, const void* records, int nranks, int first_rank, const trs_view* out,
                      bool argmax, cudaStream_t stream) {
  const OutDesc o = describe(out);
  if (o.n == 0) return Error{};
  const unsigned g = blocks_for(o.n);
  const int am = argmax ? 1 : 0;
  switch (dtype) {
    case TRS_F32: max_records_kernel<float><<<g, kThreads, 0, stream>>>(static_cast<const MaxRecord<float>*>(records), nranks, first_rank, o, out->data, am); break;
    case TRS_F64: max_records_kernel<double><<<g, kThreads, 0, stream>>>(static_cast<const MaxRecord<double>*>(records), nranks, first_rank, o, out->data, am); break;
    case TRS_I32: max_records_kernel<int32_t><<<g, kThreads, 0, stream>>>(static_cast<const MaxRecord<int32_t>*>(records), nranks, first_rank, o, out->data, am); break;
    case TRS_I64: max_records_kernel<int64_t><<<g, kThreads, 0, stream>>>(static_cast<const MaxRecord<int64_t>*>(records), nranks, first_rank, o, out->data, am); break;
    default: return make_error(TRS_ERR_DTYPE, "unknown dtype");
  }
  return check_launch("max record combine kernel");
}

size_t max_record_size(int dtype) {
  switch (dtype) {
    case TRS_F32: return sizeof(MaxRecord<float>);
    case TRS_F64: return sizeof(MaxRecord<double>);
    case TRS_I32: return sizeof(MaxRecord<int32_t>);
    case TRS_I64: return sizeof(MaxRecord<int64_t>);
  }
  return 0;
}

}  // namespace trs
