// ew_kernels.cuh -- the element-wise kernel templates and their per-dtype
// launcher (instantiated once per element type in ew_f32.cu, ew_f64.cu,
// ew_i32.cu and ew_i64.cu so the four compile in parallel).
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
#pragma once

#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "kernels.cuh"

namespace trs {
namespace ewk {

template <class T, int V>
struct alignas(sizeof(T) * V) VecT {
  T v[V];
};

template <class T, int V>
__device__ __forceinline__ VecT<T, V> load_vec(const T* p) {
  VecT<T, V> r;
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
__device__ __forceinline__ void store_vec(T* p, const VecT<T, V>& r) {
  if constexpr (sizeof(T) * V == 16) {
    int4 x;
    memcpy(&x, &r, 16);
    *reinterpret_cast<int4*>(p) = x;
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = r.v[i];
  }
}

template <class Acc>
__device__ __forceinline__ void write_partial(Acc acc, Acc* partials) {
  __shared__ Acc red[32];
  Acc s = block_sum<Acc>(acc, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

// --------------------------------------------------------------------------
// ew_vec_kernel: chunk g covers V consecutive elements of one row of the
// innermost folded dimension; chunks are numbered row-major, so consecutive
// threads touch consecutive addresses.  Each thread handles U chunks per
// iteration, issuing all loads before any arithmetic.
template <class T, int V, int U, bool WRITE, bool SUM, bool BIG>
__global__ void __launch_bounds__(kThreads)
ew_vec_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  Acc acc = Acc(0);
  const int nd = d.nd, j = nd - 1;
  const int n_ops = p.n_in + 1;
  const T* in0 = static_cast<const T*>(d.in[0]);
  const T* in1 = static_cast<const T*>(d.in[1]);
  const T* in2 = static_cast<const T*>(d.in[2]);
  T* out = static_cast<T*>(d.out);
  const bool b0 = d.st[1][j] == 0, b1 = d.st[2][j] == 0, b2 = d.st[3][j] == 0;
  const uint64_t step = (uint64_t)gridDim.x * kThreads * U;
  for (uint64_t base = (uint64_t)blockIdx.x * kThreads * U + threadIdx.x; base < d.n_chunks;
       base += step) {
    VecT<T, V> va[U], vb[U], vc[U];
    int64_t oo[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint64_t g = base + (uint64_t)u * kThreads;
      ok[u] = g < d.n_chunks;
      if (!ok[u]) g = 0;
      uint64_t row, col;
      if constexpr (BIG) {
        row = g / d.cpr;
        col = g - row * d.cpr;
      } else {
        uint32_t r32 = fdiv((uint32_t)g, d.f_cpr);
        row = r32;
        col = (uint32_t)g - r32 * d.f_cpr.d;
      }
      int64_t o[kMaxOperands];
#pragma unroll
      for (int k = 0; k < kMaxOperands; ++k) o[k] = d.off[k];
      uint64_t r = row;
      for (int dd = nd - 2; dd > 0; --dd) {
        uint64_t q;
        if constexpr (BIG) q = r / (uint64_t)d.shape[dd];
        else q = fdiv((uint32_t)r, d.f_dim[dd]);
        const int64_t c = (int64_t)(r - q * (uint64_t)d.shape[dd]);
        r = q;
#pragma unroll
        for (int k = 0; k < kMaxOperands; ++k) o[k] += c * d.st[k][dd];
      }
      if (nd >= 2) {
#pragma unroll
        for (int k = 0; k < kMaxOperands; ++k) o[k] += (int64_t)r * d.st[k][0];
      }
      const int64_t e = (int64_t)col * V;
      oo[u] = o[0] + e;
      if (b0) {
        T s = __ldg(in0 + o[1]);
#pragma unroll
        for (int i = 0; i < V; ++i) va[u].v[i] = s;
      } else {
        va[u] = load_vec<T, V>(in0 + o[1] + e);
      }
      if (n_ops > 2) {
        if (b1) {
          T s = __ldg(in1 + o[2]);
#pragma unroll
          for (int i = 0; i < V; ++i) vb[u].v[i] = s;
        } else {
          vb[u] = load_vec<T, V>(in1 + o[2] + e);
        }
      }
      if (n_ops > 3) {
        if (b2) {
          T s = __ldg(in2 + o[3]);
#pragma unroll
          for (int i = 0; i < V; ++i) vc[u].v[i] = s;
        } else {
          vc[u] = load_vec<T, V>(in2 + o[3] + e);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      VecT<T, V> r;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        r.v[i] = apply_program<T>(p, va[u].v[i], vb[u].v[i], vc[u].v[i]);
        if (SUM && ok[u]) acc = acc + A::to_acc(r.v[i]);
      }
      if (WRITE && ok[u]) store_vec<T, V>(out + oo[u], r);
    }
  }
  if constexpr (SUM) write_partial<Acc>(acc, partials);
}

// --------------------------------------------------------------------------
// ew_tile_kernel: tiles of 32 (along i) x 32 (along j, the output's
// unit-stride dimension).  Transposed inputs (unit stride along i) are read
// with lanes along i into shared memory, then every operand is combined with
// lanes along j.  The padded row (33) keeps both phases free of bank
// conflicts.
template <class T, bool WRITE, bool SUM>
__global__ void __launch_bounds__(kThreads)
ew_tile_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  __shared__ T tile[3][32][33];
  Acc acc = Acc(0);
  const int j = d.nd - 1, ti = d.ti;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int64_t Ni = d.shape[ti], Nj = d.shape[j];
  const T* ins[3] = {static_cast<const T*>(d.in[0]), static_cast<const T*>(d.in[1]),
                     static_cast<const T*>(d.in[2])};
  T* out = static_cast<T*>(d.out);
  const int n_in = p.n_in;
  for (uint64_t t = blockIdx.x; t < d.n_tiles; t += gridDim.x) {
    uint64_t rest = t / d.tiles_j;
    const int64_t j0 = (int64_t)(t - rest * d.tiles_j) * 32;
    uint64_t b = rest / d.tiles_i;
    const int64_t i0 = (int64_t)(rest - b * d.tiles_i) * 32;
    int64_t o[kMaxOperands];
#pragma unroll
    for (int k = 0; k < kMaxOperands; ++k) o[k] = d.off[k];
    for (int q = d.n_batch - 1; q >= 0; --q) {
      const int dd = d.batch_dim[q];
      const uint64_t nb = b / (uint64_t)d.shape[dd];
      const int64_t c = (int64_t)(b - nb * (uint64_t)d.shape[dd]);
      b = nb;
#pragma unroll
      for (int k = 0; k < kMaxOperands; ++k) o[k] += c * d.st[k][dd];
    }
    // phase 1: transposed inputs, lanes along i
    for (int k = 0; k < n_in; ++k) {
      if (!d.transposed[k]) continue;
      const int64_t ii = i0 + tx;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t jj = j0 + ty + 8 * r;
        if (ii < Ni && jj < Nj) tile[k][ty + 8 * r][tx] = __ldg(ins[k] + o[k + 1] + ii + jj * d.st[k + 1][j]);
      }
    }
    __syncthreads();
    // phase 2: lanes along j
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t ii = i0 + ty + 8 * r;
      const int64_t jj = j0 + tx;
      if (ii < Ni && jj < Nj) {
        T v[3] = {T(0), T(0), T(0)};
        for (int k = 0; k < n_in; ++k) {
          if (d.transposed[k])
            v[k] = tile[k][tx][ty + 8 * r];
          else
            v[k] = __ldg(ins[k] + o[k + 1] + ii * d.st[k + 1][ti] + jj * d.st[k + 1][j]);
        }
        const T res = apply_program<T>(p, v[0], v[1], v[2]);
        if (SUM) acc = acc + A::to_acc(res);
        if (WRITE) out[o[0] + ii * d.st[0][ti] + jj] = res;
      }
    }
    __syncthreads();
  }
  if constexpr (SUM) write_partial<Acc>(acc, partials);
}

// --------------------------------------------------------------------------
// ew_generic_kernel: one element per thread, every operand's offset decoded
// from the row-major element index.
template <class T, bool WRITE, bool SUM>
__global__ void __launch_bounds__(kThreads)
ew_generic_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  using A = Arith<T>;
  using Acc = typename A::Acc;
  Acc acc = Acc(0);
  const int nd = d.nd;
  const T* ins[3] = {static_cast<const T*>(d.in[0]), static_cast<const T*>(d.in[1]),
                     static_cast<const T*>(d.in[2])};
  T* out = static_cast<T*>(d.out);
  const int n_in = p.n_in;
  const uint64_t step = (uint64_t)gridDim.x * kThreads;
  for (uint64_t g = (uint64_t)blockIdx.x * kThreads + threadIdx.x; g < (uint64_t)d.n; g += step) {
    int64_t o[kMaxOperands];
#pragma unroll
    for (int k = 0; k < kMaxOperands; ++k) o[k] = d.off[k];
    uint64_t r = g;
    for (int dd = nd - 1; dd > 0; --dd) {
      const uint64_t q = r / (uint64_t)d.shape[dd];
      const int64_t c = (int64_t)(r - q * (uint64_t)d.shape[dd]);
      r = q;
#pragma unroll
      for (int k = 0; k < kMaxOperands; ++k) o[k] += c * d.st[k][dd];
    }
#pragma unroll
    for (int k = 0; k < kMaxOperands; ++k) o[k] += (int64_t)r * d.st[k][0];
    T v[3] = {T(0), T(0), T(0)};
    for (int k = 0; k < n_in; ++k) v[k] = __ldg(ins[k] + o[k + 1]);
    const T res = apply_program<T>(p, v[0], v[1], v[2]);
    if (SUM) acc = acc + A::to_acc(res);
    if (WRITE) out[o[0]] = res;
  }
  if constexpr (SUM) write_partial<Acc>(acc, partials);
}

// Adds the per-block partials in a fixed order and rounds once.
template <class T>
__global__ void __launch_bounds__(1024)
sum_finalize_kernel(const typename Arith<T>::Acc* partials, int n, T* out,
                    typename Arith<T>::Acc* raw_out) {
  using Acc = typename Arith<T>::Acc;
  __shared__ Acc red[32];
  Acc s = Acc(0);
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = s + partials[i];
  s = block_sum<Acc>(s, red);
  if (threadIdx.x == 0) {
    if (out) *out = Arith<T>::from_acc(s);
    if (raw_out) *raw_out = s;
  }
}

// Blocks per SM a kernel can keep resident (cached per kernel).
template <class K>
int resident_blocks(K kernel, int threads) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find((const void*)kernel);
  if (it != cache.end()) return it->second;
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0) != cudaSuccess || b < 1) {
    cudaGetLastError();
    b = 1;
  }
  cache[(const void*)kernel] = b;
  return b;
}

}  // namespace ewk

template <class T>
Error ew_launch(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                const SumTarget* sum, const EwPrepared& pr, cudaStream_t stream) {
  using Acc = typename Arith<T>::Acc;
  const EwFold& f = pr.fold;
  const DeviceInfo& dev = current_device_info();
  EwDev d;
  std::memset(&d, 0, sizeof(d));
  d.nd = f.nd;
  for (int i = 0; i < f.nd; ++i) d.shape[i] = f.shape[i];
  for (int k = 0; k < kMaxOperands; ++k) {
    d.off[k] = f.off[k];
    for (int i = 0; i < f.nd; ++i) d.st[k][i] = f.st[k][i];
  }
  for (int k = 0; k < 3; ++k) d.in[k] = k < prog.n_in ? in[k].data : in[0].data;
  d.out = out ? out->data : nullptr;
  d.n = f.n;
  EwParams p;
  p.n_in = prog.n_in;
  p.op1 = prog.op1;
  p.op2 = prog.op2;
  p.epi = prog.epilogue;
  p.p0 = prog.p0;
  p.p1 = prog.p1;
  p.e_const = std::is_same<T, float>::value ? std::log((double)2.7182817f) : 2.718281828459045;
  p.div_flag = nullptr;

  const bool want_sum = sum != nullptr;
  const bool write = out != nullptr;
  if (!want_sum && !write) return Error{};

  // integer division reports a zero divisor through a flag
  Scratch flag_mem;
  const bool int_div = !is_float(pr.dtype) &&
                       ((prog.n_in >= 2 && prog.op1 == TRS_DIV) || (prog.n_in >= 3 && prog.op2 == TRS_DIV) ||
                        prog.epilogue == TRS_UN_DIV_SCALAR);
  if (int_div && f.n > 0) {
    Error e = flag_mem.alloc(sizeof(int), stream);
    if (!e.ok()) return e;
    cudaError_t ce = cudaMemsetAsync(flag_mem.get(), 0, sizeof(int), stream);
    if (ce != cudaSuccess) return cuda_error(ce, "cudaMemsetAsync");
    p.div_flag = flag_mem.as<int>();
  }

  // grid and kernel choice
  const void* kernel = nullptr;
  int blocks = 1;
  auto grid_for = [&](const void* k, int per_sm, uint64_t work_blocks) {
    uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
    uint64_t b = work_blocks < cap ? work_blocks : cap;
    kernel = k;
    blocks = (int)(b < 1 ? 1 : b);
  };
  constexpr int U = 4;
  if (pr.choice.variant == kEwVec) {
    const int V = pr.choice.vec;
    const int j = f.nd - 1;
    d.vec = V;
    d.n_chunks = (uint64_t)f.n / V;
    d.cpr = (uint64_t)f.shape[j] / V;
    bool big = d.n_chunks >= (1ull << 32) || d.cpr == 0;
    for (int i = 0; i < f.nd; ++i)
      if ((uint64_t)f.shape[i] >= (1ull << 32)) big = true;
    if (!big) {
      d.f_cpr = make_fastdiv((uint32_t)d.cpr);
      for (int i = 0; i < f.nd; ++i) d.f_dim[i] = make_fastdiv((uint32_t)f.shape[i]);
    }
    const uint64_t wb = (d.n_chunks + (uint64_t)kThreads * U - 1) / ((uint64_t)kThreads * U);
    constexpr int VW = 16 / sizeof(T);
#define TRS_PICK_VEC(VV, W, S, B)                                                       \
  {                                                                                     \
    auto k = ewk::ew_vec_kernel<T, VV, U, W, S, B>;                                          \
    grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb);                         \
  }
#define TRS_PICK_VEC_WS(VV, B)                                                          \
  if (write && want_sum) TRS_PICK_VEC(VV, true, true, B)                                \
  else if (write) TRS_PICK_VEC(VV, true, false, B)                                      \
  else TRS_PICK_VEC(VV, false, true, B)
    if (V == VW) {
      if (big) TRS_PICK_VEC_WS(VW, true) else TRS_PICK_VEC_WS(VW, false)
    } else {
      if (big) TRS_PICK_VEC_WS(1, true) else TRS_PICK_VEC_WS(1, false)
    }
#undef TRS_PICK_VEC_WS
#undef TRS_PICK_VEC
  } else if (pr.choice.variant == kEwTile) {
    const int j = f.nd - 1, ti = pr.choice.tile_dim;
    d.ti = ti;
    for (int k = 0; k < prog.n_in; ++k) {
      const int64_t s = f.st[k + 1][j];
      d.transposed[k] = (s != 0 && s != 1) ? 1 : 0;
    }
    d.n_batch = 0;
    for (int i = 0; i < f.nd; ++i)
      if (i != ti && i != j) d.batch_dim[d.n_batch++] = i;
    d.tiles_i = ((uint64_t)f.shape[ti] + 31) / 32;
    d.tiles_j = ((uint64_t)f.shape[j] + 31) / 32;
    uint64_t nb = 1;
    for (int q = 0; q < d.n_batch; ++q) nb *= (uint64_t)f.shape[d.batch_dim[q]];
    d.n_tiles = d.tiles_i * d.tiles_j * nb;
    if (write && want_sum) { auto k = ewk::ew_tile_kernel<T, true, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), d.n_tiles); }
    else if (write) { auto k = ewk::ew_tile_kernel<T, true, false>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), d.n_tiles); }
    else { auto k = ewk::ew_tile_kernel<T, false, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), d.n_tiles); }
  } else {
    const uint64_t wb = ((uint64_t)f.n + kThreads - 1) / kThreads;
    if (write && want_sum) { auto k = ewk::ew_generic_kernel<T, true, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
    else if (write) { auto k = ewk::ew_generic_kernel<T, true, false>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
    else { auto k = ewk::ew_generic_kernel<T, false, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
  }

  Scratch partials;
  Acc* part = nullptr;
  if (want_sum) {
    Error e = partials.alloc(sizeof(Acc) * (size_t)blocks, stream);
    if (!e.ok()) return e;
    part = partials.as<Acc>();
  }
  if (f.n > 0) {
    void* args[] = {(void*)&d, (void*)&p, (void*)&part};
    cudaError_t ce = cudaLaunchKernel(kernel, dim3(blocks), dim3(kThreads), args, 0, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "element-wise kernel launch");
    Error e = check_launch("element-wise kernel");
    if (!e.ok()) return e;
  } else if (want_sum) {
    cudaError_t ce = cudaMemsetAsync(part, 0, sizeof(Acc) * (size_t)blocks, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "cudaMemsetAsync");
  }
  if (want_sum) {
    T* sum_out = nullptr;
    if (sum->view) sum_out = static_cast<T*>(sum->view->data) + sum->view->offset;
    ewk::sum_finalize_kernel<T><<<1, 1024, 0, stream>>>(part, blocks, sum_out,
                                                   static_cast<Acc*>(sum->raw_acc));
    Error e = check_launch("sum finalize kernel");
    if (!e.ok()) return e;
  }
  if (p.div_flag) {
    int host_flag = 0;
    cudaError_t ce = cudaMemcpyAsync(&host_flag, p.div_flag, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(stream);
    if (ce != cudaSuccess) return cuda_error(ce, "reading the division flag");
    if (host_flag & 1) return make_error(TRS_ERR_DIV_ZERO, "attempt to divide by zero");
    if (host_flag & 2) return make_error(TRS_ERR_DIV_ZERO, "attempt to divide with overflow");
  }
  return Error{};
}


}  // namespace trs
