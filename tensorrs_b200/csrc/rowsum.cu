// rowsum.cu -- an element-wise program, the sums of its result along the
// last axis and the sum of all of it, in one pass over HBM: the chain
//     let y = &a + &b;  let r = y.sum_axis(1);  let s = y.sum();
// (binary_op, ops.rs:240-300; sum_axis, base.rs:1051-1107; sum,
// base.rs:1024-1030), which the reference runs as three passes and the
// separate entry points here as three launches.
//
// One warp per row of the result: its lanes walk the row in 16-byte chunks
// (all of a lane's loads issued before the first result is combined),
// write Y, and add every result to an f64 accumulator (wrapping unsigned for
// integers) -- the same accumulation as trs_sum_axis and trs_sum.  The warp
// folds its lanes in a fixed order, rounds the row's sum once into the
// row-sums output and keeps the unrounded accumulator; a one-CTA kernel,
// launched by programmatic dependent launch, adds the rows' accumulators in
// row order and rounds the total once.  Per element: the inputs read once,
// Y written once; the row sums and the total add one element per row and one.
#include <cuda_runtime.h>

#include <cstring>
#include <type_traits>

#include "kernels.cuh"

namespace trs {
namespace {

constexpr int kRowWarps = 4;  // rows (warps) per CTA
constexpr int kRowThreads = 32 * kRowWarps;
// Fewer rows than this leave most SMs idle with a warp per row: such calls
// take the three separate passes instead.
constexpr int64_t kMinRows = 256;

struct RowSumDev {
  const void* in[3];
  int64_t off[3];   // element offset of row 0 of each input
  int64_t rs[3];    // row stride of each input (0: the same row for every row)
  int unit[3];      // 1: the input runs along the row with unit stride; 0: one value per row
  int stream[3];    // 1: read once (streaming loads); 0: re-read by other rows
  void* out;        // Y, contiguous
  int64_t out_off;
  void* rows_out;   // row sums, contiguous, or null
  int64_t rows_off;
  uint32_t rows, inner;
};

template <class T, int V>
struct alignas(sizeof(T) * V) Chunk {
  T v[V];
};

template <class T, int V>
__device__ __forceinline__ Chunk<T, V> load_chunk(const T* p, bool stream) {
  Chunk<T, V> r;
  if constexpr (sizeof(T) * V == 16) {
    const int4 x = stream ? __ldcs(reinterpret_cast<const int4*>(p)) : __ldg(reinterpret_cast<const int4*>(p));
    memcpy(&r, &x, 16);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = stream ? __ldcs(p + i) : __ldg(p + i);
  }
  return r;
}

template <class T, int V>
__device__ __forceinline__ void store_chunk(T* p, const Chunk<T, V>& r) {
  if constexpr (sizeof(T) * V == 16) {
    int4 x;
    memcpy(&x, &r, 16);
    __stcs(reinterpret_cast<int4*>(p), x);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) __stcs(p + i, r.v[i]);
  }
}

// PROG is kAdd, kSub, kMul or a runtime program code (ops read from p).
template <class T, int V, int PROG>
__global__ void __launch_bounds__(kRowThreads)
ew_row_sums_kernel(const RowSumDev d, const EwParams p, typename Arith<T>::Acc* row_acc) {
  pdl_launch_dependents();  // the total's fold may be scheduled now
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int NIN = prog_inputs(PROG);
  constexpr int U = NIN == 3 ? 4 : 8;  // chunks per lane in flight
  const int lane = threadIdx.x & 31;
  const uint32_t cpr = d.inner / V;
  T* out = static_cast<T*>(d.out);
  for (uint32_t row = blockIdx.x * kRowWarps + (threadIdx.x >> 5); row < d.rows; row += gridDim.x * kRowWarps) {
    const T* src[NIN];
#pragma unroll
    for (int k = 0; k < NIN; ++k) src[k] = static_cast<const T*>(d.in[k]) + d.off[k] + (int64_t)row * d.rs[k];
    T* dst = out + d.out_off + (int64_t)row * d.inner;
    Acc acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = Acc(0);
    for (uint32_t c0 = lane; c0 < cpr; c0 += 32 * U) {
      Chunk<T, V> v[U][NIN];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t c = c0 + (uint32_t)u * 32;
        if (c < cpr) {
#pragma unroll
          for (int k = 0; k < NIN; ++k) {
            if (d.unit[k]) {
              v[u][k] = load_chunk<T, V>(src[k] + (size_t)c * V, d.stream[k] != 0);
            } else {
              const T s = __ldg(src[k]);
#pragma unroll
              for (int i = 0; i < V; ++i) v[u][k].v[i] = s;
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t c = c0 + (uint32_t)u * 32;
        if (c < cpr) {
          Chunk<T, V> r;
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const T a = v[u][0].v[i];
            const T b = NIN >= 2 ? v[u][NIN >= 2 ? 1 : 0].v[i] : T(0);
            const T cc = NIN >= 3 ? v[u][NIN >= 3 ? 2 : 0].v[i] : T(0);
            r.v[i] = apply_prog<T, PROG>(p, a, b, cc);
            acc[i] = acc[i] + A::to_acc(r.v[i]);
          }
          store_chunk<T, V>(dst + (size_t)c * V, r);
        }
      }
    }
    Acc t = acc[0];
#pragma unroll
    for (int i = 1; i < V; ++i) t = t + acc[i];
    for (int o = 16; o > 0; o >>= 1) t = t + __shfl_down_sync(0xffffffffu, t, o);
    if (lane == 0) {
      if (d.rows_out) static_cast<T*>(d.rows_out)[d.rows_off + row] = A::from_acc(t);
      row_acc[row] = t;
    }
  }
}

// The total: the rows' accumulators added in a fixed order, rounded once.
template <class T>
__global__ void __launch_bounds__(1024)
row_total_kernel(const typename Arith<T>::Acc* row_acc, uint32_t rows, T* total) {
  pdl_wait();  // the row kernel's accumulators
  using Acc = typename Arith<T>::Acc;
  __shared__ Acc red[32];
  Acc s = Acc(0);
  for (uint32_t i = threadIdx.x; i < rows; i += blockDim.x) s = s + row_acc[i];
  s = block_sum<Acc>(s, red);
  if (threadIdx.x == 0) *total = Arith<T>::from_acc(s);
}

bool row_major(const int64_t* shape, const int64_t* strides, int nd) {
  int64_t want = 1;
  for (int i = nd - 1; i >= 0; --i) {
    if (shape[i] == 1) continue;
    if (strides[i] != want) return false;
    want *= shape[i];
  }
  return true;
}

template <class T, int V>
const void* pick_row_kernel(int code) {
  switch (code) {
    case kAdd: return (const void*)ew_row_sums_kernel<T, V, kAdd>;
    case kSub: return (const void*)ew_row_sums_kernel<T, V, kSub>;
    case kMul: return (const void*)ew_row_sums_kernel<T, V, kMul>;
    case kRunSimple1: return (const void*)ew_row_sums_kernel<T, V, kRunSimple1>;
    case kRunSimple2: return (const void*)ew_row_sums_kernel<T, V, kRunSimple2>;
    case kRunSimple3: return (const void*)ew_row_sums_kernel<T, V, kRunSimple3>;
  }
  if constexpr (std::is_floating_point<T>::value) {
    switch (code) {
      case kRunFull1: return (const void*)ew_row_sums_kernel<T, V, kRunFull1>;
      case kRunFull2: return (const void*)ew_row_sums_kernel<T, V, kRunFull2>;
      case kRunFull3: return (const void*)ew_row_sums_kernel<T, V, kRunFull3>;
    }
  }
  return nullptr;
}

template <class T>
Error launch_row_sums(const trs_ew_program& prog, RowSumDev& d, bool vec, const trs_view* total,
                      cudaStream_t stream) {
  using Acc = typename Arith<T>::Acc;
  constexpr int VW = 16 / (int)sizeof(T);
  const bool fl = std::is_floating_point<T>::value;
  // a plain add, subtract or multiply has its own instantiation; every other
  // program reads its ops at run time
  int code = program_code(prog, fl);
  if (code != kAdd && code != kSub && code != kMul)
    code = ((is_simple_program(prog) || !fl) ? kRunSimple1 : kRunFull1) + (prog.n_in - 1);
  const void* k = vec ? pick_row_kernel<T, VW>(code) : pick_row_kernel<T, 1>(code);
  if (!k) return make_error(TRS_ERR_ARG, "no row-sums kernel for this program");
  EwParams p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = prog.n_in;
  p.op1 = prog.op1;
  p.op2 = prog.op2;
  p.epi = prog.epilogue;
  p.p0 = prog.p0;
  p.p1 = prog.p1;
  p.e_const = std::is_same<T, float>::value ? std::log2((double)2.7182817f) : 2.718281828459045;
  p.div_flag = nullptr;
  Scratch acc_mem;
  Error e = acc_mem.alloc(sizeof(Acc) * (size_t)d.rows, stream);
  if (!e.ok()) return e;
  Acc* acc = acc_mem.as<Acc>();
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, kRowThreads, 0);
  const uint64_t need = ((uint64_t)d.rows + kRowWarps - 1) / kRowWarps;
  const unsigned grid = (unsigned)(need < cap ? need : cap);
  void* args[] = {(void*)&d, (void*)&p, (void*)&acc};
  cudaError_t ce = cudaLaunchKernel(k, dim3(grid), dim3(kRowThreads), args, 0, stream);
  if (ce != cudaSuccess) return cuda_error(ce, "row-sums kernel launch");
  e = check_launch("row-sums kernel");
  if (!e.ok()) return e;
  if (total) {
    T* tp = static_cast<T*>(total->data) + total->offset;
    uint32_t rows = d.rows;
    void* targs[] = {(void*)&acc, (void*)&rows, (void*)&tp};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ce = cudaLaunchKernelExC(&cfg, (const void*)row_total_kernel<T>, targs);
    if (ce != cudaSuccess) return cuda_error(ce, "row total launch");
    e = check_launch("row total kernel");
    if (!e.ok()) return e;
  }
  return Error{};
}

}  // namespace

Error run_row_sums_fused(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                         const trs_view* rows_out, const trs_view* total, cudaStream_t stream, bool* taken) {
  *taken = false;
  const int nd = out->ndim;
  const int64_t n = numel_of(out->shape, nd);
  if (nd < 1 || n == 0) return Error{};
  const int dt = out->dtype;
  // integer division reports a zero divisor through a flag: not here
  if (!is_float(dt) && ((prog.n_in >= 2 && prog.op1 == TRS_DIV) || (prog.n_in >= 3 && prog.op2 == TRS_DIV) ||
                        prog.epilogue == TRS_UN_DIV_SCALAR))
    return Error{};
  const int64_t inner = out->shape[nd - 1], rows = n / inner;
  if (rows < kMinRows || inner >= (1ll << 31) || rows >= (1ll << 31)) return Error{};
  if (!row_major(out->shape, out->strides, nd)) return Error{};
  if (rows_out && !row_major(rows_out->shape, rows_out->strides, rows_out->ndim)) return Error{};
  const int es = dtype_size(dt);
  const int VW = 16 / es;
  auto aligned = [&](const void* base, int64_t off) {
    return ((uintptr_t)base + (uintptr_t)(off * (int64_t)es)) % 16 == 0;
  };
  RowSumDev d;
  std::memset(&d, 0, sizeof(d));
  bool vec = inner % VW == 0 && aligned(out->data, out->offset);
  for (int k = 0; k < prog.n_in; ++k) {
    int64_t st[kMaxDims];
    if (!broadcast_strides(&in[k], out->shape, nd, st)) return Error{};
    const int64_t is = inner == 1 ? 0 : st[nd - 1];
    if (is != 0 && is != 1) return Error{};
    // the leading dimensions must step as one row index: st[i] = rs * (rows after i)
    int64_t rs = 0, after = 1;
    bool have = false;
    for (int i = nd - 2; i >= 0; --i) {
      if (out->shape[i] == 1) continue;
      if (!have) {
        rs = st[i];
        have = true;
      } else if (st[i] != rs * after) {
        return Error{};
      }
      after *= out->shape[i];
    }
    d.in[k] = in[k].data;
    d.off[k] = in[k].offset;
    d.rs[k] = rs;
    d.unit[k] = is == 1 ? 1 : 0;
    d.stream[k] = (rs != 0 || rows == 1) ? 1 : 0;
    if (is == 1) vec = vec && rs % VW == 0 && aligned(in[k].data, in[k].offset);
  }
  for (int k = prog.n_in; k < 3; ++k) d.in[k] = in[0].data;
  d.out = out->data;
  d.out_off = out->offset;
  d.rows_out = rows_out ? rows_out->data : nullptr;
  d.rows_off = rows_out ? rows_out->offset : 0;
  d.rows = (uint32_t)rows;
  d.inner = (uint32_t)inner;
  *taken = true;
  switch (dt) {
    case TRS_F32: return launch_row_sums<float>(prog, d, vec, total, stream);
    case TRS_F64: return launch_row_sums<double>(prog, d, vec, total, stream);
    case TRS_I32: return launch_row_sums<int32_t>(prog, d, vec, total, stream);
    case TRS_I64: return launch_row_sums<int64_t>(prog, d, vec, total, stream);
  }
  return make_error(TRS_ERR_DTYPE, "unknown dtype");
}

}  // namespace trs
