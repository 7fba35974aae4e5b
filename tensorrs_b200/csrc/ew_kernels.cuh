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
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "kernels.cuh"

// Tuning knobs (the defaults are the shipped configuration):
//   TRS_STREAM_ENABLE  1: rows >= 4 KiB take the bulk-copy pipeline
//   TRS_VEC_PERSISTENT 1: the vec kernel runs a grid of resident CTAs that
//                      loop; 0: one CTA per block of work (no loop)
#ifndef TRS_STREAM_ENABLE
#define TRS_STREAM_ENABLE 1
#endif
#ifndef TRS_VEC_PERSISTENT
#define TRS_VEC_PERSISTENT 1
#endif
//   TRS_STREAM_TRANSCENDENTAL 0: programs with transcendentals take the vec
//                      kernel, whose 32 warps per SM hide their arithmetic
//                      latency better (measured: sigmoid over 64 MiB 0.50 of
//                      the HBM peak against 0.40 on the pipeline); 1: the
//                      bulk-copy pipeline
#ifndef TRS_STREAM_TRANSCENDENTAL
#define TRS_STREAM_TRANSCENDENTAL 0
#endif
//   TRS_STREAM_MIN_BYTES  tensors with fewer elements x element size than this
//                      take the vec kernel: the pipeline's set-up does not pay
//                      off on a few tiles per CTA (measured on a 4 MiB bias
//                      add: 7.1 us against 9.2 us through the pipeline)
#ifndef TRS_STREAM_MIN_BYTES
#define TRS_STREAM_MIN_BYTES (16 << 20)
#endif

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

// Streaming forms for operands touched once (evict-first in L1 and L2), so
// the broadcast operands that are reused stay cached.
template <class T, int V>
__device__ __forceinline__ VecT<T, V> load_vec_stream(const T* p) {
  VecT<T, V> r;
  if constexpr (sizeof(T) * V == 16) {
    int4 x = __ldcs(reinterpret_cast<const int4*>(p));
    memcpy(&r, &x, 16);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = __ldcs(p + i);
  }
  return r;
}

template <class T, int V>
__device__ __forceinline__ void store_vec_stream(T* p, const VecT<T, V>& r) {
  if constexpr (sizeof(T) * V == 16) {
    int4 x;
    memcpy(&x, &r, 16);
    __stcs(reinterpret_cast<int4*>(p), x);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) __stcs(p + i, r.v[i]);
  }
}

// A compile-time program over one chunk of V elements of each input: the
// sigmoid programs on f32 take the packed sigmoid two elements at a time
// (bit-identical to the scalar form), every other program goes element by
// element.
template <class T, int PROG, int V>
__device__ __forceinline__ VecT<T, V> apply_prog_vec(const EwParams& p, const VecT<T, V>& a,
                                                     const VecT<T, V>& b) {
  VecT<T, V> r;
  if constexpr (std::is_same<T, float>::value && V % 2 == 0 && (PROG == kSigmoid || PROG == kMulSigmoid)) {
#pragma unroll
    for (int i = 0; i < V; i += 2) {
      float2 x = make_float2(a.v[i], a.v[i + 1]);
      if constexpr (PROG == kMulSigmoid) x = __fmul2_rn(x, make_float2(b.v[i], b.v[i + 1]));
      const float2 s = expf32::sigmoid2(x);
      r.v[i] = s.x;
      r.v[i + 1] = s.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.v[i] = apply_prog<T, PROG>(p, a.v[i], b.v[i], T(0));
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
// threads touch consecutive addresses.  Each thread handles two chunks per
// iteration, issuing every load before any arithmetic.  Chunk indices are
// 32-bit within a launch; the host splits larger tensors into launches over
// row ranges (row0).  The kernel is templated on the input count so no
// offset of an absent operand is computed, which keeps it at <= 64
// registers and 4 CTAs (1024 threads) per SM.
template <class T, int V, int PROG, bool WRITE, bool SUM>
__global__ void __launch_bounds__(kThreads, 4)
ew_vec_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  if constexpr (SUM) pdl_launch_dependents();  // sum_finalize_kernel may be scheduled now
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int NIN = prog_inputs(PROG);
  constexpr int U = NIN == 1 ? 4 : 2;
  Acc acc[V];  // one accumulator per lane: independent add chains
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = Acc(0);
  const int nd = d.nd, j = nd - 1;
  const uint32_t n_chunks = (uint32_t)d.n_chunks;
  const uint32_t cpr = d.f_cpr.d;
  for (uint32_t base = blockIdx.x * (kThreads * U) + threadIdx.x; base < n_chunks;
       base += gridDim.x * (kThreads * U)) {
    VecT<T, V> v[U][3];
    int64_t oo[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t g = base + (uint32_t)u * kThreads;
      ok[u] = g < n_chunks;
      if (!ok[u]) g = 0;
      const uint32_t row32 = fdiv(g, d.f_cpr);
      const int64_t e = (int64_t)(g - row32 * cpr) * V;
      int64_t o[NIN + 1];
#pragma unroll
      for (int k = 0; k <= NIN; ++k) o[k] = d.off[k];
      uint32_t r = (uint32_t)d.row0 + row32;
      for (int dd = nd - 2; dd > 0; --dd) {
        const uint32_t q = fdiv(r, d.f_dim[dd]);
        const int64_t c = (int64_t)(r - q * d.f_dim[dd].d);
        r = q;
#pragma unroll
        for (int k = 0; k <= NIN; ++k) o[k] += c * d.st[k][dd];
      }
      if (nd >= 2) {
#pragma unroll
        for (int k = 0; k <= NIN; ++k) o[k] += (int64_t)r * d.st[k][0];
      }
      oo[u] = o[0] + e;
#pragma unroll
      for (int k = 0; k < NIN; ++k) {
        const T* src = static_cast<const T*>(d.in[k]) + o[k + 1];
        if (d.st[k + 1][j] == 0) {
          const T sv = __ldg(src);
#pragma unroll
          for (int i = 0; i < V; ++i) v[u][k].v[i] = sv;
        } else if (d.stream[k]) {
          v[u][k] = load_vec_stream<T, V>(src + e);
        } else {
          v[u][k] = load_vec<T, V>(src + e);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      VecT<T, V> r;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const T a = v[u][0].v[i];
        const T b = NIN >= 2 ? v[u][NIN >= 2 ? 1 : 0].v[i] : T(0);
        const T c = NIN >= 3 ? v[u][NIN >= 3 ? 2 : 0].v[i] : T(0);
        r.v[i] = apply_prog<T, PROG>(p, a, b, c);
        if (SUM && ok[u]) acc[i] = acc[i] + A::to_acc(r.v[i]);
      }
      if (WRITE && ok[u]) store_vec_stream<T, V>(static_cast<T*>(d.out) + oo[u], r);
    }
  }
  if constexpr (SUM) {
    Acc t = acc[0];
#pragma unroll
    for (int i = 1; i < V; ++i) t = t + acc[i];
    write_partial<Acc>(t, partials);
  }
}

// --------------------------------------------------------------------------
// ew_stream_kernel: the bulk-copy pipeline, warp-specialised.  Work is split
// into tiles of up to kTileBytes of one row; each CTA walks its tiles
// (t = blockIdx.x + k * gridDim.x) through a ring of `stages` shared-memory
// stages.  Warp 0 is the producer: per tile it waits until the stage is free
// (the stage's `empty` mbarrier), stores the tile's per-row scalar operands
// into the stage, arms the stage's `full` mbarrier with the byte count and
// issues one cp.async.bulk per unit-stride input.  Warps 1..8 consume: wait on
// `full`, combine the tile from shared memory, stream the result out, and
// release the stage with one arrive per warp on `empty`.  No CTA-wide barrier
// runs inside the loop, and up to `stages` tiles are in flight per CTA.
constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = 32 * (1 + kConsumerWarps);
constexpr int kTileBytes = 16384;
constexpr int kStageBudget = 100 * 1024;  // shared memory per CTA: two CTAs per SM

__host__ __device__ constexpr int stream_stage_bytes(int nb) { return nb * kTileBytes; }
__host__ __device__ constexpr int stream_stages(int nb) {
  return kStageBudget / stream_stage_bytes(nb) > 8 ? 8 : kStageBudget / stream_stage_bytes(nb);
}

template <class T, int NIN>
__device__ __forceinline__ void stream_tile_geometry(const EwDev& d, uint32_t t, int64_t* off,
                                                     int64_t& col0, uint32_t& len) {
  constexpr int TILE = kTileBytes / (int)sizeof(T);
  const uint32_t row32 = fdiv(t, d.f_tpr);
  col0 = (int64_t)(t - row32 * d.f_tpr.d) * TILE;
  const int64_t rem = d.inner - col0;
  len = (uint32_t)(rem < TILE ? rem : TILE);
#pragma unroll
  for (int k = 0; k <= NIN; ++k) off[k] = d.off[k];
  uint32_t r = (uint32_t)d.row0 + row32;
  for (int dd = d.nd - 2; dd > 0; --dd) {
    const uint32_t q = fdiv(r, d.f_dim[dd]);
    const int64_t c = (int64_t)(r - q * d.f_dim[dd].d);
    r = q;
#pragma unroll
    for (int k = 0; k <= NIN; ++k) off[k] += c * d.st[k][dd];
  }
  if (d.nd >= 2) {
#pragma unroll
    for (int k = 0; k <= NIN; ++k) off[k] += (int64_t)r * d.st[k][0];
  }
}

template <class T, int PROG, int NB, bool WRITE, bool SUM>
__global__ void __launch_bounds__(kStreamThreads)
ew_stream_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  if constexpr (SUM) pdl_launch_dependents();  // sum_finalize_kernel may be scheduled now
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int NIN = prog_inputs(PROG);
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int S = stream_stages(NB);
  constexpr int SB = stream_stage_bytes(NB);
  extern __shared__ __align__(128) unsigned char smem[];
  // stage s: NB tiles; after the stages, the barriers
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * SB);
  uint64_t* empty = full + S;
  __shared__ Acc red[32];
  const int j = d.nd - 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n_tiles = (uint32_t)d.n_tiles_s;
  const uint32_t first = blockIdx.x, stride = gridDim.x;
  const uint32_t my_tiles = first < n_tiles ? (n_tiles - first + stride - 1) / stride : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  uint32_t issued = 0;  // producer: tiles whose copies were issued
  Acc acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = Acc(0);

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      for (uint32_t k = 0; k < my_tiles; ++k) {
        const int s = (int)(k % S);
        if (k >= (uint32_t)S && !mbar_wait(&empty[s], ((k / S) - 1) & 1u)) {
          failed = true;
          break;
        }
        fence_proxy_async();
        int64_t off[NIN + 1];
        int64_t col0;
        uint32_t len;
        stream_tile_geometry<T, NIN>(d, first + k * stride, off, col0, len);
        unsigned char* stage = smem + s * SB;
        const uint32_t bytes = len * (uint32_t)sizeof(T);
        mbar_arrive_expect_tx(&full[s], bytes * NB);
#pragma unroll
        for (int kk = 0; kk < NIN; ++kk) {
          const int slot = d.bulk_slot[kk];
          if (slot >= 0)
            bulk_g2s(stage + slot * kTileBytes, static_cast<const T*>(d.in[kk]) + off[kk + 1] + col0, bytes,
                     &full[s]);
        }
        issued = k + 1;
      }
      if (failed) atomicOr(d.err, kAsyncWaitTimeout);
    }
  } else {
    // ---- consumers ----
    const int ct = threadIdx.x - 32;  // 0 .. 32*kConsumerWarps-1
    for (uint32_t k = 0; k < my_tiles; ++k) {
      const int s = (int)(k % S);
      // geometry and the per-row scalar operands first, so their latency
      // overlaps the wait for the tile
      int64_t off[NIN + 1];
      int64_t col0;
      uint32_t len;
      stream_tile_geometry<T, NIN>(d, first + k * stride, off, col0, len);
      T scalars[3];
#pragma unroll
      for (int kk = 0; kk < NIN; ++kk)
        scalars[kk] = d.bulk_slot[kk] < 0 ? __ldg(static_cast<const T*>(d.in[kk]) + off[kk + 1]) : T(0);
      // the warp leaves together, so the __syncwarp below never waits on a
      // lane that gave up
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (k / S) & 1u))) {
        failed = true;
        break;
      }
      const unsigned char* stage = smem + s * SB;
      const uint32_t chunks = len / V;
      // the first chunk of each thread rotates by three warps per tile, so
      // the leftover chunks of a tile that does not divide evenly fall on a
      // different warp each time (a warp that finishes early moves on)
      constexpr uint32_t kC = 32 * kConsumerWarps;
      const uint32_t c0 = ((uint32_t)ct + kC - (k * 96u) % kC) % kC;
#pragma unroll 4
      for (uint32_t c = c0; c < chunks; c += kC) {
        VecT<T, V> in[3];
#pragma unroll
        for (int kk = 0; kk < NIN; ++kk) {
          const int slot = d.bulk_slot[kk];
          if (slot >= 0) {
            in[kk] = *reinterpret_cast<const VecT<T, V>*>(stage + slot * kTileBytes + c * 16);
          } else {
            const T sv = scalars[kk];
#pragma unroll
            for (int i = 0; i < V; ++i) in[kk].v[i] = sv;
          }
        }
        VecT<T, V> r;
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const T a = in[0].v[i];
          const T b = NIN >= 2 ? in[NIN >= 2 ? 1 : 0].v[i] : T(0);
          const T cc = NIN >= 3 ? in[NIN >= 3 ? 2 : 0].v[i] : T(0);
          r.v[i] = apply_prog<T, PROG>(p, a, b, cc);
          if (SUM) acc[i] = acc[i] + A::to_acc(r.v[i]);
        }
        if (WRITE) store_vec_stream<T, V>(static_cast<T*>(d.out) + off[0] + col0 + (int64_t)c * V, r);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (failed && lane == 0) atomicOr(d.err, kAsyncWaitTimeout);
  }
  // Before the CTA exits every copy it issued must have landed: the consumers
  // waited on every tile's `full` barrier unless they gave up, in which case
  // the producer drains the stages still in flight (bounded).
  const bool any_failed = __syncthreads_or(failed);
  if (any_failed) {
    if (threadIdx.x == 0) {
      const uint32_t start = issued > (uint32_t)S ? issued - S : 0;
      for (uint32_t k = start; k < issued; ++k) mbar_wait(&full[k % S], (k / S) & 1u);
    }
    __syncthreads();
    return;
  }
  if constexpr (SUM) {
    Acc t = acc[0];
#pragma unroll
    for (int i = 1; i < V; ++i) t = t + acc[i];
    t = block_sum<Acc>(t, red);
    if (threadIdx.x == 0) partials[blockIdx.x] = t;
  }
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
  if constexpr (SUM) pdl_launch_dependents();  // sum_finalize_kernel may be scheduled now
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
// ew_tr_kernel: the same layouts as ew_tile_kernel (an input running along
// another dimension i than the output's unit-stride dimension j, such as B^T)
// when every row start is 16-byte aligned.  Tiles are TS x TS elements
// (TS = 256 bytes: 64 f32 / 32 f64).  Each thread first issues all of its
// loads of a tile: transposed inputs go from global to shared memory with
// 16-byte cp.async (their rows are the tile's columns), the other inputs into
// registers with 16-byte loads in the output's layout (or one scalar per row
// when constant along j).  After one barrier each thread reads its transposed
// values down the shared columns, applies the compile-time program and
// stores 16 bytes of output.  The 16-byte chunks of a shared row are
// XOR-swizzled by the row's chunk group, which keeps both the cp.async writes
// and the column reads at most two-way bank conflicted.  Tile indices are
// decoded with 32-bit fast division when they fit, and interior tiles skip
// the bounds checks.  (Staging every input in shared memory with the next
// tile's copies in flight measured slower: the extra shared-memory traffic
// and instructions outweighed the overlap.)

// Shared-memory tile of input k: from the launch descriptor (TM < 0), or
// known at compile time from the mask TM of transposed inputs (bit k set: input
// k is transposed; its tile follows those of the lower transposed inputs).
constexpr int popc_c(int x) { return x ? (x & 1) + popc_c(x >> 1) : 0; }
template <int TM>
__device__ __forceinline__ int tr_slot(const EwDev& d, int k) {
  if constexpr (TM < 0) return d.tslot[k];
  else return ((TM >> k) & 1) ? popc_c(TM & ((1 << k) - 1)) : -1;
}

// The sigmoid epilogue's long arithmetic phase overlaps other CTAs' loads:
// its kernels are held to 64 registers so four CTAs fit on an SM.
template <class T, int PROG, bool WRITE, bool SUM, int TM = -1>
__global__ void __launch_bounds__(kThreads, PROG == kMulSigmoid ? 4 : 3)
ew_tr_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  if constexpr (SUM) pdl_launch_dependents();  // sum_finalize_kernel may be scheduled now
  using A = Arith<T>;
  using Acc = typename A::Acc;
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int TS = 256 / (int)sizeof(T);
  constexpr int CPR = TS / V;                 // 16-byte chunks per tile row
  constexpr int VPT = TS * CPR / kThreads;    // chunks per thread per input
  constexpr int NIN = prog_inputs(PROG);
  extern __shared__ __align__(128) unsigned char tsm[];
  Acc acc = Acc(0);
  const int j = d.nd - 1, ti = d.ti;
  const int64_t Ni = d.shape[ti], Nj = d.shape[j];
  const T* ins[3] = {static_cast<const T*>(d.in[0]), static_cast<const T*>(d.in[1]),
                     static_cast<const T*>(d.in[2])};
  T* out = static_cast<T*>(d.out);
  for (uint64_t t = blockIdx.x; t < d.n_tiles; t += gridDim.x) {
    int64_t i0, j0;
    int64_t o[kMaxOperands];
#pragma unroll
    for (int k = 0; k < kMaxOperands; ++k) o[k] = d.off[k];
    if (d.tile32) {  // 32-bit decode by fast division
      const uint32_t t32 = (uint32_t)t;
      const uint32_t rest = fdiv(t32, d.f_tj);
      j0 = (int64_t)(t32 - rest * d.f_tj.d) * TS;
      uint32_t b = fdiv(rest, d.f_ti);
      i0 = (int64_t)(rest - b * d.f_ti.d) * TS;
      for (int q = d.n_batch - 1; q >= 0; --q) {
        const int dd = d.batch_dim[q];
        const uint32_t nb = fdiv(b, d.f_dim[dd]);
        const int64_t c = (int64_t)(b - nb * d.f_dim[dd].d);
        b = nb;
#pragma unroll
        for (int k = 0; k < kMaxOperands; ++k) o[k] += c * d.st[k][dd];
      }
    } else {
      uint64_t rest = t / d.tiles_j;
      j0 = (int64_t)(t - rest * d.tiles_j) * TS;
      uint64_t b = rest / d.tiles_i;
      i0 = (int64_t)(rest - b * d.tiles_i) * TS;
      for (int q = d.n_batch - 1; q >= 0; --q) {
        const int dd = d.batch_dim[q];
        const uint64_t nb = b / (uint64_t)d.shape[dd];
        const int64_t c = (int64_t)(b - nb * (uint64_t)d.shape[dd]);
        b = nb;
#pragma unroll
        for (int k = 0; k < kMaxOperands; ++k) o[k] += c * d.st[k][dd];
      }
    }
    const bool full = i0 + TS <= Ni && j0 + TS <= Nj;  // interior: no bounds checks
    // 1. transposed inputs: global -> shared, tile row = j offset
#pragma unroll
    for (int k = 0; k < NIN; ++k) {
      const int slot = tr_slot<TM>(d, k);
      if (slot < 0) continue;
      unsigned char* base = tsm + slot * (TS * 256);
      const int64_t sj = d.st[k + 1][j];
#pragma unroll
      for (int r = 0; r < VPT; ++r) {
        const int v = threadIdx.x + r * kThreads;
        const int row = v / CPR, ch = v % CPR;
        const int64_t jj = j0 + row, ii = i0 + (int64_t)ch * V;
        if (full || (jj < Nj && ii < Ni))
          cp_async16(base + row * 256 + ((ch ^ ((row / V) & 15)) * 16), ins[k] + o[k + 1] + ii + jj * sj);
      }
    }
    cp_async_commit();
    // 2. the other inputs: registers, in the output's layout (row = i offset)
    VecT<T, V> rv[NIN][VPT];
#pragma unroll
    for (int k = 0; k < NIN; ++k) {
      if (tr_slot<TM>(d, k) >= 0) continue;
      const int64_t sj = d.st[k + 1][j], si = d.st[k + 1][ti];
#pragma unroll
      for (int r = 0; r < VPT; ++r) {
        const int v = threadIdx.x + r * kThreads;
        const int row = v / CPR, ch = v % CPR;
        const int64_t ii = i0 + row, jj = j0 + (int64_t)ch * V;
        if (full || (ii < Ni && jj < Nj)) {
          const T* src = ins[k] + o[k + 1] + ii * si + jj * sj;
          if (sj == 1) {
            rv[k][r] = load_vec<T, V>(src);
          } else {
            const T sc = __ldg(src);
#pragma unroll
            for (int q = 0; q < V; ++q) rv[k][r].v[q] = sc;
          }
        }
      }
    }
    cp_async_wait_all();
    __syncthreads();
    // 3. combine, store 16 bytes per chunk
#pragma unroll
    for (int r = 0; r < VPT; ++r) {
      const int v = threadIdx.x + r * kThreads;
      const int row = v / CPR, ch = v % CPR;
      const int64_t ii = i0 + row, jj = j0 + (int64_t)ch * V;
      if (full || (ii < Ni && jj < Nj)) {
        VecT<T, V> res;
#pragma unroll
        for (int q = 0; q < V; ++q) {
          T a[3] = {T(0), T(0), T(0)};
#pragma unroll
          for (int k = 0; k < NIN; ++k) {
            const int slot = tr_slot<TM>(d, k);
            if (slot >= 0) {
              const int jr = ch * V + q;  // the transposed input's tile row
              a[k] = *reinterpret_cast<const T*>(tsm + slot * (TS * 256) + jr * 256 +
                                                 (((row / V) ^ (ch & 15)) * 16) + (row % V) * (int)sizeof(T));
            } else {
              a[k] = rv[k][r].v[q];
            }
          }
          res.v[q] = apply_prog<T, PROG>(p, a[0], a[1], a[2]);
          if constexpr (SUM) acc = acc + A::to_acc(res.v[q]);
        }
        if constexpr (WRITE) store_vec_stream<T, V>(out + o[0] + ii * d.st[0][ti] + jj, res);
      }
    }
    __syncthreads();
  }
  if constexpr (SUM) write_partial<Acc>(acc, partials);
}

// ew_tr2d_kernel: ew_tr_kernel for the fused multiply programs on two
// folded dimensions (i = 0, j = 1), with the mask TM of transposed inputs
// fixed at compile time and every offset within 2^31 elements of its
// operand's base: the tile's offsets are 32-bit, and each thread's chunk
// coordinates inside a tile are computed once.  Software-pipelined: the
// copies of the CTA's next tile (into the second of two shared buffers) and
// its register loads are issued before the current tile is combined.
template <class T, int PROG, int TM>
__global__ void __launch_bounds__(kThreads, 3)
ew_tr2d_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc*) {
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int TS = 256 / (int)sizeof(T);
  constexpr int CPR = TS / V;
  constexpr int VPT = TS * CPR / kThreads;
  constexpr int NIN = 2;
  constexpr int NT = popc_c(TM);          // transposed inputs (shared tiles)
  constexpr int kBuf = NT * TS * 256;     // bytes of one buffer
  extern __shared__ __align__(128) unsigned char tsm[];
  const int32_t Ni = (int32_t)d.shape[0], Nj = (int32_t)d.shape[1];
  const T* ins[2] = {static_cast<const T*>(d.in[0]) + d.off[1], static_cast<const T*>(d.in[1]) + d.off[2]};
  T* out = static_cast<T*>(d.out) + d.off[0];
  const int32_t si[2] = {(int32_t)d.st[1][0], (int32_t)d.st[2][0]};
  const int32_t sj[2] = {(int32_t)d.st[1][1], (int32_t)d.st[2][1]};
  const int32_t so = (int32_t)d.st[0][0];
  int row[VPT], ch[VPT];
#pragma unroll
  for (int r = 0; r < VPT; ++r) {
    const int v = threadIdx.x + r * kThreads;
    row[r] = v / CPR;
    ch[r] = v % CPR;
  }
  const uint32_t n_tiles = (uint32_t)d.n_tiles;
  auto origin = [&](uint32_t t, int32_t* i0, int32_t* j0) {
    const uint32_t ti = fdiv(t, d.f_tj);
    *j0 = (int32_t)(t - ti * d.f_tj.d) * TS;
    *i0 = (int32_t)ti * TS;
  };
  // the tile's transposed inputs -> buffer `buf`, its other inputs -> rv
  auto fetch = [&](int32_t i0, int32_t j0, int buf, VecT<T, V> (&rv)[NIN][VPT]) {
    const bool full = i0 + TS <= Ni && j0 + TS <= Nj;
#pragma unroll
    for (int k = 0; k < NIN; ++k) {
      if ((TM >> k) & 1) {
        unsigned char* base = tsm + buf * kBuf + popc_c(TM & ((1 << k) - 1)) * (TS * 256);
#pragma unroll
        for (int r = 0; r < VPT; ++r) {
          const int32_t jj = j0 + row[r], ii = i0 + ch[r] * V;
          if (full || (jj < Nj && ii < Ni))
            cp_async16(base + row[r] * 256 + ((ch[r] ^ ((row[r] / V) & 15)) * 16), ins[k] + ii + jj * sj[k]);
        }
      } else {
#pragma unroll
        for (int r = 0; r < VPT; ++r) {
          const int32_t ii = i0 + row[r], jj = j0 + ch[r] * V;
          if (full || (ii < Ni && jj < Nj)) rv[k][r] = load_vec<T, V>(ins[k] + ii * si[k] + jj);
        }
      }
    }
  };
  VecT<T, V> rcur[NIN][VPT], rnxt[NIN][VPT];
  uint32_t t = blockIdx.x;
  int32_t i0 = 0, j0 = 0;
  if (t < n_tiles) {
    origin(t, &i0, &j0);
    fetch(i0, j0, 0, rcur);
  }
  cp_async_commit();
  int buf = 0;
  for (; t < n_tiles; t += gridDim.x, buf ^= 1) {
    const uint32_t tn = t + gridDim.x;
    int32_t ni0 = 0, nj0 = 0;
    if (tn < n_tiles) {
      origin(tn, &ni0, &nj0);
      fetch(ni0, nj0, buf ^ 1, rnxt);
    }
    cp_async_commit();
    cp_async_wait_prev();  // this tile's copies (the next tile's stay in flight)
    __syncthreads();
    const bool full = i0 + TS <= Ni && j0 + TS <= Nj;
#pragma unroll
    for (int r = 0; r < VPT; ++r) {
      const int32_t ii = i0 + row[r], jj = j0 + ch[r] * V;
      if (full || (ii < Ni && jj < Nj)) {
        VecT<T, V> a[2];
#pragma unroll
        for (int q = 0; q < V; ++q) {
#pragma unroll
          for (int k = 0; k < NIN; ++k) {
            if ((TM >> k) & 1) {
              a[k].v[q] = *reinterpret_cast<const T*>(tsm + buf * kBuf + popc_c(TM & ((1 << k) - 1)) * (TS * 256) +
                                                      (ch[r] * V + q) * 256 + (((row[r] / V) ^ (ch[r] & 15)) * 16) +
                                                      (row[r] % V) * (int)sizeof(T));
            } else {
              a[k].v[q] = rcur[k][r].v[q];
            }
          }
        }
        store_vec_stream<T, V>(out + ii * so + jj, apply_prog_vec<T, PROG, V>(p, a[0], a[NIN - 1]));
      }
    }
    __syncthreads();  // the next iteration's copies go into this buffer
#pragma unroll
    for (int k = 0; k < NIN; ++k)
#pragma unroll
      for (int r = 0; r < VPT; ++r) rcur[k][r] = rnxt[k][r];
    i0 = ni0;
    j0 = nj0;
  }
  cp_async_wait_all();
}

// ew_flat1_kernel: a one-input map with a transcendental program (sigmoid,
// tanh) over a contiguous 1-D range of fewer than 2^31 16-byte chunks: the
// vector kernel's data flow (four chunks per thread loaded, then mapped)
// with plain chunk indices instead of the strided row decode; held to 40
// registers so six CTAs fit on an SM (more warps to cover the loads).
template <class T, int PROG>
__global__ void __launch_bounds__(kThreads, 6)
ew_flat1_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc*) {
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int U = 4;
  const T* in = static_cast<const T*>(d.in[0]) + d.off[1];
  T* out = static_cast<T*>(d.out) + d.off[0];
  const uint32_t n = (uint32_t)d.n_chunks;
  const bool stream = d.stream[0] != 0;
  for (uint32_t base = blockIdx.x * (kThreads * U) + threadIdx.x; base < n; base += gridDim.x * (kThreads * U)) {
    VecT<T, V> v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t g = base + (uint32_t)u * kThreads;
      if (g < n) v[u] = stream ? load_vec_stream<T, V>(in + (size_t)g * V) : load_vec<T, V>(in + (size_t)g * V);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t g = base + (uint32_t)u * kThreads;
      if (g < n) {
        store_vec_stream<T, V>(out + (size_t)g * V, apply_prog_vec<T, PROG, V>(p, v[u], v[u]));
      }
    }
  }
}

// --------------------------------------------------------------------------
// ew_generic_kernel: one element per thread, every operand's offset decoded
// from the row-major element index.
template <class T, bool WRITE, bool SUM>
__global__ void __launch_bounds__(kThreads)
ew_generic_kernel(const EwDev d, const EwParams p, typename Arith<T>::Acc* partials) {
  if constexpr (SUM) pdl_launch_dependents();  // sum_finalize_kernel may be scheduled now
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
  pdl_wait();  // the partials of the kernel before it
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

// sum_finalize_kernel for a tensor split on axis 0 across ranks: the
// partials of this rank fold in a fixed order as above, then the ranks
// exchange their accumulators over NVLink peer memory instead of through a
// collective library call -- thread r stores this rank's accumulator and the
// call's sequence number into rank r's slot buffer (release: the value
// before the number), threads r < world wait for rank r's number to reach
// this call's in this rank's own buffer (acquire), and thread 0 adds the
// world accumulators in rank order and rounds once.  Every rank adds the same
// values in the same order, so all ranks get the same result.  The slot set
// alternates with the parity of the sequence number: a rank can be at most
// one call ahead of a peer still reading (it cannot finish a call before
// every peer has written that call's value), so the value a reader needs is
// never overwritten.  Each wait polls at most kPeerPolls times, sleeping in
// between (about 2 s in all); a wait that runs out sets kAsyncPeerTimeout in
// the async-error word and the result is NaN (floats) or 0 (integers).
constexpr unsigned kPeerPolls = 1u << 23;

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <class Acc>
__device__ __forceinline__ unsigned long long acc_bits(Acc a) {
  if constexpr (sizeof(Acc) == 8) {
    unsigned long long u;
    memcpy(&u, &a, 8);
    return u;
  } else {
    return (unsigned long long)a;
  }
}
template <class Acc>
__device__ __forceinline__ Acc acc_from_bits(unsigned long long u) {
  if constexpr (sizeof(Acc) == 8) {
    Acc a;
    memcpy(&a, &u, 8);
    return a;
  } else {
    return (Acc)u;
  }
}

template <class T>
__global__ void __launch_bounds__(1024)
sum_exchange_kernel(const typename Arith<T>::Acc* partials, int n, T* out, const PeerExchange x) {
  pdl_wait();  // the partials of the kernel before it
  using Acc = typename Arith<T>::Acc;
  __shared__ Acc red[32];
  __shared__ unsigned long long vals[kMaxExchangeRanks];
  __shared__ int failed;
  Acc s = Acc(0);
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = s + partials[i];
  s = block_sum<Acc>(s, red);
  if (threadIdx.x == 0) {
    red[0] = s;
    failed = 0;
  }
  __syncthreads();
  const int t = threadIdx.x;
  const unsigned long long set = (x.seq & 1ull) * (unsigned long long)x.world;
  if (t < x.world) {
    unsigned long long* slot = x.peers[t] + 2 * (set + (unsigned long long)x.rank);
    st_relaxed_sys(slot, acc_bits<Acc>(red[0]));
    st_release_sys(slot + 1, x.seq);
  }
  if (t < x.world) {
    const unsigned long long* mine = x.peers[x.rank] + 2 * (set + (unsigned long long)t);
    unsigned polls = 0;
    while (ld_acquire_sys(mine + 1) < x.seq) {
      if (++polls > kPeerPolls) {
        atomicOr(&failed, 1);
        break;
      }
      __nanosleep(256);
    }
    vals[t] = ld_relaxed_sys(mine);
  }
  __syncthreads();
  if (t == 0) {
    if (failed) {
      if (x.err) atomicOr(x.err, kAsyncPeerTimeout);
      if (out) {
        if constexpr (IsFloat<T>::value)
          *out = Arith<T>::from_acc(Acc(NAN));
        else
          *out = T(0);
      }
    } else {
      Acc total = Acc(0);
      for (int r = 0; r < x.world; ++r) total = total + acc_from_bits<Acc>(vals[r]);
      if (out) *out = Arith<T>::from_acc(total);
    }
  }
}

// Blocks per SM a kernel can keep resident (cached per kernel).
inline int resident_blocks(const void* kernel, int threads) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(kernel);
  if (it != cache.end()) return it->second;
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0) != cudaSuccess || b < 1) {
    cudaGetLastError();
    b = 1;
  }
  cache[kernel] = b;
  return b;
}

template <class K>
int resident_blocks(K kernel, int threads) {
  return resident_blocks((const void*)kernel, threads);
}

using trs::allow_smem;
using trs::resident_blocks_smem;

// Which (write, sum) forms a program code is instantiated with: every code
// writes; sums are instantiated for the runtime codes, Y = A & B + c, and
// the plain sum of one input.
template <class T, int PROG>
const void* pick_vec_ws(int vw, bool write, bool want_sum) {
  constexpr bool with_sum = prog_is_runtime(PROG) || PROG == kMulAdd;
  constexpr bool sum_only = prog_is_runtime(PROG) || PROG == kPack;
  constexpr int VW = 16 / (int)sizeof(T);
  if (vw == VW) {
    if (write && !want_sum) return (const void*)ew_vec_kernel<T, VW, PROG, true, false>;
    if constexpr (with_sum)
      if (write && want_sum) return (const void*)ew_vec_kernel<T, VW, PROG, true, true>;
    if constexpr (sum_only)
      if (!write && want_sum) return (const void*)ew_vec_kernel<T, VW, PROG, false, true>;
    return nullptr;
  }
  if constexpr (prog_is_runtime(PROG)) {
    if (write && !want_sum) return (const void*)ew_vec_kernel<T, 1, PROG, true, false>;
    if (write && want_sum) return (const void*)ew_vec_kernel<T, 1, PROG, true, true>;
    return (const void*)ew_vec_kernel<T, 1, PROG, false, true>;
  }
  return nullptr;
}

template <class T, int PROG, int NB>
const void* pick_stream_ws(bool write, bool want_sum) {
  constexpr bool with_sum = prog_is_runtime(PROG) || PROG == kMulAdd;
  constexpr bool sum_only = prog_is_runtime(PROG) || PROG == kPack;
  if (write && !want_sum) return (const void*)ew_stream_kernel<T, PROG, NB, true, false>;
  if constexpr (with_sum)
    if (write && want_sum) return (const void*)ew_stream_kernel<T, PROG, NB, true, true>;
  if constexpr (sum_only)
    if (!write && want_sum) return (const void*)ew_stream_kernel<T, PROG, NB, false, true>;
  return nullptr;
}

// Bulk-input counts instantiated per code: the runtime codes take every
// count, the specialised ones the layouts of their workloads.
template <class T, int PROG>
const void* pick_stream_nb(int nb, bool write, bool want_sum) {
  constexpr int NIN = prog_inputs(PROG);
  if constexpr (prog_is_runtime(PROG)) {
    if (nb == 1) return pick_stream_ws<T, PROG, 1>(write, want_sum);
    if constexpr (NIN >= 2)
      if (nb == 2) return pick_stream_ws<T, PROG, 2>(write, want_sum);
    if constexpr (NIN >= 3)
      if (nb == 3) return pick_stream_ws<T, PROG, 3>(write, want_sum);
    return nullptr;
  } else {
    if (nb == NIN) return pick_stream_ws<T, PROG, NIN>(write, want_sum);
    if constexpr (PROG == kMulAddRelu || NIN == 2)
      if (nb == 1) return pick_stream_ws<T, PROG, 1>(write, want_sum);
    return nullptr;
  }
}

template <class T, int PROG>
const void* pick_tr_ws(bool write, bool want_sum, int tmask) {
  if (write && !want_sum) {
    // the fused programs of the transposed layouts get kernels specialised on
    // which inputs are transposed
    if constexpr (PROG == kMul || PROG == kMulSigmoid) {
      switch (tmask) {
        case 1: return (const void*)ew_tr_kernel<T, PROG, true, false, 1>;
        case 2: return (const void*)ew_tr_kernel<T, PROG, true, false, 2>;
        case 3: return (const void*)ew_tr_kernel<T, PROG, true, false, 3>;
      }
    }
    return (const void*)ew_tr_kernel<T, PROG, true, false>;
  }
  if constexpr (prog_is_runtime(PROG)) {
    if (write && want_sum) return (const void*)ew_tr_kernel<T, PROG, true, true>;
    return (const void*)ew_tr_kernel<T, PROG, false, true>;
  }
  return nullptr;
}

template <class T, int PROG>
const void* pick_tr_code(bool write, bool want_sum, int tmask) {
  if constexpr (prog_is_runtime(PROG) || PROG == kPack || PROG == kAdd || PROG == kSub || PROG == kMul ||
                PROG == kMulSigmoid)
    return pick_tr_ws<T, PROG>(write, want_sum, tmask);
  return nullptr;
}

template <class T, class F>
const void* by_code(int code, F f) {
  switch (code) {
    case kRunSimple1: return f(std::integral_constant<int, kRunSimple1>{});
    case kRunSimple2: return f(std::integral_constant<int, kRunSimple2>{});
    case kRunSimple3: return f(std::integral_constant<int, kRunSimple3>{});
    case kPack: return f(std::integral_constant<int, kPack>{});
    case kAdd: return f(std::integral_constant<int, kAdd>{});
    case kSub: return f(std::integral_constant<int, kSub>{});
    case kMul: return f(std::integral_constant<int, kMul>{});
    case kDiv: return f(std::integral_constant<int, kDiv>{});
    case kMulAdd: return f(std::integral_constant<int, kMulAdd>{});
  }
  if constexpr (IsFloat<T>::value) {
    switch (code) {
      case kRunFull1: return f(std::integral_constant<int, kRunFull1>{});
      case kRunFull2: return f(std::integral_constant<int, kRunFull2>{});
      case kRunFull3: return f(std::integral_constant<int, kRunFull3>{});
      case kMulAddRelu: return f(std::integral_constant<int, kMulAddRelu>{});
      case kMulSigmoid: return f(std::integral_constant<int, kMulSigmoid>{});
      case kSigmoid: return f(std::integral_constant<int, kSigmoid>{});
      case kTanh: return f(std::integral_constant<int, kTanh>{});
      case kRelu: return f(std::integral_constant<int, kRelu>{});
    }
  }
  return nullptr;
}

// The vec kernel for a program code, falling back to the runtime code of the
// same input count when the specialised form is not instantiated.
template <class T>
const void* pick_vec(int code, int fallback, int vw, bool write, bool want_sum) {
  const void* k = by_code<T>(code, [&](auto c) { return pick_vec_ws<T, decltype(c)::value>(vw, write, want_sum); });
  if (!k) k = by_code<T>(fallback, [&](auto c) { return pick_vec_ws<T, decltype(c)::value>(vw, write, want_sum); });
  return k;
}

template <class T>
const void* pick_flat1(int code) {
  if constexpr (IsFloat<T>::value) {
    if (code == kSigmoid) return (const void*)ew_flat1_kernel<T, kSigmoid>;
    if (code == kTanh) return (const void*)ew_flat1_kernel<T, kTanh>;
  }
  return nullptr;
}

template <class T>
const void* pick_tr(int code, int fallback, bool write, bool want_sum, int tmask) {
  const void* k =
      by_code<T>(code, [&](auto c) { return pick_tr_code<T, decltype(c)::value>(write, want_sum, tmask); });
  if (!k)
    k = by_code<T>(fallback, [&](auto c) { return pick_tr_code<T, decltype(c)::value>(write, want_sum, -1); });
  return k;
}

template <class T>
const void* pick_stream(int code, int fallback, int nb, bool write, bool want_sum) {
  const void* k = by_code<T>(code, [&](auto c) { return pick_stream_nb<T, decltype(c)::value>(nb, write, want_sum); });
  if (!k) k = by_code<T>(fallback, [&](auto c) { return pick_stream_nb<T, decltype(c)::value>(nb, write, want_sum); });
  return k;
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
  p.e_const = std::is_same<T, float>::value ? std::log2((double)2.7182817f) : 2.718281828459045;
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

  // grid and kernel choice; the vec kernel may take several launches (row
  // ranges of fewer than 2^31 chunks each)
  const void* kernel = nullptr;
  int blocks = 1;
  int n_launch = 1;
  uint64_t rows_per_launch = 0, total_rows = 0, stream_tpr = 0;
  int stream_smem = 0;
  constexpr int kEwStream = 100;  // internal variant: the bulk-copy pipeline
  constexpr int kEwTr = 101;      // internal variant: the vectorised tile kernel
  auto grid_for = [&](const void* k, int per_sm, uint64_t work_blocks) {
    uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
    uint64_t b = work_blocks < cap ? work_blocks : cap;
    kernel = k;
    blocks = (int)(b < 1 ? 1 : b);
  };
  int variant = pr.choice.variant;
  if (variant == kEwVec && f.n > 0) {
    const int V = pr.choice.vec;
    const int j = f.nd - 1;
    const uint64_t cpr = (uint64_t)f.shape[j] / V;
    total_rows = (uint64_t)f.n / (uint64_t)f.shape[j];
    bool fits = cpr > 0 && cpr < (1ull << 31) && total_rows < (1ull << 32);
    for (int i = 0; i < f.nd; ++i)
      if ((uint64_t)f.shape[i] >= (1ull << 32)) fits = false;
    if (!fits) variant = kEwGeneric;  // index spaces beyond 32 bits take the generic kernel
    // operands read once stream past the caches; broadcast ones stay cached
    int nb = 0;
    for (int k = 0; k < prog.n_in; ++k) {
      bool reused = false;
      for (int i = 0; i < f.nd; ++i)
        if (f.st[k + 1][i] == 0 && f.shape[i] > 1) reused = true;
      d.stream[k] = reused ? 0 : 1;
      // the bulk pipeline copies every input that runs along the row; inputs
      // constant along it (per-row scalars) go through the stage's scalar slots
      d.bulk_slot[k] = f.st[k + 1][j] == 1 ? nb++ : -1;
    }
    constexpr int VW = 16 / sizeof(T);
    const int code = program_code(prog, IsFloat<T>::value);
    const bool simple = is_simple_program(prog) || !IsFloat<T>::value;
    const int fallback = (simple ? kRunSimple1 : kRunFull1) + (prog.n_in - 1);
    // rows of at least 4 KiB (every unit-stride input 16-byte aligned, which
    // the vector width V == VW guarantees) take the bulk-copy pipeline
    const void* sk = nullptr;
    if (TRS_STREAM_ENABLE && fits && V == VW && nb > 0 && (uint64_t)f.shape[j] * sizeof(T) >= 4096 &&
        (uint64_t)f.n * sizeof(T) >= (uint64_t)TRS_STREAM_MIN_BYTES &&
        (TRS_STREAM_TRANSCENDENTAL || simple))
      sk = ewk::pick_stream<T>(code, fallback, nb, write, want_sum);
    int* err = sk ? async_error_word() : nullptr;
    if (sk && err) {
      variant = kEwStream;
      constexpr uint64_t TILE = ewk::kTileBytes / sizeof(T);
      const uint64_t tpr = ((uint64_t)f.shape[j] + TILE - 1) / TILE;
      d.inner = f.shape[j];
      d.err = err;
      d.f_tpr = make_fastdiv((uint32_t)tpr);
      for (int i = 0; i < f.nd; ++i) d.f_dim[i] = make_fastdiv((uint32_t)f.shape[i]);
      rows_per_launch = ((1ull << 31) - 1) / tpr;
      if (rows_per_launch > total_rows) rows_per_launch = total_rows;
      n_launch = (int)((total_rows + rows_per_launch - 1) / rows_per_launch);
      stream_smem = ewk::stream_stages(nb) * (ewk::stream_stage_bytes(nb) + 16);
      ewk::allow_smem(sk, stream_smem);
      grid_for(sk, ewk::resident_blocks_smem(sk, ewk::kStreamThreads, stream_smem), rows_per_launch * tpr);
      stream_tpr = tpr;
    } else if (fits) {
      d.vec = V;
      d.f_cpr = make_fastdiv((uint32_t)cpr);
      for (int i = 0; i < f.nd; ++i) d.f_dim[i] = make_fastdiv((uint32_t)f.shape[i]);
      rows_per_launch = ((1ull << 31) - 1) / cpr;
      if (rows_per_launch > total_rows) rows_per_launch = total_rows;
      n_launch = (int)((total_rows + rows_per_launch - 1) / rows_per_launch);
      const uint64_t chunks = rows_per_launch * cpr;
      const uint64_t per_block = (uint64_t)kThreads * (prog.n_in == 1 ? 4 : 2);
      const uint64_t wb = (chunks + per_block - 1) / per_block;
      const void* k = ewk::pick_vec<T>(V == VW ? code : fallback, fallback, V, write, want_sum);
      // a contiguous 1-D transcendental map: plain chunk indices
      if (f.nd == 1 && prog.n_in == 1 && V == VW && write && !want_sum && f.st[0][0] == 1 && f.st[1][0] == 1) {
        const void* k1 = ewk::pick_flat1<T>(code);
        if (k1) k = k1;
      }
      if (TRS_VEC_PERSISTENT) {
        grid_for(k, ewk::resident_blocks(k, kThreads), wb);
      } else {
        kernel = k;
        blocks = (int)(wb < 1 ? 1 : (wb > 0x7fffffffull ? 0x7fffffffull : wb));
      }
    }
  }
  int tr_smem = 0;
  if (variant == kEwTile && f.n > 0) {
    // the vectorised tile kernel when every row start is 16-byte aligned
    constexpr int VW = 16 / sizeof(T);
    const int j = f.nd - 1, ti = pr.choice.tile_dim;
    bool ok = f.shape[ti] % VW == 0 && f.shape[j] % VW == 0;
    auto aligned = [&](const void* base, int64_t off) {
      return ((uintptr_t)base + (uintptr_t)(off * (int64_t)sizeof(T))) % 16 == 0;
    };
    int nt = 0;
    for (int k = 0; k < prog.n_in && ok; ++k) {
      const int64_t sj = f.st[k + 1][j], si = f.st[k + 1][ti];
      d.tslot[k] = -1;
      if (sj != 0 && sj != 1) {  // transposed: unit stride along i required
        ok = si == 1 && sj % VW == 0 && aligned(in[k].data, f.off[k + 1]);
        d.tslot[k] = nt++;
      } else if (sj == 1) {
        ok = si % VW == 0 && aligned(in[k].data, f.off[k + 1]);
      }
      for (int i = 0; i < f.nd && ok; ++i)
        if (i != ti && i != j && f.st[k + 1][i] % VW) ok = false;
    }
    if (ok && write) {
      ok = f.st[0][j] == 1 && f.st[0][ti] % VW == 0 && aligned(out->data, f.off[0]);
      for (int i = 0; i < f.nd && ok; ++i)
        if (i != ti && i != j && f.st[0][i] % VW) ok = false;
    }
    const int code = program_code(prog, IsFloat<T>::value);
    const bool simple = is_simple_program(prog) || !IsFloat<T>::value;
    const int fallback = (simple ? kRunSimple1 : kRunFull1) + (prog.n_in - 1);
    int tmask = 0;  // inputs read through shared-memory tiles
    for (int k = 0; k < prog.n_in; ++k)
      if (d.tslot[k] >= 0) tmask |= 1 << k;
    const void* tk = ok && nt > 0 ? ewk::pick_tr<T>(code, fallback, write, want_sum, tmask) : nullptr;
    // two folded dimensions, a fused multiply program, 32-bit offsets: the
    // 2-D kernel
    bool two_d = tk && f.nd == 2 && ti == 0 && j == 1 && write && !want_sum && tmask >= 1 && tmask <= 3 &&
                 prog.n_in == 2 && (code == kMul || code == kMulSigmoid);
    for (int k = 0; k <= prog.n_in && two_d; ++k) {
      const uint64_t span = (uint64_t)(f.shape[0] - 1) * (uint64_t)std::llabs(f.st[k][0]) +
                            (uint64_t)(f.shape[1] - 1) * (uint64_t)std::llabs(f.st[k][1]);
      if (span >= (1ull << 31)) two_d = false;
    }
    if (two_d) {
      const void* k2 = nullptr;
      if (code == kMul) {
        k2 = tmask == 1 ? (const void*)ewk::ew_tr2d_kernel<T, kMul, 1>
             : tmask == 2 ? (const void*)ewk::ew_tr2d_kernel<T, kMul, 2>
                          : (const void*)ewk::ew_tr2d_kernel<T, kMul, 3>;
      } else {
        k2 = tmask == 1 ? (const void*)ewk::ew_tr2d_kernel<T, kMulSigmoid, 1>
             : tmask == 2 ? (const void*)ewk::ew_tr2d_kernel<T, kMulSigmoid, 2>
                          : (const void*)ewk::ew_tr2d_kernel<T, kMulSigmoid, 3>;
      }
      tk = k2;
    }
    if (tk) {
      constexpr int TS = 256 / sizeof(T);
      d.ti = ti;
      d.n_batch = 0;
      for (int i = 0; i < f.nd; ++i)
        if (i != ti && i != j) d.batch_dim[d.n_batch++] = i;
      d.tiles_i = ((uint64_t)f.shape[ti] + TS - 1) / TS;
      d.tiles_j = ((uint64_t)f.shape[j] + TS - 1) / TS;
      uint64_t nbt = 1;
      for (int q = 0; q < d.n_batch; ++q) nbt *= (uint64_t)f.shape[d.batch_dim[q]];
      d.n_tiles = d.tiles_i * d.tiles_j * nbt;
      d.tile32 = d.n_tiles < (1ull << 32) ? 1 : 0;  // always, for the 2-D kernel (offsets < 2^31)
      for (int q = 0; q < d.n_batch; ++q)
        if ((uint64_t)f.shape[d.batch_dim[q]] >= (1ull << 32)) d.tile32 = 0;
      if (d.tile32) {
        d.f_tj = make_fastdiv((uint32_t)d.tiles_j);
        d.f_ti = make_fastdiv((uint32_t)d.tiles_i);
        for (int q = 0; q < d.n_batch; ++q)
          d.f_dim[d.batch_dim[q]] = make_fastdiv((uint32_t)f.shape[d.batch_dim[q]]);
      }
      tr_smem = (two_d ? 2 : 1) * nt * TS * 256;  // the 2-D kernel double-buffers its tiles
      ewk::allow_smem(tk, tr_smem);
      grid_for(tk, ewk::resident_blocks_smem(tk, kThreads, tr_smem), d.n_tiles);
      variant = kEwTr;
    }
  }
  if (variant == kEwTile) {
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
  } else if (variant == kEwGeneric) {
    const uint64_t wb = ((uint64_t)f.n + kThreads - 1) / kThreads;
    if (write && want_sum) { auto k = ewk::ew_generic_kernel<T, true, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
    else if (write) { auto k = ewk::ew_generic_kernel<T, true, false>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
    else { auto k = ewk::ew_generic_kernel<T, false, true>; grid_for((const void*)k, ewk::resident_blocks(k, kThreads), wb); }
  }

  Scratch partials;
  Acc* part = nullptr;
  const int n_part = blocks * n_launch;
  if (want_sum && sum->partials) {
    if (sizeof(Acc) * (size_t)n_part > sum->partials_bytes)
      return make_error(TRS_ERR_ARG, "the sum needs " + std::to_string(sizeof(Acc) * (size_t)n_part) +
                                         " bytes of partials, more than the " +
                                         std::to_string(sum->partials_bytes) + " provided");
    part = static_cast<Acc*>(sum->partials);
  } else if (want_sum) {
    Error e = partials.alloc(sizeof(Acc) * (size_t)n_part, stream);
    if (!e.ok()) return e;
    part = partials.as<Acc>();
  }
  if (f.n > 0) {
    for (int l = 0; l < n_launch; ++l) {
      if (variant == kEwVec || variant == kEwStream) {
        d.row0 = (uint64_t)l * rows_per_launch;
        const uint64_t rows = total_rows - d.row0 < rows_per_launch ? total_rows - d.row0 : rows_per_launch;
        d.n_chunks = rows * d.f_cpr.d;
        d.n_tiles_s = rows * stream_tpr;
      }
      Acc* part_l = part ? part + (size_t)l * blocks : nullptr;
      void* args[] = {(void*)&d, (void*)&p, (void*)&part_l};
      const bool st = variant == kEwStream;
      const size_t dyn = st ? (size_t)stream_smem : (variant == kEwTr ? (size_t)tr_smem : 0);
      cudaError_t ce = cudaLaunchKernel(kernel, dim3(blocks), dim3(st ? ewk::kStreamThreads : kThreads), args,
                                        dyn, stream);
      if (ce != cudaSuccess) return cuda_error(ce, "element-wise kernel launch");
      Error e = check_launch("element-wise kernel");
      if (!e.ok()) return e;
    }
  } else if (want_sum) {
    cudaError_t ce = cudaMemsetAsync(part, 0, sizeof(Acc) * (size_t)n_part, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "cudaMemsetAsync");
  }
  if (want_sum) {
    T* sum_out = nullptr;
    if (sum->view) sum_out = static_cast<T*>(sum->view->data) + sum->view->offset;
    // launched with programmatic stream serialization: scheduled while the
    // element-wise kernel finishes, it waits for that grid in pdl_wait
    Acc* raw = static_cast<Acc*>(sum->raw_acc);
    const PeerExchange* xc = sum->exchange;
    void* fargs[] = {(void*)&part, (void*)&n_part, (void*)&sum_out, (void*)&raw};
    void* xargs[] = {(void*)&part, (void*)&n_part, (void*)&sum_out, (void*)xc};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t fe =
        xc ? cudaLaunchKernelExC(&cfg, (const void*)ewk::sum_exchange_kernel<T>, xargs)
           : cudaLaunchKernelExC(&cfg, (const void*)ewk::sum_finalize_kernel<T>, fargs);
    if (fe != cudaSuccess) return cuda_error(fe, "sum finalize launch");
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
