// matmul.cu -- Tensor::matmul (linalg/tensor/base.rs:896-1013) and the
// im2col pair unfold_2d / fold_2d (linalg/tensor/conv.rs:360-488).
//
// matmul keeps the reference's arithmetic: every output element is
//     acc = 0;  for k in 0 .. K-1:  acc = acc + a[i, k] * b[k, j]
// in the element type, each product and each sum rounded once (integers
// wrap), so the result is bit-identical to the reference's for every dtype.
// The order over k is what fixes the f32/f64 roundings, so every output stays
// with one thread, which walks k in order; what the kernel reorganises is
// everything around that chain:
//   * a CTA of 256 threads owns a BM x BN output tile; each thread owns a
//     TM x TN block of it (8 x 8 for 4-byte types, 8 x 4 for 8-byte ones);
//   * K advances in BK-deep slabs; the next slab of A and B is copied from
//     global to shared memory asynchronously (cp.async, zero-filled beyond
//     the matrix) while the current one is multiplied (two buffers), with
//     coalesced reads chosen by which dimension of each operand is
//     unit-stride;
//   * the arithmetic is the scalar multiply and add, rounded separately:
//     the FP32 lanes (32 per SM sub-partition per clock) bind a multiply and
//     an add per output either way, and sm_100's packed f32x2 forms, which
//     would only free issue slots, may be fused into a multiply-add by the
//     compiler, which would round once where the reference rounds twice;
//   * batch dimensions broadcast as the reference's do (a dimension of 1 is
//     reused), each batch index decoding its own offsets into A, B and out.
// Both operands are read through their strides (transposed views need no
// copy), as the reference reads them.  This is CUDA-core work by design: the
// tensor cores accumulate in an order and with roundings of their own, which
// cannot reproduce the reference's chain.
//
// unfold_2d writes every window as one row (one thread per output element,
// coalesced writes); fold_2d gives each output pixel one thread that adds the
// values of the windows covering it in the reference's order -- windows by
// increasing (oh, ow) -- starting from +0, so its sums round exactly as the
// reference's `image[..] += src[..]` loop does.
#include <algorithm>
#include <array>
#include <cstdlib>
#include <map>
#include <mutex>
#include <type_traits>
#include <cstring>
#include <string>

#include "kernels.cuh"
#include "tma.cuh"

// Tuning knob: CTAs of the matmul kernel an SM keeps resident (its register
// budget per thread follows); the default is the shipped configuration.
#ifndef TRS_MM_MINB
#define TRS_MM_MINB 2
#endif

namespace trs {
namespace {

template <class T> struct MmTile { static constexpr int TM = 8, TN = 8, BK = 16; };
template <> struct MmTile<double> { static constexpr int TM = 8, TN = 4, BK = 8; };
template <> struct MmTile<int64_t> { static constexpr int TM = 8, TN = 4, BK = 8; };

struct MmDev {
  const void* a;
  const void* b;
  void* out;
  int64_t M, N, K;
  int64_t sam, sak, sbk, sbn, som, son;  // strides of the two matrix dimensions
  int64_t a_off, b_off, o_off;
  int nb;                                // batch dimensions of the output
  int64_t bshape[kMaxDims];
  int64_t a_bst[kMaxDims], b_bst[kMaxDims], o_bst[kMaxDims];  // 0 where broadcast
  int64_t batches;
  int a_kfast, b_nfast;                  // k (of A) / n (of B) is the unit-stride dimension
};

// The accumulators of one thread: TM x TN values, each advanced by the
// reference's step acc = acc + a * b with the product and the sum rounded
// separately (__fmul_rn / __fadd_rn for f32, which the compiler never fuses).
template <class T, int TM, int TN>
struct AccTile {
  T v[TM][TN];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) v[i][j] = T(0);
  }
  __device__ __forceinline__ void step(const T (&a)[TM], const T (&b)[TN]) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) v[i][j] = Arith<T>::add(v[i][j], Arith<T>::mul(a[i], b[j]));
  }
  __device__ __forceinline__ T get(int i, int j) const { return v[i][j]; }
};

// f32 on sm_100's packed units, two outputs per instruction.  The product is
// taken as fma(a, b, +0) in f32x2: a * b + 0 rounds exactly as the product
// alone, except that a -0 product becomes +0 -- which cannot change the chain,
// since acc starts at +0 and a round-to-nearest sum is -0 only when both of its
// terms are -0, so acc is never -0 and acc + (+-0) == acc.  The sum is a
// separate f32x2 add.  (A packed multiply followed by a packed add was
// contracted into one FMA by the compiler; an FMA followed by an add is not.)
#ifndef TRS_MM_PACKED
#define TRS_MM_PACKED 1
#endif
#if TRS_MM_PACKED
template <int TM, int TN>
struct AccTile<float, TM, TN> {
  static_assert(TN % 2 == 0, "pairs of columns");
  float2 v[TM][TN / 2];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN / 2; ++j) v[i][j] = make_float2(0.0f, 0.0f);
  }
  __device__ __forceinline__ void step(const float (&a)[TM], const float (&b)[TN]) {
    const float2 zero2 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const float2 a2 = make_float2(a[i], a[i]);
#pragma unroll
      for (int j = 0; j < TN / 2; ++j)
        v[i][j] = __fadd2_rn(v[i][j], __ffma2_rn(a2, make_float2(b[2 * j], b[2 * j + 1]), zero2));
    }
  }
  __device__ __forceinline__ float get(int i, int j) const { return (j & 1) ? v[i][j >> 1].y : v[i][j >> 1].x; }
};
#endif

// Asynchronous global -> shared copy of one element (4 or 8 bytes); src_bytes
// 0 writes zeros without reading (the slab's padding beyond M, N or K).
template <int BYTES>
__device__ __forceinline__ void cp_async_elem(void* smem_dst, const void* gsrc, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(smem_u32(smem_dst)), "l"(gsrc), "n"(BYTES),
               "r"(src_bytes)
               : "memory");
}

// Four consecutive elements of a shared row (16-byte aligned) in registers.
template <class T>
__device__ __forceinline__ void lds4(const T* p, T (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const int4 x = *reinterpret_cast<const int4*>(p);
    memcpy(v, &x, 16);
  } else {
    const int4 x = *reinterpret_cast<const int4*>(p);
    const int4 y = *reinterpret_cast<const int4*>(p + 2);
    memcpy(v, &x, 16);
    memcpy(v + 2, &y, 16);
  }
}

// Each thread owns rows {g * 64 + ty * 4 + i} and columns {h * 64 + tx * 4 + j}
// of the tile (i, j < 4; g < TM / 4, h < TN / 4): its fragment reads are 4
// consecutive elements, and the 16 threads of a row of the warp read one
// contiguous run, so the shared-memory reads are conflict-free.
template <class T>
__global__ void __launch_bounds__(kThreads, TRS_MM_MINB) matmul_kernel(const MmDev d) {
  constexpr int TM = MmTile<T>::TM, TN = MmTile<T>::TN, BK = MmTile<T>::BK;
  constexpr int BM = 16 * TM, BN = 16 * TN;
  constexpr int GM = TM / 4, GN = TN / 4;
  constexpr int LA = BM * BK / kThreads, LB = BN * BK / kThreads;
  constexpr int PAD = 16 / (int)sizeof(T);  // keeps each shared row 16-byte aligned
  constexpr int ES = (int)sizeof(T);
  __shared__ __align__(16) T As[2][BK][BM + PAD];
  __shared__ __align__(16) T Bs[2][BK][BN + PAD];
  const T* ga = static_cast<const T*>(d.a);
  const T* gb = static_cast<const T*>(d.b);
  T* go = static_cast<T*>(d.out);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  for (int64_t z = blockIdx.z; z < d.batches; z += gridDim.z) {
    int64_t ao = d.a_off, bo = d.b_off, oo = d.o_off;
    {
      int64_t r = z;
      for (int i = d.nb - 1; i >= 0; --i) {
        const int64_t c = r % d.bshape[i];
        r /= d.bshape[i];
        ao += c * d.a_bst[i];
        bo += c * d.b_bst[i];
        oo += c * d.o_bst[i];
      }
    }
    // slab k0 of A and B into shared buffer `buf`: slot q of this thread is
    // element e = tid + q * 256, laid out so consecutive threads read
    // consecutive addresses of the unit-stride dimension
    auto issue = [&](int64_t k0, int buf) {
#pragma unroll
      for (int q = 0; q < LA; ++q) {
        const int e = threadIdx.x + q * kThreads;
        const int rr = d.a_kfast ? e / BK : e % BM, kk = d.a_kfast ? e % BK : e / BM;
        const int64_t row = m0 + rr, k = k0 + kk;
        const bool in = row < d.M && k < d.K;
        cp_async_elem<ES>(&As[buf][kk][rr], in ? ga + ao + row * d.sam + k * d.sak : ga + d.a_off, in ? ES : 0);
      }
#pragma unroll
      for (int q = 0; q < LB; ++q) {
        const int e = threadIdx.x + q * kThreads;
        const int cc = d.b_nfast ? e % BN : e / BK, kk = d.b_nfast ? e / BN : e % BK;
        const int64_t col = n0 + cc, k = k0 + kk;
        const bool in = col < d.N && k < d.K;
        cp_async_elem<ES>(&Bs[buf][kk][cc], in ? gb + bo + k * d.sbk + col * d.sbn : gb + d.b_off, in ? ES : 0);
      }
      cp_async_commit();
    };

    AccTile<T, TM, TN> acc;  // +0: T::default() of the reference
    acc.zero();
    __syncthreads();  // the previous batch's last slab has been read
    issue(0, 0);
    int buf = 0;
    for (int64_t k0 = 0; k0 < d.K; k0 += BK, buf ^= 1) {
      const bool more = k0 + BK < d.K;
      if (more) {
        issue(k0 + BK, buf ^ 1);  // in flight while this slab is multiplied
        cp_async_wait_prev();
      } else {
        cp_async_wait_all();
      }
      __syncthreads();  // slab k0 is in shared memory for every thread
      const int kmax = d.K - k0 < BK ? (int)(d.K - k0) : BK;
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        if (kk < kmax) {  // k walks 0 .. K-1 in order, one step per kk
          T av[TM], bv[TN];
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            T v[4];
            lds4<T>(&As[buf][kk][g * 64 + ty * 4], v);
#pragma unroll
            for (int i = 0; i < 4; ++i) av[g * 4 + i] = v[i];
          }
#pragma unroll
          for (int h = 0; h < GN; ++h) {
            T v[4];
            lds4<T>(&Bs[buf][kk][h * 64 + tx * 4], v);
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[h * 4 + j] = v[j];
          }
          acc.step(av, bv);
        }
      }
      __syncthreads();  // every thread is done with `buf` before it is refilled
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t row = m0 + (i / 4) * 64 + ty * 4 + (i % 4);
      if (row >= d.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t col = n0 + (j / 4) * 64 + tx * 4 + (j % 4);
        if (col < d.N) go[oo + row * d.som + col * d.son] = acc.get(i, j);
      }
    }
  }
}

// ---- unfold_2d / fold_2d ----------------------------------------------------

struct ColsDev {
  const void* src;
  void* dst;
  int64_t B, C, H, W, kh, kw, sh, sw, ph, pw, OH, OW;
  int64_t x_off, xs[4];   // the image ([B, C, H, W] view): unfold's input, fold's output
  int64_t x_len, c_len;   // storage lengths of the image's and the columns' views
  int64_t c_off, cs[2];   // the columns ([B*OH*OW, C*kh*kw] view): unfold's output, fold's input
  int64_t patch, rows;
  // fold: the columns offset of window (oh, ow) for a fixed pixel is linear,
  // base + oh * step_oh + ow * step_ow, with
  // step_oh = OW * cs0 - sh * kw * cs1 and step_ow = cs0 - sw * cs1
  int64_t step_oh, step_ow;
  // 32-bit index decode (every index below 2^32): divisors of the decode
  FastDiv f_patch, f_kk, f_kw, f_ow, f_oh, f_w, f_h, f_c, f_sh, f_sw;
};

// Columns elements (unfold) or image pixels (fold) per thread per iteration:
// their loads are all issued before the first result is used, so each thread
// keeps that many gathered loads in flight.
constexpr int kColsU = 8;

// Elements idx .. of the columns, row-major: row = (b, oh, ow), col = (c, i,
// j); 32-bit decode with divisors fixed at launch.  Thread t of a block takes
// elements base + u * kThreads (u < kColsU): coalesced stores.
template <class T>
__global__ void __launch_bounds__(kThreads) unfold_kernel(const ColsDev d) {
  const T* x = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const uint32_t n = (uint32_t)(d.rows * d.patch);
  const int32_t H = (int32_t)d.H, W = (int32_t)d.W;
  const uint32_t step = gridDim.x * (kThreads * kColsU);
  for (uint32_t base = blockIdx.x * (kThreads * kColsU) + threadIdx.x; base < n; base += step) {
    T v[kColsU];
    uint32_t at[kColsU];
#pragma unroll
    for (int u = 0; u < kColsU; ++u) {
      const uint32_t idx = base + (uint32_t)u * kThreads;
      at[u] = idx;
      v[u] = T(0);
      if (idx < n) {
        const uint32_t row = fdiv(idx, d.f_patch), col = idx - row * d.f_patch.d;
        const uint32_t r1 = fdiv(row, d.f_ow), ow = row - r1 * d.f_ow.d;
        const uint32_t b = fdiv(r1, d.f_oh), oh = r1 - b * d.f_oh.d;
        const uint32_t c = fdiv(col, d.f_kk), r = col - c * d.f_kk.d;
        const uint32_t i = fdiv(r, d.f_kw), j = r - i * d.f_kw.d;
        const int32_t y = (int32_t)(oh * (uint32_t)d.sh + i) - (int32_t)d.ph;
        const int32_t xx = (int32_t)(ow * (uint32_t)d.sw + j) - (int32_t)d.pw;
        if (y >= 0 && y < H && xx >= 0 && xx < W)
          v[u] = x[d.x_off + (int64_t)b * d.xs[0] + (int64_t)c * d.xs[1] + (int64_t)y * d.xs[2] +
                   (int64_t)xx * d.xs[3]];
      }
    }
#pragma unroll
    for (int u = 0; u < kColsU; ++u) {
      if (at[u] < n) {
        const uint32_t row = fdiv(at[u], d.f_patch), col = at[u] - row * d.f_patch.d;
        out[d.c_off + (int64_t)row * d.cs[0] + (int64_t)col * d.cs[1]] = v[u];
      }
    }
  }
}

// Largest patch (columns of a row) whose column table fits a CTA's shared
// memory in the tile kernel below.
constexpr int kUnfoldTab = 2048;

// unfold by tiles of kUtRows output rows x kUtCols columns, transposed
// through shared memory so both sides are coalesced, with the patch's column
// table in shared memory (one 8-byte entry per column: its image offset and
// (i, j), written once per CTA; offsets within 31 bits).  In the gather, lane
// r of a warp takes output row r0 + r -- consecutive rows are consecutive ow,
// so consecutive image columns -- for one column at a time, whose table entry
// is the same for the whole warp (a broadcast read); values go to
// tile[col][row] (pitch kUtRows + 1: conflict-free both ways).  After a
// barrier each warp stores whole tile rows, lanes along the columns.
constexpr int kUtRows = 32;
constexpr int kUtCols = 64;

// I32: every index the kernel forms (padding offsets included) lies within
// (-2^31, 2^31), so the index arithmetic runs in 32 bits.
template <class T, bool I32>
__global__ void __launch_bounds__(kThreads) unfold_tile_kernel(const ColsDev d) {
  using Idx = typename std::conditional<I32, int32_t, int64_t>::type;
  __shared__ T tile[kUtCols][kUtRows + 1];
  __shared__ int2 tab[kUnfoldTab];  // (image offset of column (c, i, j), i << 16 | j)
  constexpr int kWarps = kThreads / 32;
  const T* x = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rows = (uint32_t)d.rows, patch = (uint32_t)d.patch;
  const uint32_t H = (uint32_t)d.H, W = (uint32_t)d.W;
  for (uint32_t col = threadIdx.x; col < patch; col += kThreads) {
    const uint32_t c = fdiv(col, d.f_kk), r = col - c * d.f_kk.d;
    const uint32_t i = fdiv(r, d.f_kw), j = r - i * d.f_kw.d;
    tab[col] = make_int2((int)((int64_t)c * d.xs[1] + (int64_t)i * d.xs[2] + (int64_t)j * d.xs[3]),
                         (int)((i << 16) | j));
  }
  __syncthreads();
  const uint32_t n_rb = (rows + kUtRows - 1) / kUtRows, n_cb = (patch + kUtCols - 1) / kUtCols;
  const uint64_t tiles = (uint64_t)n_rb * n_cb;
  for (uint64_t tl = blockIdx.x; tl < tiles; tl += gridDim.x) {
    // column blocks fastest: neighbouring CTAs gather from the same image rows
    const uint32_t rb = (uint32_t)(tl / n_cb), cb = (uint32_t)(tl - (uint64_t)rb * n_cb);
    const uint32_t r0 = rb * kUtRows, c0 = cb * kUtCols;
    const uint32_t row = r0 + (uint32_t)lane;  // this lane's output row
    const bool row_ok = row < rows;
    const uint32_t r1 = fdiv(row, d.f_ow), ow = row - r1 * d.f_ow.d;
    const uint32_t b = fdiv(r1, d.f_oh), oh = r1 - b * d.f_oh.d;
    const int32_t y0 = (int32_t)(oh * (uint32_t)d.sh) - (int32_t)d.ph;
    const int32_t x0 = (int32_t)(ow * (uint32_t)d.sw) - (int32_t)d.pw;
    const Idx base = (Idx)d.x_off + (Idx)b * (Idx)d.xs[0] + (Idx)y0 * (Idx)d.xs[2] + (Idx)x0 * (Idx)d.xs[3];
    T v[kUtCols / kWarps];
#pragma unroll
    for (int k = 0; k < kUtCols / kWarps; ++k) {
      const uint32_t col = c0 + (uint32_t)(warp + k * kWarps);
      v[k] = T(0);
      if (col < patch) {
        const int2 e = tab[col];
        const uint32_t ij = (uint32_t)e.y;
        const uint32_t y = (uint32_t)(y0 + (int32_t)(ij >> 16)), xx = (uint32_t)(x0 + (int32_t)(ij & 0xFFFFu));
        if (row_ok && y < H && xx < W) v[k] = x[base + (Idx)e.x];
      }
    }
#pragma unroll
    for (int k = 0; k < kUtCols / kWarps; ++k) tile[warp + k * kWarps][lane] = v[k];
    __syncthreads();
    // store: warp w writes tile rows w, w + 8, ...; lanes along the columns
#pragma unroll
    for (int rr = warp; rr < kUtRows; rr += kWarps) {
      const uint32_t orow = r0 + (uint32_t)rr;
      if (orow < rows) {
        const Idx ob = (Idx)d.c_off + (Idx)orow * (Idx)d.cs[0];
#pragma unroll
        for (int h = 0; h < kUtCols / 32; ++h) {
          const uint32_t col = c0 + (uint32_t)(lane + 32 * h);
          if (col < patch) out[ob + (Idx)col * (Idx)d.cs[1]] = tile[lane + 32 * h][rr];
        }
      }
    }
    __syncthreads();  // the tile is free for the next one
  }
}

// One thread per output pixel (b, c, y, x), row-major: adds the values of the
// windows covering the pixel, windows by increasing (oh, ow), from +0.  When
// at most kFoldRegs windows can cover a pixel (ceil(kh / sh) * ceil(kw / sw),
// every usual convolution), the values are all loaded before the first
// addition; otherwise they are added as they are loaded.
constexpr int kFoldRegs = 16;

template <class T, bool REGS>
__global__ void __launch_bounds__(kThreads) fold_kernel(const ColsDev d) {
  using A = Arith<T>;
  const T* cols = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const uint32_t n = (uint32_t)(d.B * d.C * d.H * d.W);
  const int32_t kh = (int32_t)d.kh, kw = (int32_t)d.kw, sh = (int32_t)d.sh, sw = (int32_t)d.sw;
  const int32_t OH = (int32_t)d.OH, OW = (int32_t)d.OW;
  for (uint32_t idx = blockIdx.x * kThreads + threadIdx.x; idx < n; idx += gridDim.x * kThreads) {
    const uint32_t q1 = fdiv(idx, d.f_w), xx = idx - q1 * d.f_w.d;
    const uint32_t q2 = fdiv(q1, d.f_h), y = q1 - q2 * d.f_h.d;
    const uint32_t b = fdiv(q2, d.f_c), c = q2 - b * d.f_c.d;
    // windows whose rows hold y: oh * sh <= y + ph <= oh * sh + kh - 1
    const int32_t yp = (int32_t)y + (int32_t)d.ph, xp = (int32_t)xx + (int32_t)d.pw;
    const int32_t oh_lo = yp - kh + 1 <= 0 ? 0 : (int32_t)fdiv((uint32_t)(yp - kh + sh), d.f_sh);
    int32_t oh_hi = (int32_t)fdiv((uint32_t)yp, d.f_sh);
    if (oh_hi > OH - 1) oh_hi = OH - 1;
    const int32_t ow_lo = xp - kw + 1 <= 0 ? 0 : (int32_t)fdiv((uint32_t)(xp - kw + sw), d.f_sw);
    int32_t ow_hi = (int32_t)fdiv((uint32_t)xp, d.f_sw);
    if (ow_hi > OW - 1) ow_hi = OW - 1;
    const int32_t nw = ow_hi - ow_lo + 1;
    // window (oh, ow) is column (c, i, j) = (c, yp - oh * sh, xp - ow * sw) of
    // row (b, oh, ow); its offset steps by step_oh / step_ow per window
    const int64_t first = d.c_off + (int64_t)b * OH * OW * d.cs[0] +
                          (((int64_t)c * kh + yp) * kw + xp) * d.cs[1] + (int64_t)oh_lo * d.step_oh +
                          (int64_t)ow_lo * d.step_ow;
    T acc = T(0);
    if constexpr (REGS) {
      const int32_t cnt = (oh_hi >= oh_lo && nw > 0) ? (oh_hi - oh_lo + 1) * nw : 0;
      T v[kFoldRegs];
      int64_t row_at = first, at = first;
      int32_t ow = ow_lo;  // window w = (oh, ow), row-major over the covering range
#pragma unroll
      for (int w = 0; w < kFoldRegs; ++w) {
        v[w] = T(0);
        if (w < cnt) {
          v[w] = cols[at];
          if (++ow > ow_hi) {
            ow = ow_lo;
            row_at += d.step_oh;
            at = row_at;
          } else {
            at += d.step_ow;
          }
        }
      }
#pragma unroll
      for (int w = 0; w < kFoldRegs; ++w)
        if (w < cnt) acc = A::add(acc, v[w]);  // windows in (oh, ow) order
    } else {
      int64_t row_at = first;
      for (int32_t oh = oh_lo; oh <= oh_hi; ++oh, row_at += d.step_oh) {
        int64_t at = row_at;
        for (int32_t ow = ow_lo; ow <= ow_hi; ++ow, at += d.step_ow) acc = A::add(acc, cols[at]);
      }
    }
    out[d.x_off + (int64_t)b * d.xs[0] + (int64_t)c * d.xs[1] + (int64_t)y * d.xs[2] + (int64_t)xx * d.xs[3]] = acc;
  }
}

// fold through shared memory.  A tile is (b, a block of CB channels, a band
// of TY output rows, every column x).  The windows that can cover the band
// are the rows (b, oh, ow) for oh in [oh_a, oh_b] and every ow: consecutive
// rows of the columns matrix, of which the tile needs the CB * kh * kw
// consecutive entries of its channels.  The CTA copies those into shared
// memory with coalesced 4- or 8-byte cp.async (entry t of window row r at
// r * segp + t, segp odd so that neighbouring windows fall in different
// banks), then each thread adds, for its pixels, the covering windows by
// increasing (oh, ow) from +0 -- the reference's order -- reading them from
// shared memory with the same linear stepping as fold_kernel.  Window rows at
// a band's edges are copied by both neighbouring tiles; tiles are numbered
// band-fastest, so the second copy usually comes from L2.
struct FoldTile {
  int32_t CB, TY, noh, seg, segp;  // channels, output rows, window rows, entries per window row (and padded)
  int32_t n_cb, n_yb;              // channel blocks, bands
  int64_t tiles;
  FastDiv f_seg, f_ty, f_yb, f_cb;
};

// WIN > 0: at most WIN x WIN windows cover a pixel (ceil(kh / sh) and
// ceil(kw / sw) <= WIN), and the window loops are unrolled WIN x WIN with each
// add predicated on the window existing, so the adds keep their (oh, ow)
// order; WIN = 0: loops bounded at run time.
// I32: the columns' and the image's storage are below 2^31 elements, so the
// global index arithmetic runs in 32 bits.
template <class T, int WIN, bool I32>
__global__ void __launch_bounds__(kThreads) fold_smem_kernel(const ColsDev d, const FoldTile t) {
  using Idx = typename std::conditional<I32, int32_t, int64_t>::type;
  using A = Arith<T>;
  extern __shared__ __align__(16) unsigned char fold_raw[];
  T* sm = reinterpret_cast<T*>(fold_raw);
  const T* cols = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const int32_t kh = (int32_t)d.kh, kw = (int32_t)d.kw, sh = (int32_t)d.sh, sw = (int32_t)d.sw;
  const int32_t OH = (int32_t)d.OH, OW = (int32_t)d.OW, H = (int32_t)d.H, W = (int32_t)d.W;
  const int32_t C = (int32_t)d.C, kk = kh * kw;
  const int32_t step_ow = t.segp - sw, step_oh = OW * t.segp - sh * kw;
  for (int64_t tile = blockIdx.x; tile < t.tiles; tile += gridDim.x) {
    // tile = (b * n_cb + cb) * n_yb + yb
    const uint32_t q1 = fdiv((uint32_t)tile, t.f_yb), yb = (uint32_t)tile - q1 * t.f_yb.d;
    const uint32_t b = fdiv(q1, t.f_cb), cb = q1 - b * t.f_cb.d;
    const int32_t y0 = (int32_t)yb * t.TY, c0 = (int32_t)cb * t.CB;
    const int32_t ty = H - y0 < t.TY ? H - y0 : t.TY, ncb = C - c0 < t.CB ? C - c0 : t.CB;
    // window rows covering output rows y0 .. y0 + ty - 1
    const int32_t lo = y0 + (int32_t)d.ph - kh + 1, hi = y0 + ty - 1 + (int32_t)d.ph;
    const int32_t oh_a = lo <= 0 ? 0 : (int32_t)fdiv((uint32_t)(lo + sh - 1), d.f_sh);
    const int32_t hq = (int32_t)fdiv((uint32_t)hi, d.f_sh);
    const int32_t oh_b = hq < OH - 1 ? hq : OH - 1;
    const int32_t noh = oh_b - oh_a + 1;
    const int32_t seg_eff = ncb * kk;
    if (noh > 0) {
      const Idx row0 = ((Idx)b * OH + oh_a) * OW;  // first window row of the tile
      const Idx src0 = (Idx)d.c_off + row0 * (Idx)d.cs[0] + (Idx)c0 * kk * (Idx)d.cs[1];
      const uint32_t n_load = (uint32_t)(noh * OW) * (uint32_t)t.seg;
      for (uint32_t i = threadIdx.x; i < n_load; i += kThreads) {
        const uint32_t r = fdiv(i, t.f_seg), e = i - r * t.f_seg.d;
        if ((int32_t)e < seg_eff)
          cp_async_elem<(int)sizeof(T)>(sm + (size_t)r * t.segp + e, cols + (src0 + (Idx)r * (Idx)d.cs[0] + (Idx)e * (Idx)d.cs[1]),
                                        (int)sizeof(T));
      }
      cp_async_commit();
      cp_async_wait_all();
    }
    __syncthreads();  // the tile's windows are in shared memory
    const uint32_t n_pix = (uint32_t)(ncb * t.TY * W);  // rows yr >= ty (last band) are skipped
    for (uint32_t pidx = threadIdx.x; pidx < n_pix; pidx += kThreads) {
      const uint32_t q = fdiv(pidx, d.f_w), x = pidx - q * d.f_w.d;
      const uint32_t cr = fdiv(q, t.f_ty), yr = q - cr * t.f_ty.d;
      if ((int32_t)yr >= ty) continue;
      const int32_t y = y0 + (int32_t)yr, c = c0 + (int32_t)cr;
      const int32_t yp = y + (int32_t)d.ph, xp = (int32_t)x + (int32_t)d.pw;
      // window ranges by the fast divisions (every dividend here is >= 0)
      const int32_t ohl = yp - kh + 1 <= 0 ? 0 : (int32_t)fdiv((uint32_t)(yp - kh + sh), d.f_sh);
      int32_t ohh = (int32_t)fdiv((uint32_t)yp, d.f_sh);
      if (ohh > OH - 1) ohh = OH - 1;
      const int32_t owl = xp - kw + 1 <= 0 ? 0 : (int32_t)fdiv((uint32_t)(xp - kw + sw), d.f_sw);
      int32_t owh = (int32_t)fdiv((uint32_t)xp, d.f_sw);
      if (owh > OW - 1) owh = OW - 1;
      T acc = T(0);
      int32_t row_at = ((ohl - oh_a) * OW + owl) * t.segp + (int32_t)cr * kk + (yp - ohl * sh) * kw + (xp - owl * sw);
      if constexpr (WIN > 0) {
#pragma unroll
        for (int dh = 0; dh < WIN; ++dh) {
#pragma unroll
          for (int dw = 0; dw < WIN; ++dw)
            if (ohl + dh <= ohh && owl + dw <= owh) acc = A::add(acc, sm[row_at + dh * step_oh + dw * step_ow]);
        }
      } else {
        for (int32_t oh = ohl; oh <= ohh; ++oh, row_at += step_oh) {
          int32_t at = row_at;
          for (int32_t ow = owl; ow <= owh; ++ow, at += step_ow) acc = A::add(acc, sm[at]);
        }
      }
      out[(Idx)d.x_off + (Idx)b * (Idx)d.xs[0] + (Idx)c * (Idx)d.xs[1] + (Idx)y * (Idx)d.xs[2] + (Idx)x * (Idx)d.xs[3]] =
          acc;
    }
    __syncthreads();  // every thread is done with the tile's windows
  }
}

// Tuning knob: 1 stores the unfold's output evict-first (st.global.cs), 0
// with the default cache policy.
#ifndef TRS_UNFOLD_CS
#define TRS_UNFOLD_CS 1
#endif

// V consecutive values of T stored as one 16-byte access at a V-aligned
// address (evict-first when TRS_UNFOLD_CS: the output is not read again).
template <class T, int V>
__device__ __forceinline__ void store_cs(T* p, const T (&v)[V]) {
  static_assert(sizeof(T) * V == 16 || V == 1, "16-byte vectors or single values");
  if constexpr (V == 1) {
    if (TRS_UNFOLD_CS) __stcs(p, v[0]); else *p = v[0];
  } else {
    uint32_t w[4];
    memcpy(w, v, 16);
    if (TRS_UNFOLD_CS)
      asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                   "r"(w[3])
                   : "memory");
    else
      asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
  }
}

// unfold by output rows.  A tile is (b, oh, a block of CB channels
// c0 .. c0 + CB - 1): the OW rows (b, oh, 0 .. OW-1) of the columns, entries
// [c0*kk, (c0 + CB)*kk) of each (kk = kh*kw).  The CTA stages the CB*kh image
// rows those windows read, y = oh*sh - ph + i, in shared memory as
// img_s[(cl*kh + i)*Ws + x + xo] for x from -xo to Ws - xo - 1 (zeros outside
// the image), which covers every x a window reads, -pw .. (OW-1)*sw + kw-1-pw;
// row (cl, i) starts at cl*CS + i*IS.  With TMA the rows arrive as kh boxes
// [Ws, 1, CB, 1] of the image seen as [B][C][H][W], one per i (CS = Ws,
// IS = CB*Ws; xo = pw rounded up to 16 bytes, so each box starts on a 16-byte
// boundary; rows, columns and channels outside the image read zeros; Ws is
// the width, among those that fit, whose loads below meet the fewest bank
// conflicts); otherwise the threads copy them, all their loads in flight at
// once (CS = kh*Ws, IS = Ws, xo = pw).  Then each thread writes one group g
// of V consecutive entries (16 bytes) of every step-th row: entry (cl, i, j)
// of window ow is img_s[e + ow*sw] with e = cl*CS + i*IS + j + xo - pw, so
// the thread keeps
// its V offsets e in registers and walks the rows with two increments --
// V shared loads and one streaming store per V entries.  Each image row is
// staged by about kh/sh tiles, from L2 after the first.
struct UnfoldRows {
  int32_t CB, n_cb, Ws, xo;  // channels per tile, channel blocks, staged row width, staged x offset
  int32_t CS, IS;            // shared strides of a channel and of a window row i
  uint32_t tiles;
  FastDiv f_ncb, f_oh, f_ws, f_kh;
};

// Staged image elements per thread per round when the threads copy them: all
// their loads are issued before the first is stored.
constexpr int kUrStage = 12;

template <class T, int V, bool TMA>
__global__ void __launch_bounds__(kThreads) unfold_rows_kernel(const __grid_constant__ CUtensorMap imap,
                                                               const ColsDev d, const UnfoldRows u, int* err) {
  extern __shared__ unsigned char ur_raw[];
  // aligned by an offset into the shared array itself (not through an
  // integer), so the compiler keeps every access a 32-bit shared one
  unsigned char* base = ur_raw + ((128u - (smem_u32(ur_raw) & 127u)) & 127u);
  T* img = reinterpret_cast<T*>(base);
  const int32_t kh = (int32_t)d.kh, kw = (int32_t)d.kw, kk = kh * kw;
  const int32_t OH = (int32_t)d.OH, OW = (int32_t)d.OW, C = (int32_t)d.C;
  const int32_t sw = (int32_t)d.sw, Ws = u.Ws;
  // TMA: kh window rows IS apart; copied: CB channels CS = kh*Ws apart
  const uint32_t stage_elems = TMA ? (uint32_t)kh * (uint32_t)u.IS : (uint32_t)u.CB * (uint32_t)u.CS;
  uint64_t& bar = *reinterpret_cast<uint64_t*>(base + ((size_t)stage_elems * sizeof(T) + 7) / 8 * 8);
  if (TMA) {
    if (threadIdx.x == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
  }
  uint32_t phase = 0;
  for (uint32_t tile = blockIdx.x; tile < u.tiles; tile += gridDim.x) {
    // tile = (b * OH + oh) * n_cb + cb
    const uint32_t r1 = fdiv(tile, u.f_ncb), b = fdiv(r1, u.f_oh);
    const int32_t cb = (int32_t)(tile - r1 * u.f_ncb.d), oh = (int32_t)(r1 - b * u.f_oh.d);
    const int32_t c0 = cb * u.CB, ncb = C - c0 < u.CB ? C - c0 : u.CB;
    const int32_t ybase = oh * (int32_t)d.sh - (int32_t)d.ph;
    if constexpr (TMA) {
      if (threadIdx.x == 0) {
        fence_proxy_async();  // the previous tile's reads (before the barrier that ended it) first
        mbar_arrive_expect_tx(&bar, (uint32_t)kh * (uint32_t)u.CB * (uint32_t)Ws * (uint32_t)sizeof(T));
        for (int32_t i = 0; i < kh; ++i) tma_load_4d(img + i * u.IS, &imap, -u.xo, ybase + i, c0, (int32_t)b, &bar);
      }
      const bool ok = cta_wait(&bar, phase);
      phase ^= 1u;
      if (!ok) {
        if (threadIdx.x == 0) {
          atomicOr(err, kAsyncWaitTimeout);
          mbar_wait(&bar, phase ^ 1u);  // the copy still in flight (bounded)
        }
        __syncthreads();
        return;
      }
    } else {
      const T* x = static_cast<const T*>(d.src);
      const int32_t H = (int32_t)d.H, W = (int32_t)d.W;
      const T* xb = x + d.x_off + (int64_t)b * d.xs[0] + (int64_t)c0 * d.xs[1];
      const int32_t n_stage = ncb * kh * Ws;
      for (int32_t e0 = threadIdx.x; e0 < n_stage; e0 += kThreads * kUrStage) {
        T v[kUrStage];
#pragma unroll
        for (int k = 0; k < kUrStage; ++k) {
          const int32_t e = e0 + k * kThreads;
          v[k] = T(0);
          if (e < n_stage) {
            const uint32_t rr = fdiv((uint32_t)e, u.f_ws), cl = fdiv(rr, u.f_kh);
            const int32_t y = ybase + (int32_t)(rr - cl * u.f_kh.d), xx = e - (int32_t)(rr * u.f_ws.d) - u.xo;
            if (y >= 0 && y < H && xx >= 0 && xx < W)
              v[k] = xb[(int64_t)cl * d.xs[1] + (int64_t)y * d.xs[2] + (int64_t)xx * d.xs[3]];
          }
        }
#pragma unroll
        for (int k = 0; k < kUrStage; ++k)
          if (e0 + k * kThreads < n_stage) img[e0 + k * kThreads] = v[k];
      }
      __syncthreads();
    }
    // groups g of V entries; G <= kThreads: step = kThreads / G rows at a
    // time, thread t on group t % G of rows t / G, t / G + step, ...
    const int32_t G = ncb * kk / V;
    const int32_t step = G <= kThreads ? kThreads / G : 1;
    T* ob = static_cast<T*>(d.dst) + d.c_off + ((int64_t)b * OH + oh) * (int64_t)OW * d.cs[0] + (int64_t)c0 * kk;
    const int64_t ostep = (int64_t)step * d.cs[0];
    for (int32_t gi = threadIdx.x; gi < (G <= kThreads ? step * G : G); gi += kThreads) {
      const int32_t g = G <= kThreads ? gi % G : gi, ow0 = G <= kThreads ? gi / G : 0;
      int32_t e[V];
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const uint32_t col = (uint32_t)(g * V + k), cl = fdiv(col, d.f_kk), r = col - cl * d.f_kk.d;
        const uint32_t i = fdiv(r, d.f_kw), j = r - i * d.f_kw.d;
        e[k] = (int32_t)cl * u.CS + (int32_t)i * u.IS + (int32_t)j + u.xo - (int32_t)d.pw;
      }
      T* op = ob + (int64_t)ow0 * d.cs[0] + g * V;
      int32_t s = ow0 * sw;
      for (int32_t ow = ow0; ow < OW; ow += step, s += step * sw, op += ostep) {
        T v[V];
#pragma unroll
        for (int k = 0; k < V; ++k) v[k] = img[e[k] + s];
        store_cs<T, V>(op, v);
      }
    }
    __syncthreads();  // the rows are free for the next tile
  }
}

// fold for stride 1 from window rows staged by TMA.  A tile is (b, a block of
// CB channels, a band of TY image rows y0 .. y0+TY-1, a strip of XS image
// columns x0 .. x0+XS-1).  Pixel (y, x) is covered by the windows
// (oh, ow) = (y + ph - i, x + pw - j), 0 <= i < kh, 0 <= j < kw, that lie in
// [0, OH) x [0, OW); the tile's windows are therefore the columns' rows
// (b, oh, ow) with oh in [y0 + ph - kh + 1, y0 + TY - 1 + ph] and ow in
// [x0 + pw - kw + 1, x0 + XS - 1 + pw]: R = TY + kh - 1 window rows of
// Q = XS + kw - 1 windows, of which the tile needs the seg = CB*kk
// consecutive entries of its channels.  One thread loads each window row
// with one TMA box [seg, Q, 1, 1] of the columns seen as [B][OH][OW][patch]
// (windows with ow outside [0, OW) arrive as zeros); window rows outside
// [0, OH) are written as zeros by the threads.  Window (r, q) entry t sits
// at r*RS + q*seg + t, so pixel (yy, xx, cl) of the tile finds window (i, j)
// at base + ii*(RS - kw) + jj*(seg - 1) + kk - 1, with ii = kh-1-i,
// jj = kw-1-j and base = yy*RS + xx*seg + cl*kk: the same offsets for every
// pixel, no window bounds.  Each thread keeps one (cl, xx) and walks the
// band's rows (RS apart in shared memory, xs2 apart in the image).  The adds
// run ii and jj upward -- windows by increasing (oh, ow), the reference's
// order -- from +0; a missing window adds +0, which changes no sum (a sum
// from +0 is never -0, and s + (+0) = s for every other s, NaN and
// infinities included).  K > 0: kh = kw = K unrolled; SEG > 0: seg = SEG at
// compile time (the offsets jj*(seg-1) become immediates).
struct FoldS1 {
  int32_t CB, TY, XS, R, Q, seg, RS;  // tile; window rows, windows per row, entries per window, row stride
  uint32_t tiles;
  FastDiv f_cb, f_nxb, f_nyb, f_ncb;
};

template <class T, int K, int SEG>
__global__ void __launch_bounds__(kThreads) fold_s1_kernel(const __grid_constant__ CUtensorMap cmap, const ColsDev d,
                                                           const FoldS1 f, int* err) {
  using A = Arith<T>;
  // the window rows from a 128-byte boundary (each row's start, RS * sizeof(T)
  // bytes apart, is one too: a TMA destination), the mbarrier after them
  extern __shared__ unsigned char fs_raw[];
  // aligned by an offset into the shared array itself (not through an
  // integer), so the compiler keeps every access a 32-bit shared one
  unsigned char* base = fs_raw + ((128u - (smem_u32(fs_raw) & 127u)) & 127u);
  T* sm = reinterpret_cast<T*>(base);
  uint64_t& bar = *reinterpret_cast<uint64_t*>(base + (size_t)f.R * f.RS * sizeof(T));
  const int32_t kh = K ? K : (int32_t)d.kh, kw = K ? K : (int32_t)d.kw, kk = kh * kw;
  const int32_t H = (int32_t)d.H, W = (int32_t)d.W, C = (int32_t)d.C, OH = (int32_t)d.OH;
  const int32_t RS = f.RS, seg = SEG ? SEG : f.seg, row_elems = f.Q * seg;
  const uint32_t box_bytes = (uint32_t)row_elems * (uint32_t)sizeof(T);
  // this thread's (cl, xx) pairs and first row: pairs = CB * XS
  const int32_t pairs = f.CB * f.XS;
  const int32_t ystep = pairs <= kThreads ? kThreads / pairs : 1;
  const int32_t n_slots = pairs <= kThreads ? ystep * pairs : pairs;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t phase = 0;
  for (uint32_t tile = blockIdx.x; tile < f.tiles; tile += gridDim.x) {
    // tile = ((b * n_cb + cb) * n_yb + yb) * n_xb + xb
    const uint32_t t1 = fdiv(tile, f.f_nxb), t2 = fdiv(t1, f.f_nyb), b = fdiv(t2, f.f_ncb);
    const int32_t xb = (int32_t)(tile - t1 * f.f_nxb.d), yb = (int32_t)(t1 - t2 * f.f_nyb.d);
    const int32_t cb = (int32_t)(t2 - b * f.f_ncb.d);
    const int32_t y0 = yb * f.TY, x0 = xb * f.XS, c0 = cb * f.CB;
    const int32_t ty = H - y0 < f.TY ? H - y0 : f.TY, xs = W - x0 < f.XS ? W - x0 : f.XS;
    const int32_t ncb = C - c0 < f.CB ? C - c0 : f.CB;
    const int32_t oh_a = y0 + (int32_t)d.ph - kh + 1, ow_a = x0 + (int32_t)d.pw - kw + 1;
    if (threadIdx.x == 0) {
      // the previous tile's reads of these rows (ordered by the barrier that
      // ended it) come before the copies' writes
      fence_proxy_async();
      uint32_t n_in = 0;
      for (int32_t r = 0; r < f.R; ++r) n_in += (oh_a + r >= 0 && oh_a + r < OH) ? 1u : 0u;
      mbar_arrive_expect_tx(&bar, n_in * box_bytes);
      for (int32_t r = 0; r < f.R; ++r)
        if (oh_a + r >= 0 && oh_a + r < OH) tma_load_4d(sm + r * RS, &cmap, c0 * kk, ow_a, oh_a + r, (int32_t)b, &bar);
    }
    for (int32_t r = 0; r < f.R; ++r)
      if (oh_a + r < 0 || oh_a + r >= OH)
        for (int32_t e = threadIdx.x; e < row_elems; e += kThreads) sm[r * RS + e] = T(0);
    const bool ok = cta_wait(&bar, phase);
    phase ^= 1u;
    if (!ok) {
      if (threadIdx.x == 0) {
        atomicOr(err, kAsyncWaitTimeout);
        mbar_wait(&bar, phase ^ 1u);  // the copies still in flight (bounded)
      }
      __syncthreads();
      return;
    }
    T* obase = static_cast<T*>(d.dst) + d.x_off + (int64_t)b * d.xs[0] + (int64_t)c0 * d.xs[1] +
               (int64_t)y0 * d.xs[2] + (int64_t)x0 * d.xs[3];
    for (int32_t slot = threadIdx.x; slot < n_slots; slot += kThreads) {
      const int32_t pair = pairs <= kThreads ? slot % pairs : slot, yy0 = pairs <= kThreads ? slot / pairs : 0;
      // pair = xx * CB + cl
      const uint32_t xx = fdiv((uint32_t)pair, f.f_cb), cl = (uint32_t)pair - xx * f.f_cb.d;
      if ((int32_t)cl >= ncb || (int32_t)xx >= xs) continue;
      const T* s = sm + yy0 * RS + (int32_t)xx * seg + (int32_t)cl * kk + (kk - 1);
      T* o = obase + (int64_t)cl * d.xs[1] + (int64_t)yy0 * d.xs[2] + (int64_t)xx * d.xs[3];
      const int64_t ostep = (int64_t)ystep * d.xs[2];
      for (int32_t yy = yy0; yy < ty; yy += ystep, s += ystep * RS, o += ostep) {
        T acc = T(0);
        if constexpr (K > 0) {
          T v[K * K];
#pragma unroll
          for (int ii = 0; ii < K; ++ii) {
            const T* sr = s + ii * (RS - K);
#pragma unroll
            for (int jj = 0; jj < K; ++jj) v[ii * K + jj] = sr[jj * (seg - 1)];
          }
#pragma unroll
          for (int w = 0; w < K * K; ++w) acc = A::add(acc, v[w]);
        } else {
          for (int32_t ii = 0; ii < kh; ++ii)
            for (int32_t jj = 0; jj < kw; ++jj) acc = A::add(acc, s[ii * (RS - kw) + jj * (seg - 1)]);
        }
        *o = acc;
      }
    }
    __syncthreads();  // every thread is done with the tile's windows
  }
}

// ---- host side ---------------------------------------------------------------

bool ranges_overlap(const trs_view* a, const trs_view* b) {
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

std::string shape_str(const int64_t* s, int n) {
  std::string r = "[";
  for (int i = 0; i < n; ++i) r += (i ? ", " : "") + std::to_string((long long)s[i]);
  return r + "]";
}

template <class T>
Error launch_matmul(const MmDev& d, cudaStream_t stream) {
  constexpr int BM = 16 * MmTile<T>::TM, BN = 16 * MmTile<T>::TN;
  const uint64_t gx = ((uint64_t)d.N + BN - 1) / BN, gy = ((uint64_t)d.M + BM - 1) / BM;
  if (gx > 0x7fffffffull || gy > 65535)
    return make_error(TRS_ERR_SHAPE, "matmul: M or N beyond the launch grid (M < 8 388 480 rows)");
  const unsigned gz = (unsigned)(d.batches < 65535 ? d.batches : 65535);
  matmul_kernel<T><<<dim3((unsigned)gx, (unsigned)gy, gz), kThreads, 0, stream>>>(d);
  return check_launch("matmul kernel");
}

Error run_matmul(const trs_view* a, const trs_view* b, const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(a, "a");
  if (!e.ok()) return e;
  e = validate_view(b, "b");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (a->dtype != b->dtype || out->dtype != a->dtype)
    return make_error(TRS_ERR_DTYPE, "matmul: a, b and the output must share one dtype");
  const int an = a->ndim, bn = b->ndim;
  if (an < 2 || bn < 2) return make_error(TRS_ERR_SHAPE, "matmul: both tensors must be at least 2D");
  const int64_t M = a->shape[an - 2], K = a->shape[an - 1], N = b->shape[bn - 1];
  if (K != b->shape[bn - 2])
    return make_error(TRS_ERR_SHAPE, "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])");
  int64_t batch[kMaxDims];
  int nb = 0;
  if (!broadcast_shapes(a->shape, an - 2, b->shape, bn - 2, batch, &nb))
    return make_error(TRS_ERR_SHAPE, "matmul: batch shapes not broadcastable");
  // the output the reference returns: [batch..., M, N]
  int64_t want[kMaxDims + 2];
  for (int i = 0; i < nb; ++i) want[i] = batch[i];
  want[nb] = M;
  want[nb + 1] = N;
  bool same = out->ndim == nb + 2;
  for (int i = 0; same && i < nb + 2; ++i) same = out->shape[i] == want[i];
  if (!same)
    return make_error(TRS_ERR_SHAPE, "matmul: the output must have shape " + shape_str(want, nb + 2));
  if (ranges_overlap(out, a) || ranges_overlap(out, b))
    return make_error(TRS_ERR_ALIAS, "matmul: the output overlaps an input");
  MmDev d;
  std::memset(&d, 0, sizeof(d));
  d.a = a->data;
  d.b = b->data;
  d.out = out->data;
  d.M = M;
  d.N = N;
  d.K = K;
  d.sam = a->strides[an - 2];
  d.sak = a->strides[an - 1];
  d.sbk = b->strides[bn - 2];
  d.sbn = b->strides[bn - 1];
  d.som = out->strides[nb];
  d.son = out->strides[nb + 1];
  d.a_off = a->offset;
  d.b_off = b->offset;
  d.o_off = out->offset;
  d.nb = nb;
  d.batches = 1;
  for (int i = 0; i < nb; ++i) {
    d.bshape[i] = batch[i];
    d.batches *= batch[i];
    // batch strides as batch_offset (base.rs:949-961) reads them: right-aligned,
    // 0 where the operand's dimension is 1 (or absent)
    const int ia = i - (nb - (an - 2)), ib = i - (nb - (bn - 2));
    d.a_bst[i] = (ia >= 0 && a->shape[ia] != 1) ? a->strides[ia] : 0;
    d.b_bst[i] = (ib >= 0 && b->shape[ib] != 1) ? b->strides[ib] : 0;
    d.o_bst[i] = out->strides[i];
  }
  d.a_kfast = d.sak == 1 || d.sam != 1;
  d.b_nfast = d.sbn == 1 || d.sbk != 1;
  if (M == 0 || N == 0 || d.batches == 0) return Error{};
  switch (a->dtype) {
    case TRS_F32: return launch_matmul<float>(d, stream);
    case TRS_F64: return launch_matmul<double>(d, stream);
    case TRS_I32: return launch_matmul<int32_t>(d, stream);
    case TRS_I64: return launch_matmul<int64_t>(d, stream);
  }
  return make_error(TRS_ERR_DTYPE, "unknown dtype");
}

// unfold_dims (conv.rs:490-510) and the window geometry.
Error cols_setup(const char* fn, const trs_view* img, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, ColsDev* d) {
  const std::string f(fn);
  if (sh <= 0 || sw <= 0) return make_error(TRS_ERR_ARG, "!!!" + f + "(): stride must be positive!!!");
  if (kh < 0 || kw < 0 || ph < 0 || pw < 0)
    return make_error(TRS_ERR_ARG, "!!!" + f + "(): kernel and padding must be non-negative!!!");
  const int64_t H = img->shape[2], W = img->shape[3];
  if (H + 2 * ph < kh || W + 2 * pw < kw)
    return make_error(TRS_ERR_SHAPE, "!!!" + f + "(): a (" + std::to_string((long long)kh) + ", " +
                                         std::to_string((long long)kw) + ") kernel does not fit a " +
                                         std::to_string((long long)H) + "x" + std::to_string((long long)W) +
                                         " input padded by (" + std::to_string((long long)ph) + ", " +
                                         std::to_string((long long)pw) + ")!!!");
  std::memset(d, 0, sizeof(*d));
  d->B = img->shape[0];
  d->C = img->shape[1];
  d->H = H;
  d->W = W;
  d->kh = kh;
  d->kw = kw;
  d->sh = sh;
  d->sw = sw;
  d->ph = ph;
  d->pw = pw;
  d->OH = (H + 2 * ph - kh) / sh + 1;
  d->OW = (W + 2 * pw - kw) / sw + 1;
  d->patch = d->C * kh * kw;
  d->rows = d->B * d->OH * d->OW;
  d->x_off = img->offset;
  d->x_len = img->storage_len;
  for (int i = 0; i < 4; ++i) d->xs[i] = img->strides[i];
  // the kernels decode indices in 32 bits
  const uint64_t lim = 1ull << 32;
  if ((uint64_t)d->rows * (uint64_t)d->patch >= lim || (uint64_t)(d->B * d->C * H * W) >= lim ||
      (uint64_t)(H + 2 * ph) >= lim || (uint64_t)(W + 2 * pw) >= lim)
    return make_error(TRS_ERR_SHAPE, "!!!" + f + "(): more than 2^32 - 1 elements!!!");
  if (d->patch > 0 && d->rows > 0) {
    d->f_patch = make_fastdiv((uint32_t)d->patch);
    d->f_kk = make_fastdiv((uint32_t)(kh * kw > 0 ? kh * kw : 1));
    d->f_kw = make_fastdiv((uint32_t)(kw > 0 ? kw : 1));
    d->f_ow = make_fastdiv((uint32_t)d->OW);
    d->f_oh = make_fastdiv((uint32_t)d->OH);
  }
  if (H > 0 && W > 0 && d->C > 0) {
    d->f_w = make_fastdiv((uint32_t)W);
    d->f_h = make_fastdiv((uint32_t)H);
    d->f_c = make_fastdiv((uint32_t)d->C);
  }
  d->f_sh = make_fastdiv((uint32_t)sh);
  d->f_sw = make_fastdiv((uint32_t)sw);
  return Error{};
}

unsigned cols_grid(const void* kernel, uint64_t items) {
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(kernel, kThreads, 0);
  const uint64_t need = (items + kThreads - 1) / kThreads;
  return (unsigned)(need < cap ? (need < 1 ? 1 : need) : cap);
}

// Shared memory a fold tile may take: five CTAs per SM.
constexpr int64_t kFoldSmemBudget = 44 * 1024;

// The largest band of output rows (8, 4, 2 or 1), then the most channels (up
// to 4), whose windows fit kFoldSmemBudget; false if none does.
bool pick_fold_tile(const ColsDev& d, int es, FoldTile* t) {
  if (d.B <= 0 || d.C <= 0 || d.H <= 0 || d.W <= 0 || d.OH <= 0 || d.OW <= 0) return false;
  for (int ty = 8; ty >= 1; ty /= 2) {
    if (ty > 1 && ty >= 2 * d.H) continue;
    for (int cb = 4; cb >= 1; cb /= 2) {
      if (cb > 1 && cb >= 2 * d.C) continue;
      const int64_t noh = (ty + d.kh - 1 + d.sh - 1) / d.sh;
      const int64_t seg = cb * d.kh * d.kw, segp = seg | 1;
      if (noh * d.OW * segp * es > kFoldSmemBudget) continue;
      t->CB = cb;
      t->TY = ty;
      t->noh = (int32_t)noh;
      t->seg = (int32_t)seg;
      t->segp = (int32_t)segp;
      t->n_cb = (int32_t)((d.C + cb - 1) / cb);
      t->n_yb = (int32_t)((d.H + ty - 1) / ty);
      t->tiles = d.B * t->n_cb * t->n_yb;
      if (t->tiles >= (1ll << 32) || (uint64_t)d.C * (uint64_t)ty * (uint64_t)d.W >= (1ull << 31)) return false;
      t->f_seg = make_fastdiv((uint32_t)seg);
      t->f_ty = make_fastdiv((uint32_t)ty);
      t->f_yb = make_fastdiv((uint32_t)t->n_yb);
      t->f_cb = make_fastdiv((uint32_t)t->n_cb);
      return true;
    }
  }
  return false;
}

// Shared memory an unfold-by-rows tile aims at (eight CTAs of 256 threads per
// SM) and the most it may take (one channel's kh image rows).
#ifndef TRS_UNFOLD_ROWS_TARGET
#define TRS_UNFOLD_ROWS_TARGET (12 * 1024)
#endif
constexpr int64_t kUnfoldRowsMax = 48 * 1024;

// With TMA staging, the shared stride (elements) between window rows i: CB
// channel rows of ws elements rounded up to 128 bytes, since every TMA
// destination in shared memory starts on a 128-byte boundary.
int64_t unfold_row_stride(int64_t CB, int64_t ws, int es) {
  const int64_t a = 128 / es;
  return (CB * ws + a - 1) / a * a;
}

// Bank conflicts of unfold_rows_kernel's shared loads for a full tile of CB
// channels with strides CS (channel) and IS (window row i): for the first
// warps and each of the V loads, the most distinct 4-byte words that share a
// bank, summed.
int64_t unfold_bank_conflicts(int64_t CB, int64_t kh, int64_t kw, int v, int64_t CS, int64_t IS, int64_t sw, int es) {
  const int64_t kk = kh * kw, G = CB * kk / v;
  const int64_t step = G <= kThreads ? kThreads / G : 1, n_slots = G <= kThreads ? step * G : G;
  int64_t total = 0;
  for (int64_t w = 0; w < 8 && w * 32 < n_slots; ++w) {
    for (int k = 0; k < v; ++k) {
      int64_t words[64];
      int n = 0;
      for (int64_t l = 0; l < 32 && w * 32 + l < n_slots; ++l) {
        const int64_t gi = w * 32 + l, g = G <= kThreads ? gi % G : gi, ow = G <= kThreads ? gi / G : 0;
        const int64_t col = g * v + k, cl = col / kk, r = col % kk, i = r / kw, j = r % kw;
        const int64_t a = (cl * CS + i * IS + j + ow * sw) * es / 4;
        for (int h = 0; h < es / 4; ++h) words[n++] = a + h;
      }
      std::sort(words, words + n);
      n = (int)(std::unique(words, words + n) - words);
      int per_bank[32] = {0}, worst = 0;
      for (int x = 0; x < n; ++x) {
        const int c = ++per_bank[((words[x] % 32) + 32) % 32];
        worst = c > worst ? c : worst;
      }
      total += worst;
    }
  }
  return total;
}

// The unfold-by-rows tile.  The columns' entries must be contiguous within a
// row; V entries per store when every row start and every channel block is
// V-aligned (V = 16 bytes / element), else 1.  *tma: the image is staged by
// TMA (unit x stride, the other strides positive multiples of 16 bytes, a
// 16-byte aligned start, box extents within 256).  False when one channel's
// image rows do not fit kUnfoldRowsMax or an index leaves 31 bits.
bool pick_unfold_rows(const ColsDev& d, int es, int* V, bool* tma, UnfoldRows* u) {
  if (d.cs[1] != 1 || d.rows <= 0 || d.patch <= 0 || d.OW <= 0 || d.kh <= 0 || d.kw <= 0) return false;
  if (d.B * d.OH * d.C >= (1ll << 32) || d.patch >= (1ll << 30) || d.OW * d.patch >= (1ll << 31)) return false;
  const int64_t kk = d.kh * d.kw, Wp = (d.OW - 1) * d.sw + d.kw, unit = 16 / es;
  const int64_t xo_t = (d.pw + unit - 1) / unit * unit, ws_t = (xo_t - d.pw + Wp + unit - 1) / unit * unit;
  bool t = d.xs[3] == 1 && d.kh <= 256 && ws_t <= 256 && d.H < (1ll << 31) && d.W < (1ll << 31);
  for (int i = 0; t && i < 3; ++i) t = d.xs[i] > 0 && (d.xs[i] * es) % 16 == 0 && d.xs[i] * es < (1ll << 40);
  t = t && (reinterpret_cast<uintptr_t>(d.src) + (uintptr_t)(d.x_off * es)) % 16 == 0;
  const int64_t xo = t ? xo_t : d.pw, Ws = t ? ws_t : Wp, row_bytes = d.kh * Ws * es;
  if (row_bytes > kUnfoldRowsMax || Ws * d.kh * 256 >= (1ll << 31)) return false;
  int v = (int)unit;
  if (d.patch % v != 0 || d.cs[0] % v != 0 || d.c_off % v != 0 || reinterpret_cast<uintptr_t>(d.dst) % 16 != 0)
    v = 1;
  int64_t cb_max = TRS_UNFOLD_ROWS_TARGET / row_bytes;
  if (cb_max < 1) cb_max = 1;
  if (t && cb_max > 256) cb_max = 256;  // the box's channel extent
  int64_t n_cb = (d.C + cb_max - 1) / cb_max;
  int64_t CB = (d.C + n_cb - 1) / n_cb;
  if (v > 1 && n_cb > 1 && (CB * kk) % v != 0) {
    // channel blocks whose entry count is a multiple of V
    int64_t m = 1;
    while ((m * kk) % v != 0) ++m;
    const int64_t up = (CB + m - 1) / m * m;
    if (up * row_bytes <= kUnfoldRowsMax && (!t || up <= 256))
      CB = up;
    else
      v = 1;
    n_cb = (d.C + CB - 1) / CB;
  }
  int64_t ws = Ws;
  if (t) {
    // the staged width (a whole number of 16-byte units, at most 32 words
    // wider) whose shared loads meet the fewest bank conflicts, found once per
    // geometry
    static std::mutex mu;
    static std::map<std::array<int64_t, 7>, int64_t> chosen;
    const std::array<int64_t, 7> key = {CB, d.kh, d.kw, (int64_t)v, Ws, d.sw, (int64_t)es};
    std::lock_guard<std::mutex> lock(mu);
    auto it = chosen.find(key);
    if (it != chosen.end()) {
      ws = it->second;
    } else {
      int64_t best = -1;
      for (int64_t w = Ws; w < Ws + 32 && w <= 256 && d.kh * unfold_row_stride(CB, w, es) * es <= kUnfoldRowsMax;
           w += unit) {
        const int64_t c = unfold_bank_conflicts(CB, d.kh, d.kw, v, w, unfold_row_stride(CB, w, es), d.sw, es);
        if (best < 0 || c < best) best = c, ws = w;
      }
      chosen[key] = ws;
    }
  }
  *V = v;
  *tma = t;
  u->CB = (int32_t)CB;
  u->n_cb = (int32_t)n_cb;
  u->Ws = (int32_t)ws;
  u->xo = (int32_t)xo;
  u->CS = (int32_t)(t ? ws : d.kh * ws);
  u->IS = (int32_t)(t ? unfold_row_stride(CB, ws, es) : ws);
  u->tiles = (uint32_t)(d.B * d.OH * n_cb);
  u->f_ncb = make_fastdiv((uint32_t)n_cb);
  u->f_oh = make_fastdiv((uint32_t)d.OH);
  u->f_ws = make_fastdiv((uint32_t)ws);
  u->f_kh = make_fastdiv((uint32_t)d.kh);
  return true;
}

// Widest strip of image columns a stride-1 fold tile takes: narrower strips
// let taller bands fit (fewer window rows staged twice) and more CTAs share an
// SM, for a few more windows staged twice at the strips' edges.
#ifndef TRS_FOLD_XS_MAX
#define TRS_FOLD_XS_MAX 32
#endif

// Shared memory a stride-1 fold tile may take.
#ifndef TRS_FOLD_S1_BUDGET
#define TRS_FOLD_S1_BUDGET (52 * 1024)
#endif

// The stride-1 fold tile: channel blocks whose entries are a whole number of
// 16-byte units (the TMA box's inner extent and start; m channels, or 2m),
// at most 256 entries and 256 windows per box; within the budget the widest
// strip of columns, then the tallest band (8, 4, 2 or 1 rows: the band's
// window rows are staged (TY + kh - 1) / TY times), then 2m channels.  False
// when the columns cannot be a TMA tensor (entries not contiguous, a row
// stride or base not 16-byte aligned) or no tile fits.
bool pick_fold_s1(const ColsDev& d, int es, FoldS1* f) {
  if (d.sh != 1 || d.sw != 1 || d.kh < 1 || d.kw < 1 || d.cs[1] != 1) return false;
  if (d.B <= 0 || d.C <= 0 || d.H <= 0 || d.W <= 0 || d.OH <= 0 || d.OW <= 0) return false;
  if (d.cs[0] <= 0 || (d.cs[0] * es) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(d.src) + (uintptr_t)(d.c_off * es)) % 16 != 0)
    return false;
  if (d.patch >= (1ll << 31) || d.B >= (1ll << 31) || d.H >= (1ll << 30) || d.W >= (1ll << 30)) return false;
  if ((uint64_t)d.cs[0] * (uint64_t)es * (uint64_t)d.OW * (uint64_t)d.OH >= (1ull << 40)) return false;  // TMA strides
  const int64_t kk = d.kh * d.kw;
  int64_t m = 1;
  while ((m * kk * es) % 16 != 0) ++m;
  if (m * kk > 256 || d.kw > 128 || m > d.C) return false;
  // strips of at most TRS_FOLD_XS_MAX columns, of equal widths
  const int64_t xs_cap = d.W + d.kw - 1 <= 256 ? d.W : 256 - (d.kw - 1);
  const int64_t xs_max = xs_cap < TRS_FOLD_XS_MAX ? xs_cap : TRS_FOLD_XS_MAX;
  const int64_t n_strips = (d.W + xs_max - 1) / xs_max;
  const int64_t xs_opts[2] = {(d.W + n_strips - 1) / n_strips, d.W < 64 ? d.W : 64};
  for (const int64_t XS : xs_opts) {
    for (int ty = 8; ty >= 1; ty /= 2) {
      if (ty > 1 && ty >= 2 * d.H) continue;
      for (int64_t CB = 2 * m; CB >= m; CB -= m) {
        if (CB > m && (CB * kk > 256 || CB > d.C)) continue;
        const int64_t Q = XS + d.kw - 1, seg = CB * kk, align = 128 / es;
        const int64_t RS = (Q * seg + align - 1) / align * align, R = ty + d.kh - 1;
        if (R * RS * es > TRS_FOLD_S1_BUDGET) continue;
        const int64_t n_cb = (d.C + CB - 1) / CB, n_yb = (d.H + ty - 1) / ty, n_xb = (d.W + XS - 1) / XS;
        if (d.B * n_cb * n_yb * n_xb >= (1ll << 32)) return false;
        f->CB = (int32_t)CB;
        f->TY = ty;
        f->XS = (int32_t)XS;
        f->R = (int32_t)R;
        f->Q = (int32_t)Q;
        f->seg = (int32_t)seg;
        f->RS = (int32_t)RS;
        f->tiles = (uint32_t)(d.B * n_cb * n_yb * n_xb);
        f->f_cb = make_fastdiv((uint32_t)CB);
        f->f_nxb = make_fastdiv((uint32_t)n_xb);
        f->f_nyb = make_fastdiv((uint32_t)n_yb);
        f->f_ncb = make_fastdiv((uint32_t)n_cb);
        return true;
      }
    }
  }
  return false;
}

template <class T>
Error launch_fold_s1(const ColsDev& d, const FoldS1& f, cudaStream_t stream) {
  // the columns [B*OH*OW, patch] as [B][OH][OW][patch] (row stride cs0)
  const cuuint64_t rs = (cuuint64_t)d.cs[0] * sizeof(T);
  CUtensorMap map;
  Error e = make_map_4d<T>("fold_2d", static_cast<const T*>(d.src) + d.c_off,
                           {(cuuint64_t)d.patch, (cuuint64_t)d.OW, (cuuint64_t)d.OH, (cuuint64_t)d.B},
                           {rs, rs * (cuuint64_t)d.OW, rs * (cuuint64_t)d.OW * (cuuint64_t)d.OH},
                           {(cuuint32_t)f.seg, (cuuint32_t)f.Q, 1, 1}, &map);
  if (!e.ok()) return e;
  const int smem = (int)((int64_t)f.R * f.RS * (int64_t)sizeof(T)) + 8 + 128;  // rows, mbarrier, alignment
  constexpr int kSeg3 = sizeof(T) == 4 ? 36 : 18;  // 3x3 windows of the fewest channels a TMA box allows
  const int form = (d.kh == 3 && d.kw == 3) ? (f.seg == kSeg3 ? 2 : 1) : 0;
  const void* k = form == 2 ? (const void*)fold_s1_kernel<T, 3, kSeg3>
                : form == 1 ? (const void*)fold_s1_kernel<T, 3, 0> : (const void*)fold_s1_kernel<T, 0, 0>;
  allow_smem(k, smem);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, kThreads, smem);
  const unsigned g = (unsigned)((uint64_t)f.tiles < cap * 64 ? (uint64_t)f.tiles : cap * 64);
  int* err = async_error_word();
  if (form == 2)
    fold_s1_kernel<T, 3, kSeg3><<<g, kThreads, smem, stream>>>(map, d, f, err);
  else if (form == 1)
    fold_s1_kernel<T, 3, 0><<<g, kThreads, smem, stream>>>(map, d, f, err);
  else
    fold_s1_kernel<T, 0, 0><<<g, kThreads, smem, stream>>>(map, d, f, err);
  return check_launch("fold_2d kernel");
}

template <class T>
Error launch_unfold_rows(const ColsDev& d, int V, bool tma, const UnfoldRows& u, cudaStream_t stream) {
  constexpr int kV = (int)(16 / sizeof(T));
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if (tma) {
    // the image as [B][C][H][W]: boxes [Ws, 1, CB, 1], one per window row
    const cuuint64_t es = sizeof(T);
    Error e = make_map_4d<T>("unfold_2d", static_cast<const T*>(d.src) + d.x_off,
                             {(cuuint64_t)d.W, (cuuint64_t)d.H, (cuuint64_t)d.C, (cuuint64_t)d.B},
                             {(cuuint64_t)d.xs[2] * es, (cuuint64_t)d.xs[1] * es, (cuuint64_t)d.xs[0] * es},
                             {(cuuint32_t)u.Ws, 1, (cuuint32_t)u.CB, 1}, &map);
    if (!e.ok()) return e;
  }
  const int64_t stage = tma ? d.kh * (int64_t)u.IS : (int64_t)u.CB * u.CS;
  const int smem = (int)((stage * (int64_t)sizeof(T) + 7) / 8 * 8) + 8 + 128;  // rows, mbarrier, alignment
  const void* k = tma ? (V > 1 ? (const void*)unfold_rows_kernel<T, kV, true> : (const void*)unfold_rows_kernel<T, 1, true>)
                      : (V > 1 ? (const void*)unfold_rows_kernel<T, kV, false> : (const void*)unfold_rows_kernel<T, 1, false>);
  allow_smem(k, smem);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, kThreads, smem);
  const unsigned g = (unsigned)((uint64_t)u.tiles < cap * 64 ? (uint64_t)u.tiles : cap * 64);
  int* err = async_error_word();
  if (tma && V > 1)
    unfold_rows_kernel<T, kV, true><<<g, kThreads, smem, stream>>>(map, d, u, err);
  else if (tma)
    unfold_rows_kernel<T, 1, true><<<g, kThreads, smem, stream>>>(map, d, u, err);
  else if (V > 1)
    unfold_rows_kernel<T, kV, false><<<g, kThreads, smem, stream>>>(map, d, u, err);
  else
    unfold_rows_kernel<T, 1, false><<<g, kThreads, smem, stream>>>(map, d, u, err);
  return check_launch("unfold_2d kernel");
}

// Tuning knob: 0 keeps the earlier tile kernels for every geometry.
#ifndef TRS_COLS_ROWS
#define TRS_COLS_ROWS 1
#endif

template <class T>
Error launch_cols(bool unfold, const ColsDev& d, cudaStream_t stream) {
  if (TRS_COLS_ROWS && !unfold) {
    FoldS1 f;
    if (pick_fold_s1(d, (int)sizeof(T), &f)) return launch_fold_s1<T>(d, f, stream);
  }
  if (TRS_COLS_ROWS && unfold) {
    UnfoldRows u;
    int V = 1;
    bool tma = false;
    if (pick_unfold_rows(d, (int)sizeof(T), &V, &tma, &u)) return launch_unfold_rows<T>(d, V, tma, u, stream);
  }
  if (!unfold) {
    FoldTile ft;
    if (pick_fold_tile(d, (int)sizeof(T), &ft)) {
      const int smem = (int)((int64_t)ft.noh * d.OW * ft.segp * (int64_t)sizeof(T));
      // windows covering a pixel, per dimension: the unrolled form up to 3
      const bool unrolled = (d.kh + d.sh - 1) / d.sh <= 3 && (d.kw + d.sw - 1) / d.sw <= 3;
      const bool i32 = (uint64_t)d.c_len < (1ull << 31) && (uint64_t)d.x_len < (1ull << 31);
      const void* k = unrolled ? (i32 ? (const void*)fold_smem_kernel<T, 3, true> : (const void*)fold_smem_kernel<T, 3, false>)
                               : (i32 ? (const void*)fold_smem_kernel<T, 0, true> : (const void*)fold_smem_kernel<T, 0, false>);
      const uint64_t cap =
          (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, kThreads, smem);
      const unsigned g = (unsigned)((uint64_t)ft.tiles < cap ? (uint64_t)ft.tiles : cap);
      if (unrolled && i32)
        fold_smem_kernel<T, 3, true><<<g, kThreads, smem, stream>>>(d, ft);
      else if (unrolled)
        fold_smem_kernel<T, 3, false><<<g, kThreads, smem, stream>>>(d, ft);
      else if (i32)
        fold_smem_kernel<T, 0, true><<<g, kThreads, smem, stream>>>(d, ft);
      else
        fold_smem_kernel<T, 0, false><<<g, kThreads, smem, stream>>>(d, ft);
      return check_launch("fold_2d kernel");
    }
  }
  if (unfold) {
    if (d.rows == 0 || d.patch == 0) return Error{};
    // the transposed tile when the patch's column table fits (patch <= 2048,
    // i and j in 16 bits) and every table offset is within 31 bits
    const uint64_t max_off = (uint64_t)std::llabs(d.xs[1]) * (uint64_t)(d.C > 0 ? d.C - 1 : 0) +
                             (uint64_t)std::llabs(d.xs[2]) * (uint64_t)(d.kh > 0 ? d.kh - 1 : 0) +
                             (uint64_t)std::llabs(d.xs[3]) * (uint64_t)(d.kw > 0 ? d.kw - 1 : 0);
    if (d.patch <= kUnfoldTab && d.kh < 65536 && d.kw < 65536 && max_off < (1ull << 31) &&
        d.rows < (1ll << 32) - kUtRows) {
      // 32-bit indices when the image's and the columns' storage, with the
      // padding's reach before the image, stay below 2^31 elements
      const uint64_t pad = (uint64_t)std::llabs(d.xs[2]) * (uint64_t)d.ph + (uint64_t)std::llabs(d.xs[3]) * (uint64_t)d.pw;
      const bool i32 = (uint64_t)d.x_len + max_off + pad < (1ull << 31) && (uint64_t)d.c_len < (1ull << 31);
      const void* kt = i32 ? (const void*)unfold_tile_kernel<T, true> : (const void*)unfold_tile_kernel<T, false>;
      const uint64_t tiles =
          (((uint64_t)d.rows + kUtRows - 1) / kUtRows) * (((uint64_t)d.patch + kUtCols - 1) / kUtCols);
      const uint64_t cap =
          (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(kt, kThreads, 0);
      const unsigned g = (unsigned)(tiles < cap ? tiles : cap);
      if (i32)
        unfold_tile_kernel<T, true><<<g, kThreads, 0, stream>>>(d);
      else
        unfold_tile_kernel<T, false><<<g, kThreads, 0, stream>>>(d);
      return check_launch("unfold_2d kernel");
    }
    const uint64_t items = ((uint64_t)d.rows * (uint64_t)d.patch + kColsU - 1) / kColsU;
    unfold_kernel<T><<<cols_grid((const void*)unfold_kernel<T>, items), kThreads, 0, stream>>>(d);
    return check_launch("unfold_2d kernel");
  }
  // windows that can cover one pixel: ceil(kh / sh) * ceil(kw / sw)
  const int64_t cover = ((d.kh + d.sh - 1) / d.sh) * ((d.kw + d.sw - 1) / d.sw);
  const bool regs = cover <= kFoldRegs;
  const uint64_t items = (uint64_t)(d.B * d.C * d.H * d.W);
  if (items == 0) return Error{};
  const void* k = regs ? (const void*)fold_kernel<T, true> : (const void*)fold_kernel<T, false>;
  const unsigned g = cols_grid(k, items);
  if (regs)
    fold_kernel<T, true><<<g, kThreads, 0, stream>>>(d);
  else
    fold_kernel<T, false><<<g, kThreads, 0, stream>>>(d);
  return check_launch("fold_2d kernel");
}

Error dispatch_cols(bool unfold, int dt, const ColsDev& d, cudaStream_t stream) {
  switch (dt) {
    case TRS_F32: return launch_cols<float>(unfold, d, stream);
    case TRS_F64: return launch_cols<double>(unfold, d, stream);
    case TRS_I32: return launch_cols<int32_t>(unfold, d, stream);
    case TRS_I64: return launch_cols<int64_t>(unfold, d, stream);
  }
  return make_error(TRS_ERR_DTYPE, "unknown dtype");
}

Error run_unfold(const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                 const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(x, "x");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (x->ndim != 4)
    return make_error(TRS_ERR_SHAPE, "!!!unfold_2d() expects [batch, channels, height, width], got " +
                                         shape_str(x->shape, x->ndim) + "!!!");
  if (out->dtype != x->dtype) return make_error(TRS_ERR_DTYPE, "unfold_2d: the output dtype differs from x");
  ColsDev d;
  e = cols_setup("unfold_2d", x, kh, kw, sh, sw, ph, pw, &d);
  if (!e.ok()) return e;
  if (out->ndim != 2 || out->shape[0] != d.rows || out->shape[1] != d.patch) {
    const int64_t want[2] = {d.rows, d.patch};
    return make_error(TRS_ERR_SHAPE, "unfold_2d: the output must have shape " + shape_str(want, 2));
  }
  if (ranges_overlap(out, x)) return make_error(TRS_ERR_ALIAS, "unfold_2d: the output overlaps x");
  d.src = x->data;
  d.dst = out->data;
  d.c_off = out->offset;
  d.c_len = out->storage_len;
  d.cs[0] = out->strides[0];
  d.cs[1] = out->strides[1];
  return dispatch_cols(true, x->dtype, d, stream);
}

Error run_fold(const trs_view* cols, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
               const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(cols, "cols");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (out->ndim != 4) return make_error(TRS_ERR_SHAPE, "fold_2d: the output must be [batch, channels, height, width]");
  if (out->dtype != cols->dtype) return make_error(TRS_ERR_DTYPE, "fold_2d: the output dtype differs from cols");
  if (sh <= 0 || sw <= 0) return make_error(TRS_ERR_ARG, "!!!fold_2d(): stride must be positive!!!");
  ColsDev d;
  e = cols_setup("fold_2d", out, kh, kw, sh, sw, ph, pw, &d);
  const bool fits = e.ok() && cols->ndim == 2 && cols->shape[0] == d.rows && cols->shape[1] == d.patch;
  if (!fits)
    return make_error(TRS_ERR_SHAPE, "!!!fold_2d(): shape " + shape_str(cols->shape, cols->ndim) +
                                         " does not match an unfold of " + shape_str(out->shape, 4) + "!!!");
  if (ranges_overlap(out, cols)) return make_error(TRS_ERR_ALIAS, "fold_2d: the output overlaps cols");
  d.src = cols->data;
  d.dst = out->data;
  d.c_off = cols->offset;
  d.c_len = cols->storage_len;
  d.cs[0] = cols->strides[0];
  d.cs[1] = cols->strides[1];
  d.step_oh = d.OW * d.cs[0] - d.sh * d.kw * d.cs[1];
  d.step_ow = d.cs[0] - d.sw * d.cs[1];
  return dispatch_cols(false, cols->dtype, d, stream);
}

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

}  // namespace
}  // namespace trs

extern "C" {

trs_status trs_matmul(const trs_view* a, const trs_view* b, trs_view* out, trs_stream stream) {
  if (!a || !b || !out) return trs::finish(trs::make_error(TRS_ERR_ARG, "null view"));
  return trs::finish(trs::run_matmul(a, b, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_unfold_2d(const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                         trs_view* out, trs_stream stream) {
  if (!x || !out) return trs::finish(trs::make_error(TRS_ERR_ARG, "null view"));
  return trs::finish(trs::run_unfold(x, kh, kw, sh, sw, ph, pw, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_fold_2d(const trs_view* cols, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                       trs_view* out, trs_stream stream) {
  if (!cols || !out) return trs::finish(trs::make_error(TRS_ERR_ARG, "null view"));
  return trs::finish(trs::run_fold(cols, kh, kw, sh, sw, ph, pw, out, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
