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
#include <cstring>
#include <string>

#include "kernels.cuh"

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
  int64_t c_off, cs[2];   // the columns ([B*OH*OW, C*kh*kw] view): unfold's output, fold's input
  int64_t patch, rows;
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
    auto at = [&](int32_t oh, int32_t ow) {
      const int32_t i = yp - oh * sh, j = xp - ow * sw;
      const int64_t row = ((int64_t)b * OH + oh) * OW + ow, col = ((int64_t)c * kh + i) * kw + j;
      return d.c_off + row * d.cs[0] + col * d.cs[1];
    };
    T acc = T(0);
    if constexpr (REGS) {
      const int32_t cnt = (oh_hi >= oh_lo && nw > 0) ? (oh_hi - oh_lo + 1) * nw : 0;
      T v[kFoldRegs];
      int32_t oh = oh_lo, ow = ow_lo;  // window w = (oh, ow), row-major over the covering range
#pragma unroll
      for (int w = 0; w < kFoldRegs; ++w) {
        v[w] = T(0);
        if (w < cnt) {
          v[w] = cols[at(oh, ow)];
          if (++ow > ow_hi) {
            ow = ow_lo;
            ++oh;
          }
        }
      }
#pragma unroll
      for (int w = 0; w < kFoldRegs; ++w)
        if (w < cnt) acc = A::add(acc, v[w]);  // windows in (oh, ow) order
    } else {
      for (int32_t oh = oh_lo; oh <= oh_hi; ++oh)
        for (int32_t ow = ow_lo; ow <= ow_hi; ++ow) acc = A::add(acc, cols[at(oh, ow)]);
    }
    out[d.x_off + (int64_t)b * d.xs[0] + (int64_t)c * d.xs[1] + (int64_t)y * d.xs[2] + (int64_t)xx * d.xs[3]] = acc;
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

template <class T>
Error launch_cols(bool unfold, const ColsDev& d, cudaStream_t stream) {
  // windows that can cover one pixel: ceil(kh / sh) * ceil(kw / sw)
  const int64_t cover = ((d.kh + d.sh - 1) / d.sh) * ((d.kw + d.sw - 1) / d.sw);
  const bool regs = cover <= kFoldRegs;
  const void* k = unfold ? (const void*)unfold_kernel<T>
                         : (regs ? (const void*)fold_kernel<T, true> : (const void*)fold_kernel<T, false>);
  const uint64_t items = unfold ? ((uint64_t)d.rows * (uint64_t)d.patch + kColsU - 1) / kColsU
                                : (uint64_t)(d.B * d.C * d.H * d.W);
  if (items == 0) return Error{};
  const unsigned g = cols_grid(k, items);
  if (unfold)
    unfold_kernel<T><<<g, kThreads, 0, stream>>>(d);
  else if (regs)
    fold_kernel<T, true><<<g, kThreads, 0, stream>>>(d);
  else
    fold_kernel<T, false><<<g, kThreads, 0, stream>>>(d);
  return check_launch(unfold ? "unfold_2d kernel" : "fold_2d kernel");
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
  d.cs[0] = cols->strides[0];
  d.cs[1] = cols->strides[1];
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
