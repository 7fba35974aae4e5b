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
//   * K advances in BK-deep slabs; the next slab of A and B is loaded from
//     global memory into registers while the current one is multiplied out of
//     shared memory (two buffers), with coalesced loads chosen by which
//     dimension of each operand is unit-stride;
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

template <class T>
__global__ void __launch_bounds__(kThreads, std::is_same<T, double>::value ? 2 : 1) matmul_kernel(const MmDev d) {
  constexpr int TM = MmTile<T>::TM, TN = MmTile<T>::TN, BK = MmTile<T>::BK;
  constexpr int BM = 16 * TM, BN = 16 * TN;
  constexpr int LA = BM * BK / kThreads, LB = BN * BK / kThreads;
  constexpr int PAD = 16 / (int)sizeof(T);  // keeps each shared row 16-byte aligned
  __shared__ __align__(16) T As[2][BK][BM + PAD];
  __shared__ __align__(16) T Bs[2][BK][BN + PAD];
  const T* ga = static_cast<const T*>(d.a);
  const T* gb = static_cast<const T*>(d.b);
  T* go = static_cast<T*>(d.out);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  // slot q of this thread in a slab: element e = tid + q * 256, laid out so
  // consecutive threads read consecutive addresses of the unit-stride dimension
  auto a_row = [&](int q) { const int e = threadIdx.x + q * kThreads; return d.a_kfast ? e / BK : e % BM; };
  auto a_kk = [&](int q) { const int e = threadIdx.x + q * kThreads; return d.a_kfast ? e % BK : e / BM; };
  auto b_col = [&](int q) { const int e = threadIdx.x + q * kThreads; return d.b_nfast ? e % BN : e / BK; };
  auto b_kk = [&](int q) { const int e = threadIdx.x + q * kThreads; return d.b_nfast ? e / BN : e % BK; };

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
    T ra[LA], rb[LB];
    auto fetch = [&](int64_t k0) {
#pragma unroll
      for (int q = 0; q < LA; ++q) {
        const int64_t row = m0 + a_row(q), k = k0 + a_kk(q);
        ra[q] = (row < d.M && k < d.K) ? ga[ao + row * d.sam + k * d.sak] : T(0);
      }
#pragma unroll
      for (int q = 0; q < LB; ++q) {
        const int64_t col = n0 + b_col(q), k = k0 + b_kk(q);
        rb[q] = (col < d.N && k < d.K) ? gb[bo + k * d.sbk + col * d.sbn] : T(0);
      }
    };
    auto stash = [&](int buf) {
#pragma unroll
      for (int q = 0; q < LA; ++q) As[buf][a_kk(q)][a_row(q)] = ra[q];
#pragma unroll
      for (int q = 0; q < LB; ++q) Bs[buf][b_kk(q)][b_col(q)] = rb[q];
    };

    AccTile<T, TM, TN> acc;  // +0: T::default() of the reference
    acc.zero();
    fetch(0);
    __syncthreads();  // the previous batch's last slab has been read
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int64_t k0 = 0; k0 < d.K; k0 += BK, buf ^= 1) {
      const bool more = k0 + BK < d.K;
      if (more) fetch(k0 + BK);  // in flight while this slab is multiplied
      const int kmax = d.K - k0 < BK ? (int)(d.K - k0) : BK;
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        if (kk < kmax) {  // k walks 0 .. K-1 in order, one step per kk
          T av[TM], bv[TN];
#pragma unroll
          for (int i = 0; i < TM; ++i) av[i] = As[buf][kk][ty * TM + i];
#pragma unroll
          for (int j = 0; j < TN; ++j) bv[j] = Bs[buf][kk][tx * TN + j];
          acc.step(av, bv);
        }
      }
      if (more) {
        stash(buf ^ 1);
        __syncthreads();
      }
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t row = m0 + ty * TM + i;
      if (row >= d.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t col = n0 + tx * TN + j;
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
};

// one thread per element of the columns, row-major
template <class T>
__global__ void __launch_bounds__(kThreads) unfold_kernel(const ColsDev d) {
  const T* x = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const uint64_t n = (uint64_t)d.rows * (uint64_t)d.patch;
  const uint64_t step = (uint64_t)gridDim.x * kThreads;
  for (uint64_t idx = (uint64_t)blockIdx.x * kThreads + threadIdx.x; idx < n; idx += step) {
    const int64_t row = (int64_t)(idx / (uint64_t)d.patch), col = (int64_t)(idx - (uint64_t)row * d.patch);
    const int64_t ow = row % d.OW, oh = (row / d.OW) % d.OH, b = row / (d.OW * d.OH);
    const int64_t kk = d.kh * d.kw;
    const int64_t c = col / kk, r = col - c * kk, i = r / d.kw, j = r - (r / d.kw) * d.kw;
    const int64_t y = oh * d.sh + i - d.ph, xx = ow * d.sw + j - d.pw;
    T v = T(0);
    if (y >= 0 && y < d.H && xx >= 0 && xx < d.W)
      v = x[d.x_off + b * d.xs[0] + c * d.xs[1] + y * d.xs[2] + xx * d.xs[3]];
    out[d.c_off + row * d.cs[0] + col * d.cs[1]] = v;
  }
}

// one thread per output pixel (b, c, y, x), row-major
template <class T>
__global__ void __launch_bounds__(kThreads) fold_kernel(const ColsDev d) {
  using A = Arith<T>;
  const T* cols = static_cast<const T*>(d.src);
  T* out = static_cast<T*>(d.dst);
  const uint64_t n = (uint64_t)(d.B * d.C * d.H * d.W);
  const uint64_t step = (uint64_t)gridDim.x * kThreads;
  for (uint64_t idx = (uint64_t)blockIdx.x * kThreads + threadIdx.x; idx < n; idx += step) {
    const int64_t xx = (int64_t)(idx % (uint64_t)d.W);
    const int64_t y = (int64_t)((idx / (uint64_t)d.W) % (uint64_t)d.H);
    const int64_t c = (int64_t)((idx / (uint64_t)(d.W * d.H)) % (uint64_t)d.C);
    const int64_t b = (int64_t)(idx / (uint64_t)(d.W * d.H * d.C));
    // windows whose row range holds y: oh * sh <= y + ph <= oh * sh + kh - 1
    const int64_t yp = y + d.ph, xp = xx + d.pw;
    int64_t oh_lo = yp - d.kh + 1 <= 0 ? 0 : (yp - d.kh + d.sh) / d.sh;
    int64_t oh_hi = yp / d.sh;
    if (oh_hi > d.OH - 1) oh_hi = d.OH - 1;
    int64_t ow_lo = xp - d.kw + 1 <= 0 ? 0 : (xp - d.kw + d.sw) / d.sw;
    int64_t ow_hi = xp / d.sw;
    if (ow_hi > d.OW - 1) ow_hi = d.OW - 1;
    T acc = T(0);
    for (int64_t oh = oh_lo; oh <= oh_hi; ++oh) {
      const int64_t i = yp - oh * d.sh;
      for (int64_t ow = ow_lo; ow <= ow_hi; ++ow) {
        const int64_t j = xp - ow * d.sw;
        const int64_t row = (b * d.OH + oh) * d.OW + ow, col = (c * d.kh + i) * d.kw + j;
        acc = A::add(acc, cols[d.c_off + row * d.cs[0] + col * d.cs[1]]);
      }
    }
    out[d.x_off + b * d.xs[0] + c * d.xs[1] + y * d.xs[2] + xx * d.xs[3]] = acc;
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
  return Error{};
}

unsigned cols_grid(const void* kernel, uint64_t items) {
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(kernel, kThreads, 0);
  const uint64_t need = (items + kThreads - 1) / kThreads;
  return (unsigned)(need < cap ? (need < 1 ? 1 : need) : cap);
}

template <class T>
Error launch_cols(bool unfold, const ColsDev& d, cudaStream_t stream) {
  const void* k = unfold ? (const void*)unfold_kernel<T> : (const void*)fold_kernel<T>;
  const uint64_t items = unfold ? (uint64_t)d.rows * (uint64_t)d.patch : (uint64_t)(d.B * d.C * d.H * d.W);
  if (items == 0) return Error{};
  const unsigned g = cols_grid(k, items);
  if (unfold)
    unfold_kernel<T><<<g, kThreads, 0, stream>>>(d);
  else
    fold_kernel<T><<<g, kThreads, 0, stream>>>(d);
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
