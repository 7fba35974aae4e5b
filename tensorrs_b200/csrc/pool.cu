// pool.cu -- the pooling layers of nn/pool.rs, each as one kernel.
//
// MaxPool2d::forward and AvgPool2d::forward (nn/pool.rs:137-144, 223-233)
// fold the channels into the batch (windows_per_channel, pool.rs:25-33), lay
// every window out as a row with unfold_2d (linalg/tensor/conv.rs:360-418: an
// im2col copy holding kh*kw values per output), and reduce the rows with
// max_axis (base.rs:1396-1436) or with sum_axis (base.rs:1051-1107) followed by
// a division by kh*kw.  Without padding a window is a strided view of the
// input, so each output here reads its window straight from the input: one
// read of the input and one write of the output, no im2col buffer.
//
//   pool_strip_kernel  kw == stride_w dividing 16 bytes, kh <= 4, unit-stride
//       rows aligned to 16 bytes: a thread loads one 16-byte strip per window
//       row, which holds the windows of 16 / (kw * size) neighbouring outputs.
//   pool_tile_fwd_kernel  any window and stride, rows aligned to 16 bytes: an
//       item is a block of window rows of one plane whose input rows are
//       staged once in shared memory (16-byte cp.async), then each output
//       reads its window from there.
//   pool_fwd_kernel  any other layout: one thread per output, scalar loads
//       (neighbouring threads share their rows through L1).
//   pool_max_bwd_kernel<T>  the gradient MaxPool2d passes back to its input:
//       max_axis's backward (autodiff/core.rs:352-375) gives each window's
//       gradient to the first of its largest elements (argmax_axis,
//       base.rs:1458-1505) and unfold's backward fold_2d (conv.rs:434-488)
//       sums, per pixel, the gradients of the windows that read it, in window
//       order from 0.  One thread per input pixel walks the windows covering
//       it in that order and finds each window's winner again; with
//       `accumulate` it adds the sum to the gradient already held (the
//       `current + grad` of autodiff/traits.rs:141-150).
//       pool_max_bwd_strip_kernel serves windows that tile the image (stride
//       == window, kw dividing 16 bytes) with 16-byte strips;
//       pool_max_bwd_rows_kernel serves f32 2x2 windows at stride 2 tiling
//       an image of even height and a width that is a multiple of 8, from TMA
//       boxes of x and grad_out;
//       pool_tile_bwd_kernel stages the rows of a block of window rows in
//       shared memory, finds each window's winner once, then lets each owned
//       pixel add the gradients of the covering windows it wins.
//
// Order of floating-point operations: max keeps the window's first element and
// replaces it only by a strictly greater one (a NaN first element stays); the
// average adds the window in row-major order in the element type, from +0,
// then divides once by kh*kw -- the reference's f32 / f64 operations in its
// order, so both are bit-exact.
#include <cstring>

#include "../../include/trs.h"
#include "kernels.cuh"
#include "tma.cuh"

namespace trs {
namespace {

enum PoolMode { kPoolMax = 0, kPoolAvg = 1 };

struct PoolDev {
  const void* x;
  const void* g;
  void* out;
  int64_t x_off, g_off, o_off;
  int64_t xs[4], gs[4], os[4];  // strides of [N, C, H, W] / [N, C, OH, OW]
  int64_t H, W, OH, OW;
  int32_t kh, kw, sh, sw;
  int64_t items;   // work items: outputs (or strips), or input pixels
  int64_t inner;   // items along the last axis of one row
  FastDiv f_inner, f_rows, f_c;  // items per row, rows per plane, channels
  FastDiv f_sh, f_sw;            // the window strides
  // tile kernels: blocks of R window rows per plane, input rows staged in
  // shared memory at a pitch of P elements
  int32_t R, P, nblk, full;          // full: whole 16-byte chunks per row
  FastDiv f_blk, f_ow, f_w, f_full;  // blocks per plane, OW, W, full
  int32_t fast;    // items < 2^32: 32-bit index arithmetic
  int32_t box_rows;  // TMA row kernel: input rows per item's box
  int32_t accumulate;
};

// items -> (n, c, row, col), the last one counted in items of the row.
__device__ __forceinline__ void pool_coords(const PoolDev& d, uint64_t i, int64_t* n, int64_t* c, int64_t* r,
                                            int64_t* q) {
  if (d.fast) {
    const uint32_t a = (uint32_t)i;
    const uint32_t b = fdiv(a, d.f_inner);
    const uint32_t e = fdiv(b, d.f_rows);
    const uint32_t f = fdiv(e, d.f_c);
    *q = a - b * d.f_inner.d;
    *r = b - e * d.f_rows.d;
    *c = e - f * d.f_c.d;
    *n = f;
  } else {
    const uint64_t t = i / d.f_inner.d;
    const uint64_t u = t / d.f_rows.d;
    const uint64_t v = u / d.f_c.d;
    *q = (int64_t)(i - t * d.f_inner.d);
    *r = (int64_t)(t - u * d.f_rows.d);
    *c = (int64_t)(u - v * d.f_c.d);
    *n = (int64_t)v;
  }
}

template <class T, int V>
struct alignas(sizeof(T) * V) PVec {
  T v[V];
};

// One window by scalar loads, in row-major order.
// The average's division by the window size n.  For a power of two the
// quotient x / n equals x * (1/n) exactly before rounding (1/n is exact), so
// the product rounds to the IEEE quotient bit for bit, zeros, infinities,
// NaN and subnormals included; other sizes divide.
template <class T>
__device__ __forceinline__ T pool_mean(T acc, int64_t n) {
  if ((n & (n - 1)) == 0) return Arith<T>::mul(acc, (T)(1.0 / (double)n));
  return Arith<T>::div(acc, (T)n, nullptr);
}

template <class T, int MODE>
__device__ __forceinline__ T pool_window(const T* __restrict__ x, int64_t base, const PoolDev& d) {
  using A = Arith<T>;
  if constexpr (MODE == kPoolMax) {
    T best = __ldg(x + base);
    for (int u = 0; u < d.kh; ++u)
      for (int v = (u == 0 ? 1 : 0); v < d.kw; ++v) {
        const T val = __ldg(x + base + u * d.xs[2] + v * d.xs[3]);
        if (val > best) best = val;
      }
    return best;
  } else {
    T acc = T(0);
    for (int u = 0; u < d.kh; ++u)
      for (int v = 0; v < d.kw; ++v) acc = A::add(acc, __ldg(x + base + u * d.xs[2] + v * d.xs[3]));
    return pool_mean<T>(acc, (int64_t)d.kh * d.kw);
  }
}

constexpr int kPoolItems = 2;  // strips per thread per pass of the strip kernels

// Any window: one thread per output, scalar loads.
template <class T, int MODE>
__global__ void __launch_bounds__(256) pool_fwd_kernel(const PoolDev d) {
  const T* __restrict__ x = static_cast<const T*>(d.x);
  T* __restrict__ out = static_cast<T*>(d.out);
  for (uint64_t it = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < (uint64_t)d.items;
       it += (uint64_t)gridDim.x * blockDim.x) {
    int64_t n, c, i, j;
    pool_coords(d, it, &n, &c, &i, &j);
    const int64_t base = d.x_off + n * d.xs[0] + c * d.xs[1] + i * d.sh * d.xs[2] + j * d.sw * d.xs[3];
    out[d.o_off + n * d.os[0] + c * d.os[1] + i * d.os[2] + j * d.os[3]] = pool_window<T, MODE>(x, base, d);
  }
}

// Windows KW wide at a stride of KW, at most KH high, over unit-stride rows
// aligned to 16 bytes: an item is one 16-byte strip of one row of windows,
// the windows of Q = 16 / (KW * size) neighbouring outputs.  Each thread takes
// kPoolItems strips per pass and issues all their row loads before combining.
template <class T, int MODE, int KW, int KH>
__global__ void __launch_bounds__(256) pool_strip_kernel(const PoolDev d) {
  constexpr int VW = 16 / sizeof(T);
  constexpr int Q = VW / KW;
  using A = Arith<T>;
  const T* __restrict__ x = static_cast<const T*>(d.x);
  T* __restrict__ out = static_cast<T*>(d.out);
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t it0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it0 < (uint64_t)d.items;
       it0 += kPoolItems * step) {
    int64_t row0[kPoolItems], obase[kPoolItems], col0[kPoolItems];
    bool live[kPoolItems], whole[kPoolItems];
    PVec<T, VW> s[kPoolItems][KH];
#pragma unroll
    for (int k = 0; k < kPoolItems; ++k) {
      const uint64_t it = it0 + (uint64_t)k * step;
      live[k] = it < (uint64_t)d.items;
      int64_t n = 0, c = 0, i = 0, q = 0;
      if (live[k]) pool_coords(d, it, &n, &c, &i, &q);
      row0[k] = d.x_off + n * d.xs[0] + c * d.xs[1] + i * d.sh * d.xs[2];
      obase[k] = d.o_off + n * d.os[0] + c * d.os[1] + i * d.os[2];
      col0[k] = q * VW;
      whole[k] = live[k] && col0[k] + VW <= d.W;
#pragma unroll
      for (int u = 0; u < KH; ++u)
        if (whole[k] && u < d.kh)
          s[k][u] = *reinterpret_cast<const PVec<T, VW>*>(x + row0[k] + u * d.xs[2] + col0[k]);
    }
#pragma unroll
    for (int k = 0; k < kPoolItems; ++k) {
      if (!live[k]) continue;
      const int64_t j0 = col0[k] / KW;  // the strip's first output
      if (whole[k]) {
        T r[Q];
#pragma unroll
        for (int o = 0; o < Q; ++o) r[o] = T(0);  // an empty window (kh == 0) averages to 0 / 0
#pragma unroll
        for (int u = 0; u < KH; ++u) {
          if (u >= d.kh) break;
#pragma unroll
          for (int o = 0; o < Q; ++o) {
#pragma unroll
            for (int v = 0; v < KW; ++v) {
              const T val = s[k][u].v[o * KW + v];
              if constexpr (MODE == kPoolMax) {
                if (u == 0 && v == 0) r[o] = val;
                else if (val > r[o]) r[o] = val;
              } else {
                r[o] = A::add(u == 0 && v == 0 ? T(0) : r[o], val);
              }
            }
          }
        }
#pragma unroll
        for (int o = 0; o < Q; ++o) {
          if (j0 + o < d.OW) {
            T res = r[o];
            if constexpr (MODE == kPoolAvg) res = pool_mean<T>(res, (int64_t)d.kh * KW);
            out[obase[k] + (j0 + o) * d.os[3]] = res;
          }
        }
      } else {
        // the row's ragged end: windows one by one
        for (int o = 0; o < Q; ++o)
          if (j0 + o < d.OW)
            out[obase[k] + (j0 + o) * d.os[3]] = pool_window<T, MODE>(x, row0[k] + (j0 + o) * KW, d);
      }
    }
  }
}

// MaxPool2d's gradient at pixel (y, xc) of one plane: the sum, from 0 and in
// window order, of the gradients of the windows that read the pixel and
// whose winner (first of the largest, strict `>`) it is.
template <class T>
__device__ __forceinline__ T pixel_grad(const PoolDev& d, const T* __restrict__ x, const T* __restrict__ g,
                                        int64_t plane, int64_t gplane, uint32_t y, uint32_t xc) {
  using A = Arith<T>;
  // windows oh with oh*sh <= y <= oh*sh + kh - 1, likewise ow
  const uint32_t oh_lo = y >= (uint32_t)d.kh ? fdiv(y - d.kh + d.sh, d.f_sh) : 0u;
  uint32_t oh_hi = fdiv(y, d.f_sh);
  if (oh_hi > (uint32_t)d.OH - 1) oh_hi = (uint32_t)d.OH - 1;
  const uint32_t ow_lo = xc >= (uint32_t)d.kw ? fdiv(xc - d.kw + d.sw, d.f_sw) : 0u;
  uint32_t ow_hi = fdiv(xc, d.f_sw);
  if (ow_hi > (uint32_t)d.OW - 1) ow_hi = (uint32_t)d.OW - 1;
  T acc = T(0);
  for (uint32_t oh = oh_lo; oh <= oh_hi; ++oh) {
    for (uint32_t ow = ow_lo; ow <= ow_hi; ++ow) {
      const int64_t base = plane + (int64_t)oh * d.sh * d.xs[2] + (int64_t)ow * d.sw * d.xs[3];
      T best = __ldg(x + base);
      int bu = 0, bv = 0;
      for (int u = 0; u < d.kh; ++u)
        for (int v = (u == 0 ? 1 : 0); v < d.kw; ++v) {
          const T val = __ldg(x + base + u * d.xs[2] + v * d.xs[3]);
          if (val > best) { best = val; bu = u; bv = v; }
        }
      if (oh * d.sh + bu == y && ow * d.sw + bv == xc)
        acc = A::add(acc, __ldg(g + gplane + (int64_t)oh * d.gs[2] + (int64_t)ow * d.gs[3]));
    }
  }
  return acc;
}

// Any window: one thread per input pixel.
template <class T>
__global__ void __launch_bounds__(256) pool_max_bwd_kernel(const PoolDev d) {
  using A = Arith<T>;
  const T* __restrict__ x = static_cast<const T*>(d.x);
  const T* __restrict__ g = static_cast<const T*>(d.g);
  T* out = static_cast<T*>(d.out);
  for (uint64_t it = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < (uint64_t)d.items;
       it += (uint64_t)gridDim.x * blockDim.x) {
    int64_t n, c, y, xc;
    pool_coords(d, it, &n, &c, &y, &xc);
    const T acc = pixel_grad<T>(d, x, g, d.x_off + n * d.xs[0] + c * d.xs[1], d.g_off + n * d.gs[0] + c * d.gs[1],
                                (uint32_t)y, (uint32_t)xc);
    const int64_t o = d.o_off + n * d.os[0] + c * d.os[1] + y * d.os[2] + xc * d.os[3];
    out[o] = d.accumulate ? A::add(out[o], acc) : acc;
  }
}

// MaxPool2d's gradient where the stride equals the window (MaxPool2d::new),
// KW wide and at most KH high, with x and grad_x in unit-stride rows aligned
// to 16 bytes.  The windows tile the image, so a pixel is read by one window
// at most.  An item is one 16-byte strip of one row of windows: the thread
// loads the strip's window rows, finds the winner of each of its Q windows
// once, and writes whole 16-byte rows of grad_x -- the window rows, and in
// the last row of windows also the rows below that no window reads (0, or
// grad_x + 0 when accumulating); columns past the last window get 0 too.
template <class T, int KW, int KH>
__global__ void __launch_bounds__(256, 3) pool_max_bwd_strip_kernel(const PoolDev d) {
  constexpr int VW = 16 / sizeof(T);
  constexpr int Q = VW / KW;
  using A = Arith<T>;
  const T* __restrict__ x = static_cast<const T*>(d.x);
  const T* __restrict__ g = static_cast<const T*>(d.g);
  T* out = static_cast<T*>(d.out);
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t it0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it0 < (uint64_t)d.items;
       it0 += kPoolItems * step) {
    int64_t plane[kPoolItems], gplane[kPoolItems], oplane[kPoolItems], col0[kPoolItems], y0[kPoolItems];
    int64_t irow[kPoolItems];
    bool live[kPoolItems], whole[kPoolItems];
    PVec<T, VW> s[kPoolItems][KH];
#pragma unroll
    for (int k = 0; k < kPoolItems; ++k) {
      const uint64_t it = it0 + (uint64_t)k * step;
      live[k] = it < (uint64_t)d.items;
      int64_t n = 0, c = 0, i = 0, q = 0;
      if (live[k]) pool_coords(d, it, &n, &c, &i, &q);
      plane[k] = d.x_off + n * d.xs[0] + c * d.xs[1];
      gplane[k] = d.g_off + n * d.gs[0] + c * d.gs[1];
      oplane[k] = d.o_off + n * d.os[0] + c * d.os[1];
      irow[k] = i;
      y0[k] = i * d.kh;
      col0[k] = q * VW;
      whole[k] = live[k] && col0[k] + VW <= d.W;
#pragma unroll
      for (int u = 0; u < KH; ++u)
        if (whole[k] && u < d.kh)
          s[k][u] = *reinterpret_cast<const PVec<T, VW>*>(x + plane[k] + (y0[k] + u) * d.xs[2] + col0[k]);
    }
#pragma unroll
    for (int k = 0; k < kPoolItems; ++k) {
      if (!live[k]) continue;
      // the cell's rows: its windows', and below the last row of windows the rest
      const int64_t y_end = irow[k] == d.OH - 1 ? d.H : y0[k] + d.kh;
      if (!whole[k]) {
        // the row's ragged end: pixel by pixel
        for (int64_t y = y0[k]; y < y_end; ++y)
          for (int64_t xc = col0[k]; xc < d.W; ++xc) {
            const T acc = pixel_grad<T>(d, x, g, plane[k], gplane[k], (uint32_t)y, (uint32_t)xc);
            T* dst = out + oplane[k] + y * d.os[2] + xc * d.os[3];
            *dst = d.accumulate ? A::add(*dst, acc) : acc;
          }
        continue;
      }
      const int64_t j0 = col0[k] / KW;
      int bu[Q], bv[Q];
      T gv[Q];
#pragma unroll
      for (int o = 0; o < Q; ++o) {
        bu[o] = -1;
        bv[o] = 0;
        gv[o] = T(0);
        if (j0 + o < d.OW) {
          T best = s[k][0].v[o * KW];
          bu[o] = 0;
#pragma unroll
          for (int u = 0; u < KH; ++u) {
            if (u >= d.kh) break;
#pragma unroll
            for (int v = 0; v < KW; ++v) {
              if (u == 0 && v == 0) continue;
              const T val = s[k][u].v[o * KW + v];
              if (val > best) { best = val; bu[o] = u; bv[o] = v; }
            }
          }
          gv[o] = A::add(T(0), __ldg(g + gplane[k] + irow[k] * d.gs[2] + (j0 + o) * d.gs[3]));
        }
      }
      for (int64_t y = y0[k]; y < y_end; ++y) {
        const int u = (int)(y - y0[k]);
        PVec<T, VW> w;
#pragma unroll
        for (int o = 0; o < Q; ++o)
#pragma unroll
          for (int v = 0; v < KW; ++v) w.v[o * KW + v] = (bu[o] == u && bv[o] == v) ? gv[o] : T(0);
        PVec<T, VW>* dst = reinterpret_cast<PVec<T, VW>*>(out + oplane[k] + y * d.os[2] + col0[k]);
        if (d.accumulate) {
          const PVec<T, VW> cur = *dst;
#pragma unroll
          for (int e = 0; e < VW; ++e) w.v[e] = A::add(cur.v[e], w.v[e]);
        }
        *dst = w;
      }
    }
  }
}

// ---- shared-memory tiles (any window and stride) ---------------------------

// Copies rows y0 .. y0 + nrows - 1 of one plane (unit-stride rows whose starts
// are 16-byte aligned) into shared memory at a pitch of P elements: 16-byte
// cp.async for the whole chunks of each row, plain loads for its last
// W % (16 / size) elements; returns after the CTA's barrier.
template <class T>
__device__ __forceinline__ void stage_rows(const PoolDev& d, T* sm, const T* __restrict__ x, int64_t plane, int64_t y0,
                                           uint32_t nrows) {
  constexpr int VW = 16 / sizeof(T);
  const uint32_t full = (uint32_t)d.full;
  const uint32_t chunks = nrows * full;
  for (uint32_t t = threadIdx.x; t < chunks; t += blockDim.x) {
    const uint32_t r = fdiv(t, d.f_full), ch = t - r * full;
    cp_async16(sm + r * d.P + ch * VW, x + plane + (y0 + r) * d.xs[2] + ch * VW);
  }
  const uint32_t tail = (uint32_t)(d.W - (int64_t)full * VW);
  if (tail)
    for (uint32_t t = threadIdx.x; t < nrows * tail; t += blockDim.x) {
      const uint32_t r = t / tail, e = full * VW + (t - r * tail);
      sm[r * d.P + e] = __ldg(x + plane + (y0 + r) * d.xs[2] + e);
    }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
}

__device__ __forceinline__ void tile_item(const PoolDev& d, uint64_t item, int64_t* n, int64_t* c, int64_t* i0) {
  const uint32_t pl = fdiv((uint32_t)item, d.f_blk);
  const uint32_t b = (uint32_t)item - pl * d.f_blk.d;
  const uint32_t nn = fdiv(pl, d.f_c);
  *n = nn;
  *c = pl - nn * d.f_c.d;
  *i0 = (int64_t)b * d.R;
}

// Forward: an item is a block of R output rows of one plane; its input rows
// are staged once, then each output reads its window from shared memory.
// KH, KW > 0: the window's size at compile time (its loops unroll); 0: the
// launch descriptor's.
template <class T, int MODE, int KH = 0, int KW = 0>
__global__ void __launch_bounds__(256) pool_tile_fwd_kernel(const PoolDev d) {
  using A = Arith<T>;
  extern __shared__ __align__(16) unsigned char pool_smem[];
  T* sm = reinterpret_cast<T*>(pool_smem);
  const T* __restrict__ x = static_cast<const T*>(d.x);
  T* __restrict__ out = static_cast<T*>(d.out);
  for (uint64_t item = blockIdx.x; item < (uint64_t)d.items; item += gridDim.x) {
    int64_t n, c, i0;
    tile_item(d, item, &n, &c, &i0);
    const uint32_t rcnt = (uint32_t)(d.OH - i0 < d.R ? d.OH - i0 : d.R);
    stage_rows<T>(d, sm, x, d.x_off + n * d.xs[0] + c * d.xs[1], i0 * d.sh, (rcnt - 1) * d.sh + d.kh);
    const int64_t oplane = d.o_off + n * d.os[0] + c * d.os[1];
    const uint32_t nout = rcnt * (uint32_t)d.OW;
    for (uint32_t o = threadIdx.x; o < nout; o += blockDim.x) {
      const uint32_t i = fdiv(o, d.f_ow), j = o - i * (uint32_t)d.OW;
      const T* w = sm + i * d.sh * d.P + j * d.sw;
      const int kh = KH > 0 ? KH : d.kh, kw = KW > 0 ? KW : d.kw;
      T r;
      if constexpr (MODE == kPoolMax) {
        r = w[0];
#pragma unroll
        for (int u = 0; u < kh; ++u)
#pragma unroll
          for (int v = 0; v < kw; ++v) {
            if (u == 0 && v == 0) continue;
            const T val = w[u * d.P + v];
            if (val > r) r = val;
          }
      } else {
        r = T(0);
#pragma unroll
        for (int u = 0; u < kh; ++u)
#pragma unroll
          for (int v = 0; v < kw; ++v) r = A::add(r, w[u * d.P + v]);
        r = pool_mean<T>(r, (int64_t)kh * kw);
      }
      out[oplane + (i0 + i) * d.os[2] + (int64_t)j * d.os[3]] = r;
    }
    __syncthreads();
  }
}

// Forward through TMA: an item is a block of R output rows of one plane; its
// (R-1)*sh + kh input rows (every column, rows past the image never read)
// arrive as one TMA box [P, rows, 1, 1] of x seen as [N][C][H][W] into shared
// memory at pitch P (the row width rounded up to 16 bytes).  PAIR (f32, 3x3
// or 2x2 windows, column stride 2): each thread computes two neighbouring
// outputs from one 16-byte load (and, for 3x3, one scalar) per window row, a
// third of the shared loads (stride-2 scalar loads meet two-way bank
// conflicts).  The CTAs are
// persistent with two stages: while an item is pooled from one stage, the
// box of the CTA's next item is in flight into the other.  Each thread owns
// one output column j and walks every step-th row of the block with two
// pointer increments, reading its window at fixed shared offsets.  Every wait
// for a box is bounded: a CTA that runs out records the async error, waits
// (bounded) for its copies still in flight and returns.
template <class T, int MODE, int KH = 0, int KW = 0, bool PAIR = false>
__global__ void __launch_bounds__(256) pool_rows_fwd_kernel(const __grid_constant__ CUtensorMap xmap, const PoolDev d,
                                                            int* err) {
  using A = Arith<T>;
  extern __shared__ unsigned char pool_rows_raw[];
  // aligned by an offset into the shared array itself (not through an
  // integer), so the compiler keeps every access a 32-bit shared one
  unsigned char* base = pool_rows_raw + ((128u - (smem_u32(pool_rows_raw) & 127u)) & 127u);
  const uint32_t box_bytes = (uint32_t)d.box_rows * (uint32_t)d.P * (uint32_t)sizeof(T);
  const uint32_t stage_bytes = (box_bytes + 127) / 128 * 128;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 2 * stage_bytes);
  T* __restrict__ out = static_cast<T*>(d.out);
  const int kh = KH > 0 ? KH : d.kh, kw = KW > 0 ? KW : d.kw;
  const int32_t OW = (int32_t)d.OW, P = d.P, sh = d.sh, sw = d.sw;
  const int32_t step = OW <= 256 ? 256 / OW : 1, n_slots = OW <= 256 ? step * OW : OW;
  auto issue = [&](uint64_t item, int s) {
    int64_t n, c, i0;
    tile_item(d, item, &n, &c, &i0);
    mbar_arrive_expect_tx(&bar[s], box_bytes);
    tma_load_4d(base + s * stage_bytes, &xmap, 0, (int32_t)(i0 * sh), (int32_t)c, (int32_t)n, &bar[s]);
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    if (blockIdx.x < (uint64_t)d.items) issue(blockIdx.x, 0);
  }
  __syncthreads();
  uint32_t phase[2] = {0u, 0u};
  int s = 0;
  for (uint64_t item = blockIdx.x; item < (uint64_t)d.items; item += gridDim.x, s ^= 1) {
    const uint64_t next = item + gridDim.x;
    if (threadIdx.x == 0 && next < (uint64_t)d.items) {
      // stage s^1 was last read by the item before this one, which ended with
      // a barrier; order those reads before the copy's writes
      fence_proxy_async();
      issue(next, s ^ 1);
    }
    const bool ok = cta_wait(&bar[s], phase[s]);
    phase[s] ^= 1u;
    if (!ok) {
      if (threadIdx.x == 0) {
        atomicOr(err, kAsyncWaitTimeout);
        mbar_wait(&bar[s], phase[s] ^ 1u);  // the copies still in flight (bounded)
        if (next < (uint64_t)d.items) mbar_wait(&bar[s ^ 1], phase[s ^ 1]);
      }
      __syncthreads();
      return;
    }
    const T* sm = reinterpret_cast<const T*>(base + s * stage_bytes);
    int64_t n, c, i0;
    tile_item(d, item, &n, &c, &i0);
    const int32_t rcnt = (int32_t)(d.OH - i0 < d.R ? d.OH - i0 : d.R);
    T* oplane = out + d.o_off + n * d.os[0] + c * d.os[1] + i0 * d.os[2];
    if constexpr (PAIR) {
      // f32, 3x3 (2x2) windows at column stride 2: outputs 2q and 2q+1 read
      // columns 4q .. 4q+4 (4q .. 4q+3) of each window row, one 16-byte load
      // and one scalar (one 16-byte load)
      const int32_t QW = (OW + 1) / 2, pstep = 256 / QW;
      if ((int32_t)threadIdx.x < pstep * QW) {
        const int32_t q = (int32_t)threadIdx.x % QW, ii = (int32_t)threadIdx.x / QW;
        const bool second = 2 * q + 1 < OW;
        const int32_t last = 4 * q + 4 < P ? 4 * q + 4 : P - 1;  // past the row only when unused
        const T* w = sm + ii * sh * P;
        T* o = oplane + (int64_t)ii * d.os[2] + (int64_t)(2 * q) * d.os[3];
        // window columns: output 2q starts at column 4q, output 2q+1 at
        // 4q + KW - 1 (3x3: 4q+2; 2x2: 4q+2 as well, the window one column
        // narrower); KW == 2 needs no fifth column
        constexpr int K = KW;
        for (int32_t i = ii; i < rcnt; i += pstep, w += pstep * sh * P, o += pstep * d.os[2]) {
          T v[K][5];
#pragma unroll
          for (int u = 0; u < K; ++u) {
            const float4 a = *reinterpret_cast<const float4*>(w + u * P + 4 * q);
            v[u][0] = a.x;
            v[u][1] = a.y;
            v[u][2] = a.z;
            v[u][3] = a.w;
            v[u][4] = K == 3 ? w[u * P + last] : T(0);
          }
          T r0, r1;
          if constexpr (MODE == kPoolMax) {
            r0 = v[0][0];
            r1 = v[0][2];
#pragma unroll
            for (int u = 0; u < K; ++u)
#pragma unroll
              for (int k = 0; k < K; ++k) {
                if (u > 0 || k > 0) {
                  if (v[u][k] > r0) r0 = v[u][k];
                  if (v[u][k + 2] > r1) r1 = v[u][k + 2];
                }
              }
          } else {
            r0 = T(0);
            r1 = T(0);
#pragma unroll
            for (int u = 0; u < K; ++u)
#pragma unroll
              for (int k = 0; k < K; ++k) {
                r0 = A::add(r0, v[u][k]);
                r1 = A::add(r1, v[u][k + 2]);
              }
            r0 = pool_mean<T>(r0, K * K);
            r1 = pool_mean<T>(r1, K * K);
          }
          o[0] = r0;
          if (second) o[d.os[3]] = r1;
        }
      }
      __syncthreads();  // every thread is done with stage s
      continue;
    }
    for (int32_t slot = threadIdx.x; slot < n_slots; slot += 256) {
      const int32_t j = OW <= 256 ? slot % OW : slot, ii = OW <= 256 ? slot / OW : 0;
      const T* w = sm + ii * sh * P + j * sw;
      T* o = oplane + (int64_t)ii * d.os[2] + (int64_t)j * d.os[3];
      for (int32_t i = ii; i < rcnt; i += step, w += step * sh * P, o += step * d.os[2]) {
        T r;
        if constexpr (MODE == kPoolMax) {
          r = w[0];
#pragma unroll
          for (int u = 0; u < kh; ++u)
#pragma unroll
            for (int v = 0; v < kw; ++v) {
              if (u == 0 && v == 0) continue;
              const T val = w[u * P + v];
              if (val > r) r = val;
            }
        } else {
          r = T(0);
#pragma unroll
          for (int u = 0; u < kh; ++u)
#pragma unroll
            for (int v = 0; v < kw; ++v) r = A::add(r, w[u * P + v]);
          r = pool_mean<T>(r, (int64_t)kh * kw);
        }
        *o = r;
      }
    }
    __syncthreads();  // every thread is done with stage s
  }
}

// MaxPool2d's gradient for f32 2x2 windows at stride 2 that tile the image
// (H even, W a multiple of 8, so every pixel lies in exactly one window and
// the gradient's rows are whole 16-byte units): an item is a block of R window
// rows of one plane; its 2R rows of x and R rows of grad_out arrive as two TMA
// boxes into one of two stages of a persistent CTA (the next item's boxes in
// flight while the current one is done).  Each thread takes two neighbouring
// windows of a window row: two 16-byte loads of x and one 8-byte load of
// grad_out from shared memory, each window's winner found as the first of
// its largest elements in row-major order (a NaN first element wins), then
// two 16-byte stores of grad_x: RN(0 + g) at the winner, +0 elsewhere (with
// ACC, added to the gradient already held, pixel by pixel).
template <bool ACC>
__global__ void __launch_bounds__(256) pool_max_bwd_rows_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const __grid_constant__ CUtensorMap gmap,
                                                                const PoolDev d, int* err) {
  using A = Arith<float>;
  extern __shared__ unsigned char pool_bwd_raw[];
  // aligned by an offset into the shared array itself, so every access stays
  // a 32-bit shared one
  unsigned char* base = pool_bwd_raw + ((128u - (smem_u32(pool_bwd_raw) & 127u)) & 127u);
  const int32_t W = (int32_t)d.W, OW = (int32_t)d.OW;
  const uint32_t xbytes = (uint32_t)(2 * d.R) * (uint32_t)W * 4u, gbytes = (uint32_t)d.R * (uint32_t)OW * 4u;
  const uint32_t xpart = (xbytes + 127) / 128 * 128, stage_bytes = xpart + (gbytes + 127) / 128 * 128;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 2 * stage_bytes);
  float* __restrict__ out = static_cast<float*>(d.out);
  const int32_t QP = OW / 2, pstep = 256 / QP;
  const bool active = (int32_t)threadIdx.x < pstep * QP;
  const int32_t q = (int32_t)threadIdx.x % QP, ii = (int32_t)threadIdx.x / QP;
  auto issue = [&](uint64_t item, int s) {
    int64_t n, c, i0;
    tile_item(d, item, &n, &c, &i0);
    mbar_arrive_expect_tx(&bar[s], xbytes + gbytes);
    tma_load_4d(base + s * stage_bytes, &xmap, 0, (int32_t)(2 * i0), (int32_t)c, (int32_t)n, &bar[s]);
    tma_load_4d(base + s * stage_bytes + xpart, &gmap, 0, (int32_t)i0, (int32_t)c, (int32_t)n, &bar[s]);
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    if (blockIdx.x < (uint64_t)d.items) issue(blockIdx.x, 0);
  }
  __syncthreads();
  uint32_t phase[2] = {0u, 0u};
  int s = 0;
  for (uint64_t item = blockIdx.x; item < (uint64_t)d.items; item += gridDim.x, s ^= 1) {
    const uint64_t next = item + gridDim.x;
    if (threadIdx.x == 0 && next < (uint64_t)d.items) {
      fence_proxy_async();  // stage s^1's reads ended with the barrier of the item before
      issue(next, s ^ 1);
    }
    const bool ok = cta_wait(&bar[s], phase[s]);
    phase[s] ^= 1u;
    if (!ok) {
      if (threadIdx.x == 0) {
        atomicOr(err, kAsyncWaitTimeout);
        mbar_wait(&bar[s], phase[s] ^ 1u);  // the copies still in flight (bounded)
        if (next < (uint64_t)d.items) mbar_wait(&bar[s ^ 1], phase[s ^ 1]);
      }
      __syncthreads();
      return;
    }
    if (active) {
      int64_t n, c, i0;
      tile_item(d, item, &n, &c, &i0);
      const int32_t rcnt = (int32_t)(d.OH - i0 < d.R ? d.OH - i0 : d.R);
      const float* sx = reinterpret_cast<const float*>(base + s * stage_bytes);
      const float* sg = reinterpret_cast<const float*>(base + s * stage_bytes + xpart);
      float* o = out + d.o_off + n * d.os[0] + c * d.os[1] + (2 * i0 + 2 * ii) * d.os[2] + 4 * q;
      for (int32_t i = ii; i < rcnt; i += pstep, o += 2 * pstep * d.os[2]) {
        const float4 a = *reinterpret_cast<const float4*>(sx + (2 * i) * W + 4 * q);
        const float4 b = *reinterpret_cast<const float4*>(sx + (2 * i + 1) * W + 4 * q);
        const float2 gv = *reinterpret_cast<const float2*>(sg + i * OW + 2 * q);
        // window 0: a.x a.y / b.x b.y; window 1: a.z a.w / b.z b.w (row-major)
        int w0 = 0, w1 = 0;
        float m0 = a.x, m1 = a.z;
        if (a.y > m0) { m0 = a.y; w0 = 1; }
        if (b.x > m0) { m0 = b.x; w0 = 2; }
        if (b.y > m0) { w0 = 3; }
        if (a.w > m1) { m1 = a.w; w1 = 1; }
        if (b.z > m1) { m1 = b.z; w1 = 2; }
        if (b.w > m1) { w1 = 3; }
        const float g0 = A::add(0.0f, gv.x), g1 = A::add(0.0f, gv.y);
        float4 r0 = make_float4(w0 == 0 ? g0 : 0.0f, w0 == 1 ? g0 : 0.0f, w1 == 0 ? g1 : 0.0f, w1 == 1 ? g1 : 0.0f);
        float4 r1 = make_float4(w0 == 2 ? g0 : 0.0f, w0 == 3 ? g0 : 0.0f, w1 == 2 ? g1 : 0.0f, w1 == 3 ? g1 : 0.0f);
        float4* o0 = reinterpret_cast<float4*>(o);
        float4* o1 = reinterpret_cast<float4*>(o + d.os[2]);
        if constexpr (ACC) {
          const float4 c0 = *o0, c1 = *o1;
          r0 = make_float4(A::add(c0.x, r0.x), A::add(c0.y, r0.y), A::add(c0.z, r0.z), A::add(c0.w, r0.w));
          r1 = make_float4(A::add(c1.x, r1.x), A::add(c1.y, r1.y), A::add(c1.z, r1.z), A::add(c1.w, r1.w));
        }
        *o0 = r0;
        *o1 = r1;
      }
    }
    __syncthreads();  // every thread is done with stage s
  }
}

// MaxPool2d's gradient: an item is a block of R window rows of one plane and
// owns the input rows from its first window row's start up to the next
// block's (the last block: to the bottom).  The rows of every window reading
// them are staged once, each window's winner is found once (an offset
// u * kw + v in shared memory), then each owned pixel adds, in window order
// from 0, the gradients of the covering windows that it wins.
template <class T>
__global__ void __launch_bounds__(256) pool_tile_bwd_kernel(const PoolDev d) {
  using A = Arith<T>;
  extern __shared__ __align__(16) unsigned char pool_smem[];
  T* sm = reinterpret_cast<T*>(pool_smem);
  const T* __restrict__ x = static_cast<const T*>(d.x);
  const T* __restrict__ g = static_cast<const T*>(d.g);
  T* out = static_cast<T*>(d.out);
  for (uint64_t item = blockIdx.x; item < (uint64_t)d.items; item += gridDim.x) {
    int64_t n, c, i0;
    tile_item(d, item, &n, &c, &i0);
    const int64_t i1 = d.OH - i0 < d.R ? d.OH : i0 + d.R;
    const uint32_t y_lo = (uint32_t)(i0 * d.sh);
    const uint32_t y_hi = (uint32_t)(i1 == d.OH ? d.H : i1 * d.sh);
    const uint32_t oh_lo = y_lo >= (uint32_t)d.kh ? fdiv(y_lo - d.kh + d.sh, d.f_sh) : 0u;
    uint32_t oh_hi = fdiv(y_hi - 1, d.f_sh);
    if (oh_hi > (uint32_t)d.OH - 1) oh_hi = (uint32_t)d.OH - 1;
    const int64_t plane = d.x_off + n * d.xs[0] + c * d.xs[1];
    const int64_t gplane = d.g_off + n * d.gs[0] + c * d.gs[1];
    const int64_t oplane = d.o_off + n * d.os[0] + c * d.os[1];
    const uint32_t sy0 = oh_lo * d.sh;
    const uint32_t srows = (uint32_t)((int64_t)oh_hi * d.sh + d.kh) - sy0;
    // the winners after the staged rows, 16-byte aligned
    int32_t* win = reinterpret_cast<int32_t*>(pool_smem + (((size_t)srows * d.P * sizeof(T) + 15) & ~(size_t)15));
    stage_rows<T>(d, sm, x, plane, sy0, srows);
    const uint32_t nwin = (oh_hi - oh_lo + 1) * (uint32_t)d.OW;
    for (uint32_t t = threadIdx.x; t < nwin; t += blockDim.x) {
      const uint32_t wr = fdiv(t, d.f_ow), ow = t - wr * (uint32_t)d.OW;
      const T* w = sm + wr * d.sh * d.P + ow * d.sw;
      T best = w[0];
      int k = 0;
      for (int u = 0; u < d.kh; ++u)
        for (int v = (u == 0 ? 1 : 0); v < d.kw; ++v) {
          const T val = w[u * d.P + v];
          if (val > best) { best = val; k = u * d.kw + v; }
        }
      win[t] = k;
    }
    __syncthreads();
    const uint32_t npx = (y_hi - y_lo) * (uint32_t)d.W;
    for (uint32_t q = threadIdx.x; q < npx; q += blockDim.x) {
      const uint32_t yr = fdiv(q, d.f_w), xc = q - yr * (uint32_t)d.W;
      const uint32_t y = y_lo + yr;
      uint32_t ohs = y >= (uint32_t)d.kh ? fdiv(y - d.kh + d.sh, d.f_sh) : 0u;
      uint32_t ohe = fdiv(y, d.f_sh);
      if (ohe > oh_hi) ohe = oh_hi;
      const uint32_t ows = xc >= (uint32_t)d.kw ? fdiv(xc - d.kw + d.sw, d.f_sw) : 0u;
      uint32_t owe = fdiv(xc, d.f_sw);
      if (owe > (uint32_t)d.OW - 1) owe = (uint32_t)d.OW - 1;
      T acc = T(0);
      for (uint32_t oh = ohs; oh <= ohe; ++oh)
        for (uint32_t ow = ows; ow <= owe; ++ow)
          if (win[(oh - oh_lo) * (uint32_t)d.OW + ow] == (int)((y - oh * d.sh) * d.kw + (xc - ow * d.sw)))
            acc = A::add(acc, __ldg(g + gplane + (int64_t)oh * d.gs[2] + (int64_t)ow * d.gs[3]));
      T* dst = out + oplane + (int64_t)y * d.os[2] + (int64_t)xc * d.os[3];
      *dst = d.accumulate ? A::add(*dst, acc) : acc;
    }
    __syncthreads();
  }
}

// One wave of 256-thread CTAs (as many per SM as fit), each thread looping.
template <class K>
unsigned pool_grid(K kernel, uint64_t items) {
  const int per_sm = resident_blocks_smem((const void*)kernel, 256, 0);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)per_sm;
  const uint64_t need = (items + 255) / 256;
  return (unsigned)(need < cap ? (need < 1 ? 1 : need) : cap);
}

// [lo, hi) byte range a view can touch.
void byte_range(const trs_view* v, int64_t* lo, int64_t* hi) {
  const int es = dtype_size(v->dtype);
  int64_t a = v->offset, b = v->offset;
  for (int i = 0; i < v->ndim; ++i) {
    const int64_t span = (v->shape[i] - 1) * v->strides[i];
    if (span > 0) b += span; else a += span;
  }
  *lo = (int64_t)(uintptr_t)v->data + a * es;
  *hi = (int64_t)(uintptr_t)v->data + (b + 1) * es;
}

bool overlaps(const trs_view* a, const trs_view* b) {
  if (numel_of(a->shape, a->ndim) == 0 || numel_of(b->shape, b->ndim) == 0) return false;
  int64_t alo, ahi, blo, bhi;
  byte_range(a, &alo, &ahi);
  byte_range(b, &blo, &bhi);
  return alo < bhi && blo < ahi;
}

Error check_4d(const trs_view* v, const char* what, int dt, const int64_t* want) {
  Error e = validate_view(v, what);
  if (!e.ok()) return e;
  if (v->dtype != dt) return make_error(TRS_ERR_DTYPE, std::string(what) + ": dtype differs from x");
  bool same = v->ndim == 4;
  for (int i = 0; same && i < 4; ++i) same = v->shape[i] == want[i];
  if (!same) return make_error(TRS_ERR_SHAPE, std::string(what) + ": wrong shape");
  return Error{};
}

// Shape rules of pool_dims (pool.rs:36-41), with_stride (pool.rs:115-118) and
// unfold_dims (conv.rs:490-510); fills the geometry of d.
Error pool_setup(const char* layer, const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, bool is_max,
                 PoolDev* d) {
  std::memset(d, 0, sizeof(*d));
  if (!x) return make_error(TRS_ERR_ARG, "null view");
  Error e = validate_view(x, "x");
  if (!e.ok()) return e;
  if (!is_float(x->dtype)) return make_error(TRS_ERR_DTYPE, std::string(layer) + " needs f32 or f64");
  if (x->ndim != 4)
    return make_error(TRS_ERR_SHAPE, std::string("!!!") + layer + " expects [batch, channels, height, width]!!!");
  if (sh <= 0 || sw <= 0) return make_error(TRS_ERR_ARG, std::string("!!!") + layer + ": stride must be positive!!!");
  if (kh < 0 || kw < 0 || kh > (1 << 20) || kw > (1 << 20) || sh > (1 << 30) || sw > (1 << 30))
    return make_error(TRS_ERR_ARG, "window or stride out of range");
  if (x->shape[2] < kh || x->shape[3] < kw)
    return make_error(TRS_ERR_SHAPE, "!!!unfold_2d(): the input is smaller than the kernel!!!");
  if (is_max && kh * kw == 0) return make_error(TRS_ERR_EMPTY_AXIS, "!!!Cannot reduce an empty axis!!!");
  // the index arithmetic divides by W, H, C and the strides as 32-bit
  // divisors, and y - kh + stride stays below 2^32
  if (x->shape[1] >= (1ll << 31) || x->shape[2] >= (1ll << 31) || x->shape[3] >= (1ll << 31))
    return make_error(TRS_ERR_ARG, "pool: a dimension of 2^31 or more");
  d->H = x->shape[2];
  d->W = x->shape[3];
  d->OH = (d->H - kh) / sh + 1;
  d->OW = (d->W - kw) / sw + 1;
  d->kh = (int32_t)kh;
  d->kw = (int32_t)kw;
  d->sh = (int32_t)sh;
  d->sw = (int32_t)sw;
  d->f_sh = make_fastdiv((uint32_t)sh);
  d->f_sw = make_fastdiv((uint32_t)sw);
  d->x = x->data;
  d->x_off = x->offset;
  for (int i = 0; i < 4; ++i) d->xs[i] = x->strides[i];
  return Error{};
}

void set_items(PoolDev* d, int64_t planes, int64_t C, int64_t rows, int64_t inner) {
  d->inner = inner;
  d->items = planes * rows * inner;
  d->fast = (uint64_t)d->items < (1ull << 32) ? 1 : 0;
  d->f_inner = make_fastdiv((uint32_t)(inner < 1 ? 1 : inner));
  d->f_rows = make_fastdiv((uint32_t)(rows < 1 ? 1 : rows));
  d->f_c = make_fastdiv((uint32_t)(C < 1 ? 1 : C));
}

// x (and, for the backward, grad_x) in unit-stride rows whose starts are all
// 16-byte aligned.
bool rows_aligned(const void* base, int64_t off, const int64_t* st, int es) {
  const int vw = 16 / es;
  if (((uintptr_t)base + (uintptr_t)(off * es)) % 16 || st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] % vw) return false;
  return true;
}

template <class K>
Error pool_launch(K kernel, const PoolDev& d, cudaStream_t stream, const char* what) {
  kernel<<<pool_grid(kernel, (uint64_t)d.items), 256, 0, stream>>>(d);
  return check_launch(what);
}

// Shared memory a tile item may use: 8 CTAs of 256 threads fit on an SM.
constexpr int64_t kPoolTileBytes = 24 << 10;

// 1: the tile kernels take windows the strip kernels could also take.
#ifndef TRS_POOL_TILE_FIRST
#define TRS_POOL_TILE_FIRST 0
#endif

// Blocks of R window rows per plane for the tile kernels; false when one
// window row does not fit or the items overflow 32-bit indexing.
bool plan_tile(PoolDev* d, bool bwd, int es, int64_t N, int64_t C, size_t* smem) {
  const int vw = 16 / es;
  const int64_t P = (d->W + vw - 1) / vw * vw;
  const int64_t e = bwd ? (d->kh - 1) / d->sh : 0;  // windows above a block reaching into it
  auto bytes = [&](int64_t R) {
    const int64_t rows = (R + e - 1) * d->sh + d->kh;
    int64_t b = (rows * P * es + 15) / 16 * 16;
    if (bwd) b += (R + e) * d->OW * 4;
    return b;
  };
  if (d->kh < 1 || d->kw < 1 || bytes(1) > kPoolTileBytes) return false;
  int64_t R = 1;
  while (R < d->OH && bytes(R + 1) <= kPoolTileBytes) ++R;
  const int64_t nblk = (d->OH + R - 1) / R;
  const int64_t items = N * C * nblk;
  if (items >= (1ll << 32) || (bwd && (R * d->sh + d->kh) * d->W >= (1ll << 32))) return false;
  d->R = (int32_t)R;
  d->P = (int32_t)P;
  d->nblk = (int32_t)nblk;
  d->full = (int32_t)(d->W / vw);
  d->items = items;
  d->f_blk = make_fastdiv((uint32_t)nblk);
  d->f_ow = make_fastdiv((uint32_t)d->OW);
  d->f_w = make_fastdiv((uint32_t)d->W);
  d->f_full = make_fastdiv((uint32_t)(d->full < 1 ? 1 : d->full));
  d->f_c = make_fastdiv((uint32_t)(C < 1 ? 1 : C));
  *smem = (size_t)bytes(R);
  return true;
}

template <class K>
Error pool_tile_launch(K kernel, const PoolDev& d, size_t smem, cudaStream_t stream, const char* what) {
  const int per_sm = resident_blocks_smem((const void*)kernel, 256, (int)smem);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)per_sm;
  const uint64_t grid = (uint64_t)d.items < cap ? (uint64_t)d.items : cap;
  kernel<<<(unsigned)grid, 256, smem, stream>>>(d);
  return check_launch(what);
}

// Shared memory a TMA row item's box may take (a CTA holds two).
constexpr int64_t kPoolRowsBytes = 24 << 10;

// Tuning knob: 0 never uses the TMA row kernel, 1 uses it wherever it
// applies, 2 where the strip kernel does not.
#ifndef TRS_POOL_ROWS
#define TRS_POOL_ROWS 2
#endif

// Blocks of R output rows per plane for the TMA row kernel: x must be a TMA
// tensor (unit-stride rows, positive strides in whole 16-byte units, a
// 16-byte aligned start), its rows at most 256 wide, the box at most 256 rows
// and kPoolRowsBytes; false otherwise or when the items overflow 32 bits.
bool plan_rows(PoolDev* d, int es, int64_t N, int64_t C, size_t* smem) {
  const int vw = 16 / es;
  for (int i = 0; i < 3; ++i)
    if (d->xs[i] <= 0 || d->xs[i] * es >= (1ll << 40)) return false;
  const int64_t P = (d->W + vw - 1) / vw * vw;
  auto rows = [&](int64_t R) { return (R - 1) * d->sh + d->kh; };
  auto fits = [&](int64_t R) { return rows(R) <= 256 && rows(R) * P * es <= kPoolRowsBytes; };
  if (d->kh < 1 || d->kw < 1 || P > 256 || !fits(1) || N >= (1ll << 31) || C >= (1ll << 31) ||
      d->H >= (1ll << 31))
    return false;
  int64_t R = 1;
  while (R < d->OH && fits(R + 1)) ++R;
  const int64_t nblk = (d->OH + R - 1) / R, items = N * C * nblk;
  if (items >= (1ll << 32)) return false;
  d->R = (int32_t)R;
  d->P = (int32_t)P;
  d->nblk = (int32_t)nblk;
  d->items = items;
  d->box_rows = (int32_t)rows(R);
  d->f_blk = make_fastdiv((uint32_t)nblk);
  d->f_c = make_fastdiv((uint32_t)(C < 1 ? 1 : C));
  *smem = (size_t)(2 * ((rows(R) * P * es + 127) / 128 * 128) + 16 + 128);  // two boxes, mbarriers, alignment
  return true;
}

template <class T, int MODE, int KH, int KW, bool PAIR = false>
Error pool_rows_launch(const PoolDev& d, const CUtensorMap& map, size_t smem, cudaStream_t stream) {
  const void* k = (const void*)pool_rows_fwd_kernel<T, MODE, KH, KW, PAIR>;
  allow_smem(k, (int)smem);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, 256, (int)smem);
  const uint64_t grid = (uint64_t)d.items < cap ? (uint64_t)d.items : cap;  // persistent
  pool_rows_fwd_kernel<T, MODE, KH, KW, PAIR><<<(unsigned)grid, 256, smem, stream>>>(map, d, async_error_word());
  return check_launch("pool rows");
}

template <class T>
Error launch_pool_rows(const PoolDev& d, int mode, int64_t N, int64_t C, size_t smem, cudaStream_t stream) {
  // x as [N][C][H][W]: boxes [P, box_rows, 1, 1]
  const cuuint64_t es = sizeof(T);
  CUtensorMap map;
  Error e = make_map_4d<T>("pool", static_cast<const T*>(d.x) + d.x_off,
                           {(cuuint64_t)d.W, (cuuint64_t)d.H, (cuuint64_t)C, (cuuint64_t)N},
                           {(cuuint64_t)d.xs[2] * es, (cuuint64_t)d.xs[1] * es, (cuuint64_t)d.xs[0] * es},
                           {(cuuint32_t)d.P, (cuuint32_t)d.box_rows, 1, 1}, &map);
  if (!e.ok()) return e;
  const bool max = mode == kPoolMax;
  if constexpr (sizeof(T) == 4) {
    if (d.kh == 3 && d.kw == 3 && d.sw == 2 && (d.OW + 1) / 2 <= 256)
      return max ? pool_rows_launch<T, kPoolMax, 3, 3, true>(d, map, smem, stream)
                 : pool_rows_launch<T, kPoolAvg, 3, 3, true>(d, map, smem, stream);
    if (d.kh == 2 && d.kw == 2 && d.sw == 2 && (d.OW + 1) / 2 <= 256)
      return max ? pool_rows_launch<T, kPoolMax, 2, 2, true>(d, map, smem, stream)
                 : pool_rows_launch<T, kPoolAvg, 2, 2, true>(d, map, smem, stream);
  }
  if (d.kh == 3 && d.kw == 3)
    return max ? pool_rows_launch<T, kPoolMax, 3, 3>(d, map, smem, stream)
               : pool_rows_launch<T, kPoolAvg, 3, 3>(d, map, smem, stream);
  if (d.kh == 2 && d.kw == 2)
    return max ? pool_rows_launch<T, kPoolMax, 2, 2>(d, map, smem, stream)
               : pool_rows_launch<T, kPoolAvg, 2, 2>(d, map, smem, stream);
  return max ? pool_rows_launch<T, kPoolMax, 0, 0>(d, map, smem, stream)
             : pool_rows_launch<T, kPoolAvg, 0, 0>(d, map, smem, stream);
}

// Tuning knob: 0 keeps MaxPool2d's gradient off the TMA row kernel.
#ifndef TRS_POOL_BWD_ROWS
#define TRS_POOL_BWD_ROWS 1
#endif

// The TMA row kernel of MaxPool2d's gradient (f32, 2x2 windows at stride 2
// tiling the image, W a multiple of 8 and at most 256): x and grad_out as TMA
// tensors, grad_x in unit-stride 16-byte aligned rows; blocks of R window rows
// whose two boxes fit kPoolRowsBytes.  False otherwise.
bool plan_bwd_rows(PoolDev* d, const trs_view* x, const trs_view* g, const trs_view* gx, int64_t N, int64_t C,
                   size_t* smem) {
  if (x->dtype != TRS_F32 || d->kh != 2 || d->kw != 2 || d->sh != 2 || d->sw != 2) return false;
  if (d->H % 2 != 0 || d->W % 8 != 0 || d->W > 256 || d->OH * 2 != d->H || d->OW * 2 != d->W) return false;
  if (!rows_aligned(x->data, x->offset, x->strides, 4) || !rows_aligned(g->data, g->offset, g->strides, 4) ||
      !rows_aligned(gx->data, gx->offset, gx->strides, 4))
    return false;
  for (int i = 0; i < 3; ++i)
    if (x->strides[i] <= 0 || g->strides[i] <= 0 || x->strides[i] * 4 >= (1ll << 40) || g->strides[i] * 4 >= (1ll << 40))
      return false;
  if (N >= (1ll << 31) || C >= (1ll << 31)) return false;
  auto bytes = [&](int64_t R) { return ((2 * R * d->W * 4 + 127) / 128 + (R * d->OW * 4 + 127) / 128) * 128; };
  int64_t R = 1;
  while (R < d->OH && 2 * (R + 1) <= 256 && bytes(R + 1) <= kPoolRowsBytes) ++R;
  const int64_t nblk = (d->OH + R - 1) / R, items = N * C * nblk;
  if (items >= (1ll << 32)) return false;
  d->R = (int32_t)R;
  d->nblk = (int32_t)nblk;
  d->items = items;
  d->f_blk = make_fastdiv((uint32_t)nblk);
  d->f_c = make_fastdiv((uint32_t)(C < 1 ? 1 : C));
  *smem = (size_t)(2 * bytes(R) + 16 + 128);  // two stages, mbarriers, alignment
  return true;
}

Error launch_pool_bwd_rows(const PoolDev& d, int64_t N, int64_t C, size_t smem, cudaStream_t stream) {
  CUtensorMap xmap, gmap;
  Error e = make_map_4d<float>("pool backward", static_cast<const float*>(d.x) + d.x_off,
                               {(cuuint64_t)d.W, (cuuint64_t)d.H, (cuuint64_t)C, (cuuint64_t)N},
                               {(cuuint64_t)d.xs[2] * 4, (cuuint64_t)d.xs[1] * 4, (cuuint64_t)d.xs[0] * 4},
                               {(cuuint32_t)d.W, (cuuint32_t)(2 * d.R), 1, 1}, &xmap);
  if (e.ok())
    e = make_map_4d<float>("pool backward", static_cast<const float*>(d.g) + d.g_off,
                           {(cuuint64_t)d.OW, (cuuint64_t)d.OH, (cuuint64_t)C, (cuuint64_t)N},
                           {(cuuint64_t)d.gs[2] * 4, (cuuint64_t)d.gs[1] * 4, (cuuint64_t)d.gs[0] * 4},
                           {(cuuint32_t)d.OW, (cuuint32_t)d.R, 1, 1}, &gmap);
  if (!e.ok()) return e;
  const void* k = d.accumulate ? (const void*)pool_max_bwd_rows_kernel<true> : (const void*)pool_max_bwd_rows_kernel<false>;
  allow_smem(k, (int)smem);
  const uint64_t cap = (uint64_t)current_device_info().sm_count * (uint64_t)resident_blocks_smem(k, 256, (int)smem);
  const unsigned grid = (unsigned)((uint64_t)d.items < cap ? (uint64_t)d.items : cap);  // persistent
  if (d.accumulate)
    pool_max_bwd_rows_kernel<true><<<grid, 256, smem, stream>>>(xmap, gmap, d, async_error_word());
  else
    pool_max_bwd_rows_kernel<false><<<grid, 256, smem, stream>>>(xmap, gmap, d, async_error_word());
  return check_launch("max pool backward rows");
}

template <class T>
Error launch_pool_fwd(PoolDev d, int mode, int64_t N, int64_t C, cudaStream_t stream) {
  constexpr int VW = 16 / sizeof(T);
  // the strip kernel: kw == stride_w dividing 16 bytes, kh <= 4, aligned rows
  const bool aligned = rows_aligned(d.x, d.x_off, d.xs, sizeof(T));
  const bool strip = d.kw == d.sw && d.kw > 0 && VW % d.kw == 0 && d.kh <= 4 && aligned;
  size_t smem = 0;
  // f32 2x2 windows at stride 2: the row kernel's paired outputs beat the strips
  const bool pair2 = sizeof(T) == 4 && d.kh == 2 && d.kw == 2 && d.sw == 2;
  if (TRS_POOL_ROWS && (TRS_POOL_ROWS == 1 || !strip || pair2) && aligned) {
    PoolDev r = d;
    if (plan_rows(&r, sizeof(T), N, C, &smem)) return launch_pool_rows<T>(r, mode, N, C, smem, stream);
  }
  if ((!strip || TRS_POOL_TILE_FIRST) && aligned && plan_tile(&d, false, sizeof(T), N, C, &smem)) {
    // the common square windows with their loops unrolled
    if (d.kh == 3 && d.kw == 3)
      return mode == kPoolMax ? pool_tile_launch(pool_tile_fwd_kernel<T, kPoolMax, 3, 3>, d, smem, stream, "pool tiles")
                              : pool_tile_launch(pool_tile_fwd_kernel<T, kPoolAvg, 3, 3>, d, smem, stream, "pool tiles");
    if (d.kh == 2 && d.kw == 2)
      return mode == kPoolMax ? pool_tile_launch(pool_tile_fwd_kernel<T, kPoolMax, 2, 2>, d, smem, stream, "pool tiles")
                              : pool_tile_launch(pool_tile_fwd_kernel<T, kPoolAvg, 2, 2>, d, smem, stream, "pool tiles");
    return mode == kPoolMax ? pool_tile_launch(pool_tile_fwd_kernel<T, kPoolMax>, d, smem, stream, "pool tiles")
                            : pool_tile_launch(pool_tile_fwd_kernel<T, kPoolAvg>, d, smem, stream, "pool tiles");
  }
  if (!strip) {
    set_items(&d, N * C, C, d.OH, d.OW);
    return mode == kPoolMax ? pool_launch(pool_fwd_kernel<T, kPoolMax>, d, stream, "pool kernel")
                            : pool_launch(pool_fwd_kernel<T, kPoolAvg>, d, stream, "pool kernel");
  }
  const int Q = VW / d.kw;
  set_items(&d, N * C, C, d.OH, (d.OW + Q - 1) / Q);
  const bool max = mode == kPoolMax;
  const bool low = d.kh <= 2;
#define TRS_POOL_STRIP(KWV)                                                                            \
  if (d.kw == KWV) {                                                                                   \
    if (low) return max ? pool_launch(pool_strip_kernel<T, kPoolMax, KWV, 2>, d, stream, "pool strips")  \
                        : pool_launch(pool_strip_kernel<T, kPoolAvg, KWV, 2>, d, stream, "pool strips"); \
    return max ? pool_launch(pool_strip_kernel<T, kPoolMax, KWV, 4>, d, stream, "pool strips")           \
               : pool_launch(pool_strip_kernel<T, kPoolAvg, KWV, 4>, d, stream, "pool strips");          \
  }
  TRS_POOL_STRIP(1)
  TRS_POOL_STRIP(2)
  if constexpr (VW >= 4) {
    TRS_POOL_STRIP(4)
  }
#undef TRS_POOL_STRIP
  return make_error(TRS_ERR_ARG, "pool: no strip kernel for this window");
}

template <class T>
Error launch_pool_bwd(PoolDev d, int64_t N, int64_t C, cudaStream_t stream) {
  constexpr int VW = 16 / sizeof(T);
  // the strip kernel: stride == window (the windows tile the image), kw
  // dividing 16 bytes, kh <= 4, x and grad_x in aligned rows
  const bool aligned = rows_aligned(d.x, d.x_off, d.xs, sizeof(T));
  const bool strip = d.kw == d.sw && d.kh == d.sh && d.kw > 0 && VW % d.kw == 0 && d.kh <= 4 && aligned &&
                     rows_aligned(d.out, d.o_off, d.os, sizeof(T));
  size_t smem = 0;
  if ((!strip || TRS_POOL_TILE_FIRST) && aligned && plan_tile(&d, true, sizeof(T), N, C, &smem))
    return pool_tile_launch(pool_tile_bwd_kernel<T>, d, smem, stream, "max pool backward tiles");
  if (!strip) {
    set_items(&d, N * C, C, d.H, d.W);
    return pool_launch(pool_max_bwd_kernel<T>, d, stream, "max pool backward kernel");
  }
  set_items(&d, N * C, C, d.OH, (d.W + VW - 1) / VW);
  const bool low = d.kh <= 2;
#define TRS_POOL_BWD_STRIP(KWV)                                                                  \
  if (d.kw == KWV)                                                                               \
    return low ? pool_launch(pool_max_bwd_strip_kernel<T, KWV, 2>, d, stream, "max pool backward strips") \
               : pool_launch(pool_max_bwd_strip_kernel<T, KWV, 4>, d, stream, "max pool backward strips");
  TRS_POOL_BWD_STRIP(1)
  TRS_POOL_BWD_STRIP(2)
  if constexpr (VW >= 4) {
    TRS_POOL_BWD_STRIP(4)
  }
#undef TRS_POOL_BWD_STRIP
  return make_error(TRS_ERR_ARG, "pool backward: no strip kernel for this window");
}

Error run_pool(int mode, const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, const trs_view* out,
               cudaStream_t stream) {
  const char* layer = mode == kPoolMax ? "MaxPool2d" : "AvgPool2d";
  PoolDev d;
  Error e = pool_setup(layer, x, kh, kw, sh, sw, mode == kPoolMax, &d);
  if (!e.ok()) return e;
  if (!out) return make_error(TRS_ERR_ARG, "null view");
  const int64_t N = x->shape[0], C = x->shape[1];
  const int64_t want[4] = {N, C, d.OH, d.OW};
  e = check_4d(out, "output", x->dtype, want);
  if (!e.ok()) return e;
  if (overlaps(x, out)) return make_error(TRS_ERR_ALIAS, "pool: the output overlaps the input");
  if (N * C * d.OH * d.OW == 0) return Error{};
  d.out = out->data;
  d.o_off = out->offset;
  for (int i = 0; i < 4; ++i) d.os[i] = out->strides[i];
  if (x->dtype == TRS_F32) return launch_pool_fwd<float>(d, mode, N, C, stream);
  return launch_pool_fwd<double>(d, mode, N, C, stream);
}

Error run_max_pool_backward(const trs_view* x, const trs_view* g, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                            int accumulate, const trs_view* gx, cudaStream_t stream) {
  PoolDev d;
  Error e = pool_setup("MaxPool2d", x, kh, kw, sh, sw, true, &d);
  if (!e.ok()) return e;
  if (!g || !gx) return make_error(TRS_ERR_ARG, "null view");
  const int64_t N = x->shape[0], C = x->shape[1];
  const int64_t gshape[4] = {N, C, d.OH, d.OW};
  e = check_4d(g, "grad_out", x->dtype, gshape);
  if (!e.ok()) return e;
  e = check_4d(gx, "grad_x", x->dtype, x->shape);
  if (!e.ok()) return e;
  if (overlaps(gx, x) || overlaps(gx, g))
    return make_error(TRS_ERR_ALIAS, "pool backward: grad_x overlaps an input");
  if (N * C * d.H * d.W == 0) return Error{};
  d.g = g->data;
  d.g_off = g->offset;
  d.out = gx->data;
  d.o_off = gx->offset;
  for (int i = 0; i < 4; ++i) {
    d.gs[i] = g->strides[i];
    d.os[i] = gx->strides[i];
  }
  d.accumulate = accumulate ? 1 : 0;
  {
    PoolDev r = d;
    size_t smem = 0;
    if (TRS_POOL_BWD_ROWS && plan_bwd_rows(&r, x, g, gx, N, C, &smem)) return launch_pool_bwd_rows(r, N, C, smem, stream);
  }
  if (x->dtype == TRS_F32) return launch_pool_bwd<float>(d, N, C, stream);
  return launch_pool_bwd<double>(d, N, C, stream);
}

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

}  // namespace
}  // namespace trs

using namespace trs;

extern "C" {

trs_status trs_max_pool2d(const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, trs_view* out,
                          trs_stream stream) {
  return finish(run_pool(kPoolMax, x, kh, kw, sh, sw, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_avg_pool2d(const trs_view* x, int64_t kh, int64_t kw, int64_t sh, int64_t sw, trs_view* out,
                          trs_stream stream) {
  return finish(run_pool(kPoolAvg, x, kh, kw, sh, sw, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_max_pool2d_backward(const trs_view* x, const trs_view* grad_out, int64_t kh, int64_t kw, int64_t sh,
                                   int64_t sw, int32_t accumulate, trs_view* grad_x, trs_stream stream) {
  return finish(run_max_pool_backward(x, grad_out, kh, kw, sh, sw, accumulate, grad_x,
                                      static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
