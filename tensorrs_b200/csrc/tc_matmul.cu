// tc_matmul.cu -- trs_matmul_tf32x3: Tensor::matmul (linalg/tensor/base.rs:
// 896-1013) for f32 on the 5th-generation tensor cores, within the sum
// tolerance instead of bit-identical.
//
// trs_matmul keeps the reference's per-output chain of separately rounded
// multiplies and adds on the CUDA cores.  This variant trades that for the
// tensor cores' rate: each f32 operand x is split into two TF32 values,
// hi = x with its 13 low mantissa bits cleared and lo = x - hi (exact in f32;
// the tensor core reads its top 19 bits), and every product is taken as
// hi*hi + hi*lo + lo*hi (the lo*lo term, below 2^-21 of the product, is
// dropped), accumulated in f32 in tensor memory.  Products keep about 21 bits;
// the accumulation order and rounding are the tensor core's, so a result
// differs from the reference's sequential chain by about the rounding error of
// an f32 sum: the tests hold it to |gpu - ref| <= 1e-5 * sum_k |a_ik b_kj|.
//
// Data flow:
//   1. tf32_split_kernel packs A into hi/lo arrays [A batches][Mp][Kp] and B
//      into [B batches][Np][Kp] (K contiguous: both operands K-major for the
//      MMA), zero-padded to multiples of 128 rows and 32 k, through 32 x 32
//      shared-memory tiles so that both the strided reads and the writes are
//      coalesced (scratch from the stream-ordered pool);
//   2. tc_gemm_kernel<BN>: one CTA of 4 warps per 128 x BN output tile, BN =
//      256 where that still gives six waves of tiles (less shared-memory
//      traffic per product, the bound of this kernel), 128 otherwise; tiles
//      in a grouped order (kTcGroup row blocks walked column by column).
//      Thread 0 streams 32-deep k slabs of the four operand tiles into a ring
//      of stages (3 x 64 KiB for BN 128, 2 x 96 KiB for BN 256) with TMA
//      (cp.async.bulk.tensor.2d, 128-byte swizzle, no multicast), completing
//      on a `full` mbarrier; thread 32 waits for a slab and issues, for each
//      of its 4 k-steps of 8, the three tcgen05.mma kind::tf32 (M 128, N BN)
//      into one f32 accumulator of BN TMEM columns (the first two share A,
//      which the collector buffer keeps between them), then tcgen05.commit
//      frees the slab through its `empty` mbarrier; a final commit signals
//      `done`, and all 4 warps read their 32 accumulator rows with
//      tcgen05.ld and write them through the output view.
// A call whose inputs hold an infinity or NaN (the split kernels raise a flag)
// takes the reference's exact chain on the CUDA cores in every CTA instead: a
// split product inf * (a zero lo part) would turn an infinite result into NaN.
// Every mbarrier wait is bounded (kWaitIters polls); a wait that runs out
// sets the async-error word and the CTA skips ahead to free its tensor
// memory and return.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "kernels.cuh"
#include "tma.cuh"

namespace trs {
namespace {

constexpr int kTcBM = 128, kTcBK = 32;
constexpr uint32_t kTcTile = kTcBM * kTcBK * 4;      // one A tile of a slab: 16 KiB

// An output tile of 128 x BN (BN = 128 or 256): a stage holds A hi, A lo
// (16 KiB each) and B hi, B lo (BN x 32 each); three stages of 64 KiB for
// BN = 128, two of 96 KiB for BN = 256; the accumulator takes BN TMEM columns.
template <int BN>
struct TcShape {
  static constexpr uint32_t tile_b = BN * kTcBK * 4;
  static constexpr uint32_t stage = 2 * kTcTile + 2 * tile_b;
  static constexpr int stages = BN == 128 ? 3 : 2;
  static constexpr uint32_t smem = stages * stage + 1024 + 256;  // + alignment slack + barriers
  static constexpr uint32_t cols = BN;
  // instruction descriptor: D f32, A and B tf32, both K-major, N = BN, M = 128
  static constexpr uint32_t idesc =
      (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
};
#ifndef TRS_TC_GROUP
#define TRS_TC_GROUP 8
#endif
constexpr int kTcGroup = TRS_TC_GROUP;               // row blocks of tiles per group of the tile order

// ---- the split / pack kernel -------------------------------------------------

struct SplitDev {
  const float* src;
  float* hi;
  float* lo;
  int* nonfinite;        // set to 1 when some element is an infinity or NaN
  int64_t rows, K;       // logical rows (M for A, N for B) and depth
  int64_t rows_p, Kp;    // padded
  int64_t s_row, s_k;    // source strides of a row and of k
  int64_t off;           // source offset
  int nb;                // batch dimensions of this operand
  int64_t bshape[kMaxDims], bst[kMaxDims];
  int k_fast;            // the source is unit-stride along k
};

__device__ __forceinline__ void tf32_split(float x, float* h, float* l) {
  if (!isfinite(x)) {  // inf / NaN carried by hi alone
    *h = x;
    *l = 0.0f;
    return;
  }
  const float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  *h = hi;
  *l = __fsub_rn(x, hi);  // exact
}

// grid: (Kp / 32, rows_p / 32, batches); block 32 x 8
__global__ void __launch_bounds__(256) tf32_split_kernel(const SplitDev d) {
  __shared__ float tile[32][33];
  const int64_t bt = blockIdx.z;
  int64_t off = d.off;
  {
    int64_t r = bt;
    for (int i = d.nb - 1; i >= 0; --i) {
      off += (r % d.bshape[i]) * d.bst[i];
      r /= d.bshape[i];
    }
  }
  const int64_t k0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int q = ty; q < 32; q += 8) {
    // read along the source's unit-stride dimension
    const int64_t r = d.k_fast ? r0 + q : r0 + tx, k = d.k_fast ? k0 + tx : k0 + q;
    float v = 0.0f;
    if (r < d.rows && k < d.K) v = d.src[off + r * d.s_row + k * d.s_k];
    if (__any_sync(0xffffffffu, (__float_as_uint(v) & 0x7F800000u) == 0x7F800000u) && tx == 0)
      atomicOr(d.nonfinite, 1);
    if (d.k_fast)
      tile[q][tx] = v;
    else
      tile[tx][q] = v;
  }
  __syncthreads();
  for (int q = ty; q < 32; q += 8) {
    const int64_t r = r0 + q, k = k0 + tx;
    float h, l;
    tf32_split(tile[q][tx], &h, &l);
    const int64_t at = (bt * d.rows_p + r) * d.Kp + k;
    d.hi[at] = h;
    d.lo[at] = l;
  }
}

// The same split for an operand already K-major with 16-byte aligned rows
// (s_k == 1, s_row and the offset multiples of 4, the base 16-byte aligned):
// no transpose, one 16-byte load and two 16-byte stores per thread and step.
// Grid-stride over the padded [batches][rows_p][Kp / 4] chunks (fewer than
// 2^32: the index decodes with 32-bit fast divisions by rows_p * Kp / 4 and
// Kp / 4).
__global__ void __launch_bounds__(256) tf32_split_vec_kernel(const SplitDev d, uint32_t n, FastDiv f_pb, FastDiv f_kq) {
  bool nonfinite = false;
  for (uint32_t i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) {
    const uint32_t bt = fdiv(i, f_pb), rem = i - bt * f_pb.d;
    const uint32_t r32 = fdiv(rem, f_kq);
    const int64_t r = r32, k = (int64_t)(rem - r32 * f_kq.d) * 4;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (r < d.rows) {
      int64_t off = d.off;
      int64_t q = bt;
      for (int j = d.nb - 1; j >= 0; --j) {
        off += (q % d.bshape[j]) * d.bst[j];
        q /= d.bshape[j];
      }
      const float* src = d.src + off + r * d.s_row + k;
      if (k + 4 <= d.K) {
        const float4 x = __ldcs(reinterpret_cast<const float4*>(src));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
      } else {
        for (int j = 0; j < 4; ++j)
          if (k + j < d.K) v[j] = src[j];
      }
    }
    float4 h, l;
    float* hp = &h.x;
    float* lp = &l.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      nonfinite |= (__float_as_uint(v[j]) & 0x7F800000u) == 0x7F800000u;
      tf32_split(v[j], hp + j, lp + j);
    }
    *reinterpret_cast<float4*>(d.hi + (size_t)i * 4) = h;
    *reinterpret_cast<float4*>(d.lo + (size_t)i * 4) = l;
  }
  if (__any_sync(0xffffffffu, nonfinite) && (threadIdx.x & 31) == 0) atomicOr(d.nonfinite, 1);
}

// +0 into every element of a view (row-major over its shape).
__global__ void __launch_bounds__(256) zero_view_kernel(const trs_view v, int64_t n) {
  float* o = static_cast<float*>(v.data);
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
    int64_t r = i, at = v.offset;
    for (int dd = v.ndim - 1; dd >= 0; --dd) {
      at += (r % v.shape[dd]) * v.strides[dd];
      r /= v.shape[dd];
    }
    o[at] = 0.0f;
  }
}

// ---- tcgen05 / TMA primitives ---------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem, K-major] * B[smem, K-major]^T, M 128, N 128, K 8 (tf32).
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

#ifndef TRS_TC_COLLECTOR
#define TRS_TC_COLLECTOR 1
#endif
// The same MMA with its A operand kept in the collector buffer for the next
// MMA (fill), or taken from it and released (lastuse).
__device__ __forceinline__ void umma_tf32_fill(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32.collector::a::fill [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_tf32_lastuse(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                                  uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32.collector::a::lastuse [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), leading offset
// unused (1), descriptor version 1, layout SWIZZLE_128B (2); the tile starts
// on a 1024-byte boundary, so the base offset is 0.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t a = (uint64_t)(smem_u32(tile) >> 4) & 0x3FFFull;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}


struct TcDev {
  int64_t M, N, Kp, Mp, Np;
  void* out;
  int64_t o_off, som, son;
  int nb;  // output batch dimensions
  int64_t bshape[kMaxDims], o_bst[kMaxDims];
  int64_t a_bidx[kMaxDims], b_bidx[kMaxDims];  // per output batch dim: stride in the operand's packed batch index
  int* err;
  const float *ahi, *alo, *bhi, *blo;  // the packed planes (for the exact path)
  int64_t K;
  const int* nonfinite;  // set by the split kernels: some input is an infinity or NaN
};

// The reference's chain acc = acc + a * b over k from +0, each step rounded
// once, for this CTA's tile: used instead of the tensor cores when an input
// holds an infinity or NaN, where a split product (inf times a zero lo part)
// would turn an infinite result into NaN.  x = hi + lo exactly (hi = x, lo = 0
// for a non-finite x), so the result is bit-identical to trs_matmul's.
template <int BN>
__device__ void tc_exact_tile(const TcDev& d, int64_t abt, int64_t bbt, int64_t oo, int64_t tile_m, int64_t tile_n) {
  float* out = static_cast<float*>(d.out);
  for (int idx = threadIdx.x; idx < kTcBM * BN; idx += blockDim.x) {
    const int64_t col = tile_n * BN + idx % BN, r = tile_m * kTcBM + idx / BN;
    if (col >= d.N || r >= d.M) continue;
    const int64_t bo = (bbt * d.Np + col) * d.Kp;
    const int64_t ao = (abt * d.Mp + r) * d.Kp;
    float acc = 0.0f;
    for (int64_t k = 0; k < d.K; ++k)
      acc = __fadd_rn(acc, __fmul_rn(__fadd_rn(d.ahi[ao + k], d.alo[ao + k]), __fadd_rn(d.bhi[bo + k], d.blo[bo + k])));
    out[oo + r * d.som + col * d.son] = acc;
  }
}

template <int BN>
__global__ void __launch_bounds__(128, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap t_ahi, const __grid_constant__ CUtensorMap t_alo,
               const __grid_constant__ CUtensorMap t_bhi, const __grid_constant__ CUtensorMap t_blo,
               const TcDev d) {
  using S = TcShape<BN>;
  extern __shared__ unsigned char tc_smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::stages * S::stage);
  uint64_t* empty = full + S::stages;
  uint64_t* done = empty + S::stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *failed = 0;
    fence_mbar_init();
  }
  __syncwarp();  // warp 0 converged for the warp-collective allocation
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // this CTA's rows in the packed operands: batch index of A and of B
  int64_t abt = 0, bbt = 0, oo = d.o_off;
  {
    int64_t r = blockIdx.z;
    for (int i = d.nb - 1; i >= 0; --i) {
      const int64_t c = r % d.bshape[i];
      r /= d.bshape[i];
      abt += c * d.a_bidx[i];
      bbt += c * d.b_bidx[i];
      oo += c * d.o_bst[i];
    }
  }
  // grouped tile order: CTAs launch in blockIdx order, and consecutive ones
  // take the tiles of kTcGroup row blocks column by column, so a wave's A and
  // B tiles are few enough to stay in L2 while the wave walks K
  int64_t tile_m, tile_n;
  {
    const int64_t gx = gridDim.x, gy = gridDim.y;
    const int64_t pid = (int64_t)blockIdx.y * gx + blockIdx.x;
    const int64_t per_group = (int64_t)kTcGroup * gx;
    const int64_t first = pid / per_group * kTcGroup;
    const int64_t rows = gy - first < kTcGroup ? gy - first : kTcGroup;
    const int64_t local = pid % per_group;
    tile_m = first + local % rows;
    tile_n = local / rows;
  }
  const int32_t a_row = (int32_t)(abt * d.Mp + tile_m * kTcBM);
  const int32_t b_row = (int32_t)(bbt * d.Np + tile_n * BN);
  const int nk = (int)(d.Kp / kTcBK);
  // an infinity or NaN among the inputs: the exact chain instead (the flag
  // is the same for every thread of the grid, so the CTA branches as one)
  if (*(volatile const int*)d.nonfinite != 0) {
    tc_exact_tile<BN>(d, abt, bbt, oo, tile_m, tile_n);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, S::cols);
    return;
  }

  if (threadIdx.x == 0) {  // TMA producer
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S::stages;
      const uint32_t ph = (uint32_t)(kb / S::stages) & 1u;
      if (kb >= S::stages && !mbar_wait(&empty[s], ph ^ 1u)) {
        atomicExch(failed, 1);
        break;
      }
      if (*(volatile int*)failed) break;
      unsigned char* st = smem + s * S::stage;
      mbar_arrive_expect_tx(&full[s], S::stage);
      const int32_t kx = kb * kTcBK;
      tma_load_2d(st, &t_ahi, kx, a_row, &full[s]);
      tma_load_2d(st + kTcTile, &t_alo, kx, a_row, &full[s]);
      tma_load_2d(st + 2 * kTcTile, &t_bhi, kx, b_row, &full[s]);
      tma_load_2d(st + 2 * kTcTile + S::tile_b, &t_blo, kx, b_row, &full[s]);
    }
  } else if (threadIdx.x == 32) {  // MMA issuer
    bool ok = true;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % S::stages;
      const uint32_t ph = (uint32_t)(kb / S::stages) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        atomicExch(failed, 1);
        ok = false;
        break;
      }
      tc_fence_after();
      unsigned char* st = smem + s * S::stage;
      const uint64_t ahi = sw128_desc(st), alo = sw128_desc(st + kTcTile);
      const uint64_t bhi = sw128_desc(st + 2 * kTcTile), blo = sw128_desc(st + 2 * kTcTile + S::tile_b);
#pragma unroll
      for (int k = 0; k < kTcBK / 8; ++k) {
        const uint64_t dk = (uint64_t)(k * 2);  // 8 tf32 = 32 bytes, in 16-byte units
#if TRS_TC_COLLECTOR
        // the first two products share A: it is read from shared memory once
        umma_tf32_fill(tmem, ahi + dk, bhi + dk, S::idesc, (kb > 0 || k > 0) ? 1u : 0u);
        umma_tf32_lastuse(tmem, ahi + dk, blo + dk, S::idesc, 1u);
#else
        umma_tf32(tmem, ahi + dk, bhi + dk, S::idesc, (kb > 0 || k > 0) ? 1u : 0u);
        umma_tf32(tmem, ahi + dk, blo + dk, S::idesc, 1u);
#endif
        umma_tf32(tmem, alo + dk, bhi + dk, S::idesc, 1u);
      }
      umma_commit(&empty[s]);  // the slab is free once these have read it
    }
    umma_commit(done);  // every MMA issued above has completed
  }

  // epilogue: warp w reads accumulator rows 32w .. 32w + 31 (its TMEM lanes)
  const bool ready = mbar_wait(done, 0);
  // tcgen05.ld is warp-collective: the whole warp takes one branch
  const bool go = __all_sync(0xffffffffu, ready && !*(volatile int*)failed);
  tc_fence_after();
  if (!go) {
    if (lane == 0 && d.err) atomicOr(d.err, kAsyncWaitTimeout);
  } else {
    float* out = static_cast<float*>(d.out);
    const int64_t row = tile_m * kTcBM + warp * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
      if (row < d.M) {
        const int64_t col0 = tile_n * BN + c * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < d.N) out[oo + row * d.som + (col0 + j) * d.son] = __uint_as_float(v[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, S::cols);
}

// ---- host side -------------------------------------------------------------------

// [batches * rows_p, Kp] f32, K contiguous, 32 x box_rows boxes with 128-byte swizzle.
Error make_map(EncodeTiled enc, CUtensorMap* map, float* base, int64_t rows_total, int64_t Kp, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows_total};
  const cuuint64_t strides[1] = {(cuuint64_t)Kp * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return make_error(TRS_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return Error{};
}

bool views_overlap(const trs_view* a, const trs_view* b) {
  if (numel_of(a->shape, a->ndim) == 0 || numel_of(b->shape, b->ndim) == 0) return false;
  auto range = [](const trs_view* v, int64_t* lo, int64_t* hi) {
    int64_t l = v->offset, h = v->offset;
    for (int i = 0; i < v->ndim; ++i) {
      const int64_t span = (v->shape[i] - 1) * v->strides[i];
      if (span > 0) h += span; else l += span;
    }
    *lo = (int64_t)(uintptr_t)v->data + l * 4;
    *hi = (int64_t)(uintptr_t)v->data + (h + 1) * 4;
  };
  int64_t alo, ahi, blo, bhi;
  range(a, &alo, &ahi);
  range(b, &blo, &bhi);
  return alo < bhi && blo < ahi;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

template <int BN>
Error launch_tc_gemm(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
                     const TcDev& td, int64_t batches, cudaStream_t stream) {
  using S = TcShape<BN>;
  allow_smem((const void*)tc_gemm_kernel<BN>, (int)S::smem);
  tc_gemm_kernel<BN><<<dim3((unsigned)(td.Np / BN), (unsigned)(td.Mp / kTcBM), (unsigned)batches), 128, S::smem,
                       stream>>>(ahi, alo, bhi, blo, td);
  return check_launch("tcgen05 tf32x3 matmul kernel");
}

Error run_tc_matmul(const trs_view* a, const trs_view* b, const trs_view* out, cudaStream_t stream) {
  Error e = validate_view(a, "a");
  if (!e.ok()) return e;
  e = validate_view(b, "b");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (a->dtype != TRS_F32 || b->dtype != TRS_F32 || out->dtype != TRS_F32)
    return make_error(TRS_ERR_DTYPE, "matmul_tf32x3: f32 operands and output only");
  const int an = a->ndim, bn = b->ndim;
  if (an < 2 || bn < 2) return make_error(TRS_ERR_SHAPE, "matmul: both tensors must be at least 2D");
  const int64_t M = a->shape[an - 2], K = a->shape[an - 1], N = b->shape[bn - 1];
  if (K != b->shape[bn - 2])
    return make_error(TRS_ERR_SHAPE, "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])");
  int64_t batch[kMaxDims];
  int nb = 0;
  if (!broadcast_shapes(a->shape, an - 2, b->shape, bn - 2, batch, &nb))
    return make_error(TRS_ERR_SHAPE, "matmul: batch shapes not broadcastable");
  bool same = out->ndim == nb + 2 && out->shape[nb] == M && out->shape[nb + 1] == N;
  for (int i = 0; same && i < nb; ++i) same = out->shape[i] == batch[i];
  if (!same) return make_error(TRS_ERR_SHAPE, "matmul_tf32x3: the output must have the shape [batch..., M, N]");
  if (views_overlap(out, a) || views_overlap(out, b))
    return make_error(TRS_ERR_ALIAS, "matmul_tf32x3: the output overlaps an input");
  int64_t batches = 1;
  for (int i = 0; i < nb; ++i) batches *= batch[i];
  if (M == 0 || N == 0 || batches == 0) return Error{};
  // the 128 x 256 tile (less shared-memory traffic per product) where it
  // still gives at least six waves of tiles, the 128 x 128 tile otherwise
  const int64_t Mp = round_up(M, kTcBM), Kp = round_up(K, kTcBK);
  const bool wide =
      round_up(N, 256) / 256 * (Mp / kTcBM) * batches >= 6 * (int64_t)current_device_info().sm_count;
  const int BN = wide ? 256 : 128;
  const int64_t Np = round_up(N, BN);
  // each operand packed over its own batch dimensions
  SplitDev sa, sb;
  std::memset(&sa, 0, sizeof(sa));
  std::memset(&sb, 0, sizeof(sb));
  int64_t a_batches = 1, b_batches = 1;
  for (int i = 0; i < an - 2; ++i) a_batches *= a->shape[i];
  for (int i = 0; i < bn - 2; ++i) b_batches *= b->shape[i];
  if (K == 0) {  // every output is the empty chain's +0
    zero_view_kernel<<<(unsigned)((batches * M * N + 255) / 256 < 65535 ? (batches * M * N + 255) / 256 : 65535), 256,
                       0, stream>>>(*out, batches * M * N);
    return check_launch("matmul zero fill");
  }
  if (Kp >= (1ll << 31) || a_batches * Mp >= (1ll << 31) || b_batches * Np >= (1ll << 31) || Mp / 32 > 65535 ||
      Np / 32 > 65535)
    return make_error(TRS_ERR_SHAPE, "matmul_tf32x3: operands beyond 2^31 packed rows or 2 M rows per batch");
  TcDev td;
  std::memset(&td, 0, sizeof(td));
  td.M = M;
  td.N = N;
  td.Kp = Kp;
  td.Mp = Mp;
  td.Np = Np;
  td.out = out->data;
  td.o_off = out->offset;
  td.som = out->strides[nb];
  td.son = out->strides[nb + 1];
  td.nb = nb;
  td.err = async_error_word();
  {
    // strides of each output batch dimension in A's and B's packed batch index
    int64_t sa_step = 1, sb_step = 1;
    int64_t a_step[kMaxDims] = {}, b_step[kMaxDims] = {};
    for (int i = an - 3; i >= 0; --i) { a_step[i] = sa_step; sa_step *= a->shape[i]; }
    for (int i = bn - 3; i >= 0; --i) { b_step[i] = sb_step; sb_step *= b->shape[i]; }
    for (int i = 0; i < nb; ++i) {
      td.bshape[i] = batch[i];
      td.o_bst[i] = out->strides[i];
      const int ia = i - (nb - (an - 2)), ib = i - (nb - (bn - 2));
      td.a_bidx[i] = (ia >= 0 && a->shape[ia] != 1) ? a_step[ia] : 0;
      td.b_bidx[i] = (ib >= 0 && b->shape[ib] != 1) ? b_step[ib] : 0;
    }
  }
  EncodeTiled enc = encode_fn(&e);
  if (!enc) return e;
  Scratch buf;
  const size_t na = (size_t)(a_batches * Mp * Kp), nbb = (size_t)(b_batches * Np * Kp);
  e = buf.alloc(sizeof(float) * 2 * (na + nbb) + 16, stream);
  if (!e.ok()) return e;
  float* ahi = buf.as<float>();
  float* alo = ahi + na;
  float* bhi = alo + na;
  float* blo = bhi + nbb;
  int* nonfinite = reinterpret_cast<int*>(blo + nbb);
  cudaError_t ce = cudaMemsetAsync(nonfinite, 0, sizeof(int), stream);
  if (ce != cudaSuccess) return cuda_error(ce, "cudaMemsetAsync");
  td.ahi = ahi;
  td.alo = alo;
  td.bhi = bhi;
  td.blo = blo;
  td.K = K;
  td.nonfinite = nonfinite;
  // split / pack
  sa.src = static_cast<const float*>(a->data);
  sa.hi = ahi;
  sa.lo = alo;
  sa.nonfinite = nonfinite;
  sa.rows = M;
  sa.K = K;
  sa.rows_p = Mp;
  sa.Kp = Kp;
  sa.s_row = a->strides[an - 2];
  sa.s_k = a->strides[an - 1];
  sa.off = a->offset;
  sa.nb = an - 2;
  for (int i = 0; i < an - 2; ++i) { sa.bshape[i] = a->shape[i]; sa.bst[i] = a->strides[i]; }
  sa.k_fast = sa.s_k == 1 || sa.s_row != 1;
  sb.src = static_cast<const float*>(b->data);
  sb.hi = bhi;
  sb.lo = blo;
  sb.nonfinite = nonfinite;
  sb.rows = N;
  sb.K = K;
  sb.rows_p = Np;
  sb.Kp = Kp;
  sb.s_row = b->strides[bn - 1];
  sb.s_k = b->strides[bn - 2];
  sb.off = b->offset;
  sb.nb = bn - 2;
  for (int i = 0; i < bn - 2; ++i) { sb.bshape[i] = b->shape[i]; sb.bst[i] = b->strides[i]; }
  sb.k_fast = sb.s_k == 1 || sb.s_row != 1;
  if (a_batches > 65535 || b_batches > 65535 || batches > 65535)
    return make_error(TRS_ERR_SHAPE, "matmul_tf32x3: more than 65535 batches");
  // an operand already K-major with 16-byte aligned rows takes the direct
  // 16-byte split; any other layout goes through the transposing tiles
  auto split = [&](const SplitDev& sd, const void* base, int64_t ops_batches, const char* what) {
    const int64_t chunks = ops_batches * sd.rows_p * (sd.Kp / 4);
    bool vec = sd.s_k == 1 && sd.s_row % 4 == 0 && sd.off % 4 == 0 && (uintptr_t)base % 16 == 0 &&
               chunks < (1ll << 32) - 256ll * 65536;
    for (int i = 0; i < sd.nb && vec; ++i) vec = sd.bst[i] % 4 == 0;
    if (vec) {
      const int64_t cap = (int64_t)current_device_info().sm_count * 8;
      const int64_t g = (chunks + 255) / 256 < cap ? (chunks + 255) / 256 : cap;
      tf32_split_vec_kernel<<<(unsigned)(g < 1 ? 1 : g), 256, 0, stream>>>(
          sd, (uint32_t)chunks, make_fastdiv((uint32_t)(sd.rows_p * (sd.Kp / 4))), make_fastdiv((uint32_t)(sd.Kp / 4)));
    } else {
      tf32_split_kernel<<<dim3((unsigned)(sd.Kp / 32), (unsigned)(sd.rows_p / 32), (unsigned)ops_batches), dim3(32, 8), 0,
                          stream>>>(sd);
    }
    return check_launch(what);
  };
  e = split(sa, a->data, a_batches, "tf32 split kernel (A)");
  if (!e.ok()) return e;
  e = split(sb, b->data, b_batches, "tf32 split kernel (B)");
  if (!e.ok()) return e;
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  e = make_map(enc, &m_ahi, ahi, a_batches * Mp, Kp, kTcBM);
  if (e.ok()) e = make_map(enc, &m_alo, alo, a_batches * Mp, Kp, kTcBM);
  if (e.ok()) e = make_map(enc, &m_bhi, bhi, b_batches * Np, Kp, BN);
  if (e.ok()) e = make_map(enc, &m_blo, blo, b_batches * Np, Kp, BN);
  if (!e.ok()) return e;
  return wide ? launch_tc_gemm<256>(m_ahi, m_alo, m_bhi, m_blo, td, batches, stream)
              : launch_tc_gemm<128>(m_ahi, m_alo, m_bhi, m_blo, td, batches, stream);
}

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

}  // namespace
}  // namespace trs

extern "C" trs_status trs_matmul_tf32x3(const trs_view* a, const trs_view* b, trs_view* out, trs_stream stream) {
  if (!a || !b || !out) return trs::finish(trs::make_error(TRS_ERR_ARG, "null view"));
  return trs::finish(trs::run_tc_matmul(a, b, out, static_cast<cudaStream_t>(stream)));
}
