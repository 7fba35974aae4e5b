// reduce.h -- reduction launch descriptors (see reduce.cu).
#pragma once

#include <cstdint>

#include "plan.h"
#include "runtime.h"

namespace trs {

enum RedMode {
  kRedSum = 0,        // sum over the reduced dims
  kRedMean = 1,       // sum / (number of reduced elements), IEEE division in T
  kRedMax = 2,        // max_axis
  kRedArgmax = 3,     // argmax_axis (i64 output)
  kRedSum3 = 4,       // sum of g & map(gate > 0 ? 1 : 0) & mul (gate, mul optional)
  kRedAffineRelu = 5  // ReLU(x & s + b) backward: out0 = sum (g&m)&x, out1 = sum g&m
};

constexpr int kRedOperands = 4;

// What to reduce, in the input's own dimensions: operand k (0 = the tensor
// being reduced, 1..3 = auxiliary inputs of the fused modes) has strides
// op_strides[k][i] along input dimension i (already broadcast to the input's
// shape); outputs m = 0, 1 have strides out_strides[m][i] along every kept
// input dimension i.
struct RedRequest {
  int mode = kRedSum;
  // raw outputs (for combining partials across ranks): sums are written as
  // the unrounded accumulator, max/argmax as MaxRecord with indices offset by
  // idx_base; out_strides then count records, not elements
  bool raw = false;
  int64_t idx_base = 0;
  uint32_t reduce_mask = 0;  // bit i set: input dimension i is reduced
  const trs_view* in[kRedOperands] = {nullptr, nullptr, nullptr, nullptr};
  int64_t op_strides[kRedOperands][kMaxDims] = {};
  const trs_view* out[2] = {nullptr, nullptr};
  int64_t out_strides[2][kMaxDims] = {};
};

// One rank's max/argmax partial of one output: the largest non-NaN value
// and its (global) index, idx < 0 when there is none; `first` is the element
// at the rank's index 0 (the reference keeps a NaN found at global index 0).
template <class T>
struct MaxRecord {
  T val;
  T first;
  int64_t idx;
};

struct RedDev {
  int mode;
  int raw;
  int64_t idx_base;
  int has_gate, has_mul;
  const void* in[kRedOperands];
  int64_t off[kRedOperands];
  void* out[2];
  int64_t out_off[2];
  // kept dims (folded)
  int nk;
  int64_t kshape[kMaxDims];
  int64_t kst[kRedOperands][kMaxDims];
  int64_t kout[2][kMaxDims];
  // reduced dims (folded)
  int nr;
  int64_t rshape[kMaxDims];
  int64_t rst[kRedOperands][kMaxDims];
  int64_t total;   // reduced elements per output
  int64_t n_out;   // outputs
  // row kernel
  int64_t L, RO;
  int inner_bcast[kRedOperands];
  // row stream kernel (bulk-copy pipeline over contiguous segments)
  int64_t tps;           // tiles per segment
  int64_t P;             // parts per output (items = n_out * P)
  int64_t tpp;           // tiles per part
  int bulk_slot[kRedOperands];
  uint32_t fk[kMaxDims][3];  // FastDiv (d, m, s) of kshape
  uint32_t fr[kMaxDims][3];  // FastDiv of rshape
  uint32_t f_tps[3];
  void* parts;           // RedAcc partial per item when P > 1
  int* err;
  // column kernel
  int64_t W;
  int64_t wst[kRedOperands];
  int64_t wout[2];
  int64_t n_out_outer;
  // column stream kernel (bulk-copy pipeline over row segments of W)
  int32_t cs_wt;       // columns per column block (its last block may be narrower)
  int32_t cs_pitch;    // bytes between staged rows (cs_wt * element size)
  int32_t cs_rt;       // rows per stage (<= 32)
  int32_t cs_cpr_pad;  // 16-byte chunks per row, rounded up to a power of two
  int64_t cs_ncb;      // column blocks
  int64_t cs_rp;       // rows per part (a multiple of cs_rt)
};

// Geometry of the column stream kernel, shared by the planner and the kernel:
// 16 KiB stages (up to 32 staged rows of at most 2 KiB each), an 80 KiB stage
// budget per CTA, and 16 KiB for combining the row groups' states.
constexpr int kCsStageBytes = 16384;
constexpr int kCsBudget = 80 * 1024;
constexpr int kCsMaxPitch = 2048;
constexpr int kCsCombBytes = 256 * 16 * 4;  // 256 threads x up to 4 columns x 16-byte states
constexpr int kSmemPerSm = 228 * 1024;

__host__ __device__ constexpr int cs_stages(int nb) {
  return kCsBudget / (nb * kCsStageBytes) > 8 ? 8
         : (kCsBudget / (nb * kCsStageBytes) < 2 ? 2 : kCsBudget / (nb * kCsStageBytes));
}

__host__ __device__ constexpr int cs_smem_bytes(int nb) {
  return cs_stages(nb) * nb * kCsStageBytes + kCsCombBytes + 2 * cs_stages(nb) * 8;
}

enum RedVariant { kRedRow = 0, kRedCol = 1, kRedGeneric = 2, kRedRowStream = 3, kRedColStream = 4 };

struct RedChoice {
  int variant = kRedGeneric;
  int nb = 0;  // bulk operands of the stream kernel
  int vec = 1;
  bool warp_mode = false;
  unsigned cluster = 1;
  int per_sm = 1;  // resident CTAs per SM the planner assumed (stream kernels)
};

Error plan_reduce(const RedRequest& q, RedDev* d, RedChoice* c);
template <class T>
Error red_launch(RedDev& d, const RedChoice& c, cudaStream_t stream);
template <class T>
bool red_stream_available(int mode, int nb);
template <class T>
bool red_cstream_available(int mode, int nb);
Error run_reduce(const RedRequest& q, cudaStream_t stream);

}  // namespace trs
