// softmax.h -- row softmax launch descriptor (see softmax.cu).
#pragma once

#include <cstdint>

#include "plan.h"
#include "runtime.h"

namespace trs {

struct SmDev {
  const void* in;
  void* out;
  int64_t in_off, out_off;
  int64_t C;                 // row length (last axis)
  int64_t in_step, out_step; // strides along the last axis
  int64_t rows;
  int nouter;                // folded leading dims (size-1 dims dropped)
  int64_t oshape[kMaxDims];
  int64_t ist[kMaxDims];
  int64_t ost[kMaxDims];
  double e_const;            // log2(E_f32) for f32, E_f64 for f64
  int stages;                // row_stream_kernel: rows staged in shared memory
  int* err;                  // async-error word (bounded waits)
  // LayerNorm: gamma / beta (F values each, stride g_st / b_st), epsilon
  const void* gamma;
  const void* beta;
  int64_t g_off, b_off, g_st, b_st;
  double ln_eps;
  int gb_vec;                // gamma and beta unit-stride and 16-byte aligned
};

Error run_softmax(const trs_view* x, const trs_view* out, cudaStream_t stream);

// LayerNorm over the last axis on the bulk-copy row pipeline, for rows of
// 4 KiB .. 96 KiB whose starts (input and output) are 16-byte aligned and
// whose step along the row is 1.  Returns TRS_NONE (nothing launched) when
// the rows do not qualify; `d` describes x / out / gamma / beta as for the
// row kernels.
Error run_layer_norm_stream(SmDev d, int dtype, cudaStream_t stream);

}  // namespace trs
