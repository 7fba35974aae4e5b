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
  int stages;                // softmax_stream_kernel: rows staged in shared memory
  int* err;                  // async-error word (bounded waits)
};

Error run_softmax(const trs_view* x, const trs_view* out, cudaStream_t stream);

}  // namespace trs
