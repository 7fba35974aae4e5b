// plan.h -- host-side view validation and dimension folding shared by every
// entry point, and the plain-old-data launch descriptors the kernels receive.
//
// The reference builds a storage-index vector per operand for every
// broadcast or strided op (storage_indices, base.rs:404-428) and then gathers
// through it.  Here the same logical->storage mapping is folded on the host
// into the fewest dimensions that describe it (size-1 dimensions dropped,
// adjacent dimensions merged when every operand steps through them as one
// run), and the kernels evaluate it on the fly.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/trs.h"

namespace trs {

constexpr int kMaxDims = TRS_MAX_DIMS;
constexpr int kMaxOperands = 4;  // output + up to three inputs

inline int dtype_size(int dt) {
  switch (dt) {
    case TRS_F32: return 4;
    case TRS_F64: return 8;
    case TRS_I32: return 4;
    case TRS_I64: return 8;
  }
  return 0;
}
inline bool is_float(int dt) { return dt == TRS_F32 || dt == TRS_F64; }

// Status plus message, carried back to trs_last_error().
struct Error {
  trs_status status = TRS_OK;
  std::string msg;
  bool ok() const { return status == TRS_OK; }
};
Error make_error(trs_status s, const std::string& msg);

int64_t numel_of(const int64_t* shape, int ndim);

// Checks rank, shape, dtype and that every element the view can reach lies
// inside [0, storage_len).  An empty view (some dimension 0) is always valid.
Error validate_view(const trs_view* v, const char* what);

// broadcast_shape (ops.rs:27-45).
bool broadcast_shapes(const int64_t* a, int an, const int64_t* b, int bn,
                      int64_t* out, int* on);

// broadcast_to (base.rs:556-599): strides of `v` seen as `target` (rank tn),
// 0 on broadcast dimensions.  False if `v` does not broadcast to `target`.
bool broadcast_strides(const trs_view* v, const int64_t* target, int tn,
                       int64_t* strides_out);

// A folded element-wise launch: output is operand 0, inputs 1..n_in.
struct EwFold {
  int nd = 1;                                // folded rank, >= 1
  int64_t shape[kMaxDims] = {1};
  int64_t st[kMaxOperands][kMaxDims] = {};   // folded strides per operand
  int64_t off[kMaxOperands] = {};            // element offsets
  int64_t n = 0;                             // number of elements
  int n_ops = 1;                             // 1 + n_in
};

// Folds `n_ops` operands that all have logical shape `shape` (rank `nd`)
// with the given per-operand strides.
void fold_dims(const int64_t* shape, int nd, const int64_t (*strides)[kMaxDims],
               const int64_t* offsets, int n_ops, EwFold* f);

enum EwVariant { kEwVec = 0, kEwTile = 1, kEwGeneric = 2 };

// Kernel choice for a folded element-wise op (see ew.cu).
struct EwChoice {
  int variant = kEwGeneric;
  int vec = 1;        // elements per vector access in the vec kernel
  int tile_dim = -1;  // the "i" dimension for the tiled transpose kernel
};
EwChoice choose_ew(const EwFold& f, const void* const* bases, int elem_size);

}  // namespace trs
