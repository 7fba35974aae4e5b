// plan.cpp -- view validation, broadcasting and dimension folding (host only).
#include "plan.h"

#include <cstring>

namespace trs {

Error make_error(trs_status s, const std::string& msg) {
  Error e;
  e.status = s;
  e.msg = msg;
  return e;
}

int64_t numel_of(const int64_t* shape, int ndim) {
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= shape[i];
  return n;
}

Error validate_view(const trs_view* v, const char* what) {
  if (!v) return make_error(TRS_ERR_ARG, std::string(what) + ": null view");
  if (v->ndim < 0 || v->ndim > kMaxDims)
    return make_error(TRS_ERR_VIEW, std::string(what) + ": rank out of range (0..8)");
  if (dtype_size(v->dtype) == 0)
    return make_error(TRS_ERR_DTYPE, std::string(what) + ": unknown dtype");
  __int128 n = 1;
  for (int i = 0; i < v->ndim; ++i) {
    if (v->shape[i] < 0) return make_error(TRS_ERR_VIEW, std::string(what) + ": negative dimension");
    n *= v->shape[i];
    if (n > ((__int128)1 << 62)) return make_error(TRS_ERR_VIEW, std::string(what) + ": too many elements");
  }
  if (n == 0) return Error{};
  if (!v->data) return make_error(TRS_ERR_ARG, std::string(what) + ": null data pointer");
  __int128 lo = v->offset, hi = v->offset;
  for (int i = 0; i < v->ndim; ++i) {
    __int128 span = (__int128)(v->shape[i] - 1) * v->strides[i];
    if (span > 0) hi += span; else lo += span;
  }
  if (lo < 0 || hi >= v->storage_len)
    return make_error(TRS_ERR_VIEW, std::string(what) +
                      ": view reaches outside its storage (offsets " +
                      std::to_string((long long)lo) + ".." + std::to_string((long long)hi) +
                      ", storage_len " + std::to_string((long long)v->storage_len) + ")");
  return Error{};
}

bool broadcast_shapes(const int64_t* a, int an, const int64_t* b, int bn,
                      int64_t* out, int* on) {
  int nd = an > bn ? an : bn;
  if (nd > kMaxDims) return false;
  for (int i = 0; i < nd; ++i) {
    int64_t da = i < an ? a[an - 1 - i] : 1;
    int64_t db = i < bn ? b[bn - 1 - i] : 1;
    if (da == db || da == 1 || db == 1)
      out[nd - 1 - i] = da > db ? da : db;
    else
      return false;
  }
  *on = nd;
  return true;
}

bool broadcast_strides(const trs_view* v, const int64_t* target, int tn,
                       int64_t* strides_out) {
  int sn = v->ndim;
  if (sn > tn) return false;
  for (int i = 0; i < tn; ++i) {
    int64_t dd = target[tn - 1 - i];
    int64_t sd = i < sn ? v->shape[sn - 1 - i] : 1;
    int64_t ss = i < sn ? v->strides[sn - 1 - i] : 0;
    if (sd == dd)
      strides_out[tn - 1 - i] = ss;
    else if (sd == 1)
      strides_out[tn - 1 - i] = 0;
    else
      return false;
  }
  return true;
}

void fold_dims(const int64_t* shape, int nd, const int64_t (*strides)[kMaxDims],
               const int64_t* offsets, int n_ops, EwFold* f) {
  f->n_ops = n_ops;
  f->n = numel_of(shape, nd);
  for (int k = 0; k < n_ops; ++k) f->off[k] = offsets[k];
  // 1. drop size-1 dimensions (their stride is never used)
  int64_t sh[kMaxDims];
  int64_t st[kMaxOperands][kMaxDims];
  int m = 0;
  for (int d = 0; d < nd; ++d) {
    if (shape[d] == 1) continue;
    sh[m] = shape[d];
    for (int k = 0; k < n_ops; ++k) st[k][m] = strides[k][d];
    ++m;
  }
  if (m == 0 || f->n == 0) {
    f->nd = 1;
    f->shape[0] = f->n;
    for (int k = 0; k < n_ops; ++k) f->st[k][0] = 1;
    if (f->n == 0) return;
    for (int k = 0; k < n_ops; ++k) f->st[k][0] = 0;  // one element
    return;
  }
  // 2. merge dimension d into d+1 while every operand steps through the pair
  //    as one run: st[d] == st[d+1] * shape[d+1]
  int64_t osh[kMaxDims];
  int64_t ost[kMaxOperands][kMaxDims];
  int q = 0;
  osh[0] = sh[0];
  for (int k = 0; k < n_ops; ++k) ost[k][0] = st[k][0];
  for (int d = 1; d < m; ++d) {
    bool merge = true;
    for (int k = 0; k < n_ops; ++k)
      if (ost[k][q] != st[k][d] * sh[d]) { merge = false; break; }
    if (merge) {
      osh[q] *= sh[d];
      for (int k = 0; k < n_ops; ++k) ost[k][q] = st[k][d];
    } else {
      ++q;
      osh[q] = sh[d];
      for (int k = 0; k < n_ops; ++k) ost[k][q] = st[k][d];
    }
  }
  f->nd = q + 1;
  for (int d = 0; d < f->nd; ++d) {
    f->shape[d] = osh[d];
    for (int k = 0; k < n_ops; ++k) f->st[k][d] = ost[k][d];
  }
}

EwChoice choose_ew(const EwFold& f, const void* const* bases, int es) {
  EwChoice c;
  const int j = f.nd - 1;
  if (f.n == 0) { c.variant = kEwVec; return c; }
  bool out_inner_unit = f.st[0][j] == 1;
  bool all_inner_ok = out_inner_unit;
  for (int k = 1; k < f.n_ops; ++k)
    if (f.st[k][j] != 0 && f.st[k][j] != 1) all_inner_ok = false;
  if (all_inner_ok) {
    c.variant = kEwVec;
    int vec = 16 / es;
    bool can = (f.shape[j] % vec) == 0;
    for (int k = 0; k < f.n_ops && can; ++k) {
      if (f.st[k][j] == 0) continue;
      uintptr_t addr = (uintptr_t)bases[k] + (uintptr_t)(f.off[k] * es);
      if (addr % 16) can = false;
      for (int d = 0; d < j; ++d)
        if (f.st[k][d] % vec) can = false;
    }
    c.vec = can ? vec : 1;
    return c;
  }
  // tiled transpose: the output (and every non-transposed input) runs along
  // j; every transposed input has unit stride along one shared dimension i.
  if (out_inner_unit && f.nd >= 2) {
    int ti = -1;
    bool ok = true;
    for (int k = 1; k < f.n_ops && ok; ++k) {
      int64_t s = f.st[k][j];
      if (s == 0 || s == 1) continue;
      int found = -1;
      for (int d = 0; d < j; ++d)
        if (f.st[k][d] == 1) found = d;
      if (found < 0 || (ti >= 0 && found != ti)) ok = false;
      ti = found;
    }
    if (ok && ti >= 0) {
      c.variant = kEwTile;
      c.tile_dim = ti;
      return c;
    }
  }
  c.variant = kEwGeneric;
  return c;
}

}  // namespace trs
