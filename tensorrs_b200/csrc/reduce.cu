// reduce.cu -- K-RED: reductions over one or more axes of a strided view.
//
// Serves sum_axis / sum_axis_keepdim (base.rs:1051-1107, 1534-1594), the
// mean its callers build (nn/layer_norm.rs:26), max_axis / argmax_axis
// (base.rs:1396-1505), reduce_broadcast_grad (base.rs:1651-1686) and the
// fused un-broadcast of a Mul backward (autodiff/core.rs:206-227).
//
// The reference walks each output's axis serially (and leaves outputs < 8192
// on one thread).  Here the reduced and kept dimensions are folded separately
// on the host and one of three kernels is chosen:
//   red_row_kernel  the innermost reduced dimension is contiguous: one warp
//                   per output for short reductions, otherwise one CTA -- or a
//                   thread-block cluster of up to 8 CTAs whose partials meet
//                   in distributed shared memory -- per output; 16-byte loads.
//   red_col_kernel  a kept dimension is contiguous (e.g. sum over axis 0):
//                   lanes run along the kept dimension, the 8 warps of a CTA
//                   and the CTAs of a cluster split the reduced rows, and the
//                   partials meet in shared / distributed shared memory.
//   red_generic_kernel one thread per output, any layout.
// Row and column reductions with enough data take the bulk-copy pipelines
// instead (red_stream_kernel, red_cstream_kernel in reduce_kernels.cuh).
// Float sums accumulate in f64 and round once; integer sums wrap.  Max and
// argmax follow the reference's strict `>` scan exactly (see MaxState).
// Every combine happens in a fixed order, so results are deterministic.
#include <cstring>

#include "kernels.cuh"
#include "reduce.h"

namespace trs {

namespace {

bool stream_available(int dtype, int mode, int nb) {
  switch (dtype) {
    case TRS_F32: return red_stream_available<float>(mode, nb);
    case TRS_F64: return red_stream_available<double>(mode, nb);
    case TRS_I32: return red_stream_available<int32_t>(mode, nb);
    case TRS_I64: return red_stream_available<int64_t>(mode, nb);
  }
  return false;
}

void set_fd(uint32_t* dst, uint64_t v) {
  const FastDiv f = make_fastdiv((uint32_t)v);
  dst[0] = f.d;
  dst[1] = f.m;
  dst[2] = f.s;
}

// The bulk-copy row reduction: every segment start 16-byte aligned, segments
// of at least 2 KiB, 32-bit output / segment / tile counts.
// Tuning knob: reductions reading fewer bytes than this keep the register
// kernels (the pipeline's set-up does not pay off on a few tiles per CTA).
#ifndef TRS_RSTREAM_MIN_BYTES
#define TRS_RSTREAM_MIN_BYTES 0
#endif

bool plan_row_stream(const RedRequest& q, RedDev* d, RedChoice* c, int nk, int nr, int es) {
  const int VW = 16 / es;
  if (q.raw || d->L * es < 2048 || d->L % VW) return false;
  if ((uint64_t)d->n_out * (uint64_t)d->total * (uint64_t)es < (uint64_t)TRS_RSTREAM_MIN_BYTES) return false;
  if ((uint64_t)d->n_out >= (1ull << 31) || (uint64_t)d->RO >= (1ull << 31)) return false;
  int nb = 0;
  for (int k = 0; k < kRedOperands; ++k) {
    d->bulk_slot[k] = -1;
    if (!q.in[k]) continue;
    bool loaded = k == 0 || (q.mode == kRedSum3 && ((k == 1 && d->has_gate) || (k == 2 && d->has_mul))) ||
                  (q.mode == kRedAffineRelu && k == 1);
    if (!loaded) continue;
    if (d->inner_bcast[k]) {
      if (q.mode == kRedAffineRelu) return false;  // x must run along the segments
      continue;
    }
    // every segment start of a bulk operand must be 16-byte aligned
    if (((uintptr_t)q.in[k]->data + (uintptr_t)(q.in[k]->offset * es)) % 16) return false;
    for (int i = 0; i < nk; ++i) if (d->kst[k][i] % VW) return false;
    for (int i = 0; i + 1 < nr; ++i) if (d->rst[k][i] % VW) return false;
    d->bulk_slot[k] = nb++;
  }
  if (d->bulk_slot[0] != 0 || (q.mode == kRedAffineRelu && d->bulk_slot[1] != 1)) return false;
  if (!stream_available(q.in[0]->dtype, q.mode, nb)) return false;
  d->err = async_error_word();
  if (!d->err) return false;
  const int64_t tile = 16384 / es;
  d->tps = (d->L + tile - 1) / tile;
  const uint64_t tiles_out = (uint64_t)d->RO * (uint64_t)d->tps;
  if (tiles_out >= (1ull << 31)) return false;
  // Split each output's tiles into P parts so the items fill the resident
  // CTAs (two per SM) in whole waves: the smallest P whose last wave is at
  // least 95% full, parts of at least 4 tiles (at most 64 parts).
  const DeviceInfo& dev = current_device_info();
  const uint64_t cap = (uint64_t)dev.sm_count * 2;
  uint64_t max_p = tiles_out / 4;
  if (max_p < 1) max_p = 1;
  if (max_p > 64) max_p = 64;
  uint64_t P = 1;
  double best = -1.0;
  // Outputs that fit one wave and occupy at least half the resident CTAs
  // keep P = 1: every item then runs from the start, more than enough copies
  // are in flight to hold HBM busy, and no partials need a second kernel.
  if ((uint64_t)d->n_out <= cap && 2 * (uint64_t)d->n_out >= cap) max_p = 1;
  for (uint64_t q = 1; q <= max_p; ++q) {
    const uint64_t tpp = (tiles_out + q - 1) / q;
    const uint64_t parts = (tiles_out + tpp - 1) / tpp;
    const uint64_t items = (uint64_t)d->n_out * parts;
    const uint64_t waves = (items + cap - 1) / cap;
    const double eff = (double)items / (double)(waves * cap);
    if (eff > best + 1e-9) { best = eff; P = q; }
    if (eff >= 0.95) break;
  }
  d->tpp = (int64_t)((tiles_out + P - 1) / P);
  d->P = (int64_t)((tiles_out + d->tpp - 1) / d->tpp);
  set_fd(d->f_tps, (uint64_t)d->tps);
  for (int i = 0; i < nk; ++i) set_fd(d->fk[i], (uint64_t)d->kshape[i]);
  for (int i = 0; i < nr; ++i) set_fd(d->fr[i], (uint64_t)d->rshape[i]);
  c->variant = kRedRowStream;
  c->nb = nb;
  return true;
}

bool cstream_available(int dtype, int mode, int nb) {
  switch (dtype) {
    case TRS_F32: return red_cstream_available<float>(mode, nb);
    case TRS_F64: return red_cstream_available<double>(mode, nb);
    case TRS_I32: return red_cstream_available<int32_t>(mode, nb);
    case TRS_I64: return red_cstream_available<int64_t>(mode, nb);
  }
  return false;
}

// The bulk-copy column reduction: W (the contiguous kept dimension) at least
// 512 bytes and a multiple of 16 bytes, every staged row segment 16-byte
// aligned, at least 1 MiB of input, 32-bit row / output / item counts.
// Chooses the column block width, the rows per stage and the split of the
// reduced rows into parts so the work items fill the resident CTAs evenly.
bool plan_col_stream(const RedRequest& q, RedDev* d, RedChoice* c, int nk_outer, int nr, int es) {
  const int VW = 16 / es;
  if (q.mode == kRedAffineRelu) return false;
  if (d->W * es < 512 || (d->W * es) % 16) return false;
  if ((uint64_t)d->total * (uint64_t)d->W * (uint64_t)es < (1ull << 20)) return false;
  if ((uint64_t)d->total >= (1ull << 31) || (uint64_t)d->n_out >= (1ull << 31)) return false;
  int nb = 0;
  for (int k = 0; k < kRedOperands; ++k) {
    d->bulk_slot[k] = -1;
    if (!q.in[k]) continue;
    const bool loaded = k == 0 || (q.mode == kRedSum3 && ((k == 1 && d->has_gate) || (k == 2 && d->has_mul)));
    if (!loaded) continue;
    if (d->wst[k] == 0 && k > 0) continue;  // constant along W: one scalar per row
    if (d->wst[k] != 1) return false;
    if (((uintptr_t)q.in[k]->data + (uintptr_t)(q.in[k]->offset * es)) % 16) return false;
    for (int i = 0; i < nk_outer; ++i) if (d->kst[k][i] % VW) return false;
    for (int i = 0; i < nr; ++i) if (d->rst[k][i] % VW) return false;
    d->bulk_slot[k] = nb++;
  }
  if (d->bulk_slot[0] != 0) return false;
  if (!cstream_available(q.in[0]->dtype, q.mode, nb)) return false;
  d->err = async_error_word();
  if (!d->err) return false;
  const int64_t pitch = d->W * es < kCsMaxPitch ? d->W * es : kCsMaxPitch;
  d->cs_pitch = (int32_t)pitch;
  d->cs_wt = (int32_t)(pitch / es);
  d->cs_rt = (int32_t)(kCsStageBytes / pitch < 32 ? kCsStageBytes / pitch : 32);
  int cpad = 1;
  while (cpad < d->cs_wt / VW) cpad *= 2;
  d->cs_cpr_pad = cpad;
  d->cs_ncb = (d->W + d->cs_wt - 1) / d->cs_wt;
  const uint64_t base = (uint64_t)d->n_out_outer * (uint64_t)d->cs_ncb;
  const DeviceInfo& dev = current_device_info();
  int per_sm = kSmemPerSm / (cs_smem_bytes(nb) + 1024);
  if (per_sm > 2) per_sm = 2;
  if (per_sm < 1) per_sm = 1;
  const uint64_t cap = (uint64_t)dev.sm_count * (uint64_t)per_sm;
  // parts of at least 8 stages of rows keep the partials under ~6% of the input
  uint64_t max_p = (uint64_t)d->total / (8ull * (uint64_t)d->cs_rt);
  if (max_p < 1) max_p = 1;
  if (max_p > 64) max_p = 64;
  uint64_t best_p = 1;
  double best_eff = -1.0;
  for (uint64_t P = 1; P <= max_p; ++P) {
    const uint64_t items = base * P;
    const uint64_t waves = (items + cap - 1) / cap;
    const double eff = (double)items / (double)(waves * cap);
    if (eff > best_eff + 1e-9) { best_eff = eff; best_p = P; }
    if (eff >= 0.9) break;
  }
  const uint64_t rt = (uint64_t)d->cs_rt;
  uint64_t rp = ((uint64_t)d->total + best_p - 1) / best_p;
  rp = (rp + rt - 1) / rt * rt;
  d->cs_rp = (int64_t)rp;
  d->P = (int64_t)(((uint64_t)d->total + rp - 1) / rp);
  if (base * (uint64_t)d->P >= (1ull << 31)) return false;
  for (int i = 0; i < nk_outer; ++i) set_fd(d->fk[i], (uint64_t)d->kshape[i]);
  for (int i = 0; i < nr; ++i) set_fd(d->fr[i], (uint64_t)d->rshape[i]);
  c->variant = kRedColStream;
  c->nb = nb;
  c->per_sm = per_sm;
  return true;
}

}  // namespace

Error plan_reduce(const RedRequest& q, RedDev* d, RedChoice* c) {
  std::memset(d, 0, sizeof(*d));
  const trs_view* x = q.in[0];
  const int nd = x->ndim;
  d->mode = q.mode;
  d->raw = q.raw ? 1 : 0;
  d->idx_base = q.idx_base;
  d->has_gate = q.in[1] != nullptr && q.mode == kRedSum3;
  d->has_mul = q.in[2] != nullptr && q.mode == kRedSum3;
  for (int k = 0; k < kRedOperands; ++k) {
    d->in[k] = q.in[k] ? q.in[k]->data : x->data;
    d->off[k] = q.in[k] ? q.in[k]->offset : 0;
  }
  for (int m = 0; m < 2; ++m) {
    d->out[m] = q.out[m] ? q.out[m]->data : nullptr;
    d->out_off[m] = q.out[m] ? q.out[m]->offset : 0;
  }
  // split the dimensions into kept and reduced, dropping size-1 dims
  int64_t ksh[kMaxDims], kst[kRedOperands + 2][kMaxDims];
  int64_t rsh[kMaxDims], rst[kRedOperands][kMaxDims];
  int nk = 0, nr = 0;
  d->total = 1;
  d->n_out = 1;
  for (int i = 0; i < nd; ++i) {
    const int64_t s = x->shape[i];
    if (q.reduce_mask & (1u << i)) {
      d->total *= s;
      if (s == 1) continue;
      rsh[nr] = s;
      for (int k = 0; k < kRedOperands; ++k) rst[k][nr] = q.in[k] ? q.op_strides[k][i] : 0;
      ++nr;
    } else {
      d->n_out *= s;
      if (s == 1) continue;
      ksh[nk] = s;
      for (int k = 0; k < kRedOperands; ++k) kst[k][nk] = q.in[k] ? q.op_strides[k][i] : 0;
      kst[kRedOperands][nk] = q.out_strides[0][i];
      kst[kRedOperands + 1][nk] = q.out_strides[1][i];
      ++nk;
    }
  }
  // fold adjacent dims of each group when every array steps through them as one run
  auto fold = [](int64_t* sh, int64_t (*st)[kMaxDims], int n_arr, int& n) {
    if (n == 0) return;
    int w = 0;
    for (int i = 1; i < n; ++i) {
      bool merge = true;
      for (int k = 0; k < n_arr; ++k)
        if (st[k][w] != st[k][i] * sh[i]) { merge = false; break; }
      if (merge) {
        sh[w] *= sh[i];
        for (int k = 0; k < n_arr; ++k) st[k][w] = st[k][i];
      } else {
        ++w;
        sh[w] = sh[i];
        for (int k = 0; k < n_arr; ++k) st[k][w] = st[k][i];
      }
    }
    n = w + 1;
  };
  const bool single_axis = q.mode == kRedMax || q.mode == kRedArgmax;
  fold(ksh, kst, kRedOperands + 2, nk);
  if (!single_axis) fold(rsh, rst, kRedOperands, nr);
  const int es = dtype_size(x->dtype);
  const int VW = 16 / es;
  c->variant = kRedGeneric;
  c->vec = 1;
  c->warp_mode = false;
  c->cluster = 1;
  // unit-stride operand classes
  auto inner_ok = [&](int64_t s0, const int64_t* ss) {
    if (s0 != 1) return false;
    for (int k = 1; k < kRedOperands; ++k)
      if (q.in[k] && ss[k] != 0 && ss[k] != 1) return false;
    return true;
  };
  // row variant: the innermost reduced dim is contiguous in operand 0
  int64_t rs_last[kRedOperands] = {0, 0, 0, 0};
  if (nr > 0)
    for (int k = 0; k < kRedOperands; ++k) rs_last[k] = rst[k][nr - 1];
  // an empty reduction (some reduced dim is 0) takes the generic kernel,
  // which writes the empty sum (0) or 0/0 for the mean
  const bool row_ok = nr > 0 && d->total > 0 && inner_ok(rs_last[0], rs_last);
  // column variant: the innermost kept dim is contiguous in operand 0
  int64_t ks_last[kRedOperands] = {0, 0, 0, 0};
  if (nk > 0)
    for (int k = 0; k < kRedOperands; ++k) ks_last[k] = kst[k][nk - 1];
  const bool col_ok = nk > 0 && d->total > 0 && !row_ok && q.mode != kRedAffineRelu &&
                      inner_ok(ks_last[0], ks_last);
  // copy the folded dims into the descriptor
  d->nk = nk;
  for (int i = 0; i < nk; ++i) {
    d->kshape[i] = ksh[i];
    for (int k = 0; k < kRedOperands; ++k) d->kst[k][i] = kst[k][i];
    d->kout[0][i] = kst[kRedOperands][i];
    d->kout[1][i] = kst[kRedOperands + 1][i];
  }
  d->nr = nr;
  for (int i = 0; i < nr; ++i) {
    d->rshape[i] = rsh[i];
    for (int k = 0; k < kRedOperands; ++k) d->rst[k][i] = rst[k][i];
  }
  if (row_ok) {
    c->variant = kRedRow;
    d->L = rsh[nr - 1];
    d->RO = d->total / d->L;
    for (int k = 0; k < kRedOperands; ++k) d->inner_bcast[k] = rs_last[k] == 0 ? 1 : 0;
    if (plan_row_stream(q, d, c, nk, nr, es)) return Error{};
    // the row kernel walks reduced dims 0..nr-2 as "outer rows"
    bool vec = (d->L % VW) == 0;
    for (int k = 0; k < kRedOperands && vec; ++k) {
      // the operands the row kernel reads with vector loads
      const bool vector_read =
          q.in[k] && !d->inner_bcast[k] &&
          (k == 0 || (k == 1 && (q.mode == kRedAffineRelu || d->has_gate)) ||
           (k == 2 && q.mode == kRedSum3 && d->has_mul));
      if (!vector_read) continue;
      if (((uintptr_t)q.in[k]->data + (uintptr_t)(q.in[k]->offset * es)) % 16) vec = false;
      for (int i = 0; i < nk; ++i) if (kst[k][i] % VW) vec = false;
      for (int i = 0; i + 1 < nr; ++i) if (rst[k][i] % VW) vec = false;
    }
    c->vec = vec ? VW : 1;
    if (d->total <= 4096 && q.mode != kRedAffineRelu) {
      c->warp_mode = true;
    } else {
      // enough CTAs to fill the GPU: up to 8 per output in a cluster
      const DeviceInfo& dev = current_device_info();
      int cl = 1;
      while (cl < 8 && (uint64_t)d->n_out * cl < (uint64_t)dev.sm_count * 4 &&
             (uint64_t)d->total / (uint64_t)(cl * 2) >= 8192)
        cl *= 2;
      c->cluster = cl;
    }
    return Error{};
  }
  if (col_ok) {
    c->variant = kRedCol;
    d->W = ksh[nk - 1];
    for (int k = 0; k < kRedOperands; ++k) d->wst[k] = ks_last[k];
    d->wout[0] = kst[kRedOperands][nk - 1];
    d->wout[1] = kst[kRedOperands + 1][nk - 1];
    d->nk = nk - 1;  // the column kernel walks the remaining kept dims as "outer"
    d->n_out_outer = d->n_out / d->W;
    if (plan_col_stream(q, d, c, nk - 1, nr, es)) return Error{};
    bool vec = (d->W % VW) == 0;
    for (int k = 0; k < kRedOperands && vec; ++k) {
      if (!q.in[k] || k > 0) continue;
      if (((uintptr_t)q.in[k]->data + (uintptr_t)(q.in[k]->offset * es)) % 16) vec = false;
      for (int i = 0; i + 1 < nk; ++i) if (kst[k][i] % VW) vec = false;
      for (int i = 0; i < nr; ++i) if (rst[k][i] % VW) vec = false;
    }
    c->vec = vec ? VW : 1;
    const DeviceInfo& dev = current_device_info();
    const uint64_t blocks = (uint64_t)((d->W + 32 * c->vec - 1) / (32 * c->vec)) * (uint64_t)d->n_out_outer;
    int cl = 1;
    while (cl < 8 && blocks * cl < (uint64_t)dev.sm_count * 4 && (uint64_t)d->total / (uint64_t)(cl * 2) >= 64)
      cl *= 2;
    c->cluster = cl;
    return Error{};
  }
  return Error{};
}

Error run_reduce(const RedRequest& q, cudaStream_t stream) {
  RedDev d;
  RedChoice c;
  Error e = plan_reduce(q, &d, &c);
  if (!e.ok()) return e;
  switch (q.in[0]->dtype) {
    case TRS_F32: return red_launch<float>(d, c, stream);
    case TRS_F64: return red_launch<double>(d, c, stream);
    case TRS_I32: return red_launch<int32_t>(d, c, stream);
    case TRS_I64: return red_launch<int64_t>(d, c, stream);
  }
  return make_error(TRS_ERR_DTYPE, "unknown dtype");
}

}  // namespace trs
