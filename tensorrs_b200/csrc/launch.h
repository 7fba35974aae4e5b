// launch.h -- host-side declarations of the element-wise launchers (ew*.cu),
// usable from plain C++ translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "plan.h"
#include "runtime.h"

namespace trs {

// The cross-rank combine of a sharded sum, done by the kernel that folds the
// per-block partials (sum_exchange_kernel): every rank's slot buffer mapped
// into this process over NVLink (comm.cpp sets it up).  A rank's buffer holds
// two sets (by the parity of the call's sequence number) of `world` slots of
// {accumulator bits, sequence number}; slot r of a set is written by rank r.
struct PeerExchange {
  unsigned long long* const* peers = nullptr;  // device array: rank r's slot buffer
  int world = 0;
  int rank = 0;
  unsigned long long seq = 0;                  // this call's number, the same on every rank
  int* err = nullptr;                          // async-error word of this device
};

// Where a fused sum goes: a one-element view of the input dtype, or (for the
// sharded path) a raw f64/u32/u64 accumulator written without rounding, or
// the view after the cross-rank combine of `exchange`.
struct SumTarget {
  const trs_view* view = nullptr;  // rounded result
  void* raw_acc = nullptr;         // accumulator before rounding
  // Caller-provided device memory for the per-block partial sums; when null
  // they come from the scratch pool.
  void* partials = nullptr;
  size_t partials_bytes = 0;
  const PeerExchange* exchange = nullptr;  // sum over the ranks before rounding
};

// Largest communicator the peer exchange serves (one slot per rank).
constexpr int kMaxExchangeRanks = 64;

// A rank's exchange buffer (one allocation, mapped by every peer through
// CUDA IPC): the sharded sums' slots (2 sets x world x {accumulator, seq}),
// then the axis-0 exchange's flags (2 parities x world seq words, written by
// the peers), then its two arenas of kAxis0Arena bytes (this rank's partial
// rows of the calls of each parity, read by the peers).
constexpr size_t kAxis0Arena = (size_t)8 << 20;
inline size_t x_flags_off(int world) { return ((size_t)2 * world * 2 * 8 + 255) / 256 * 256; }
inline size_t x_arena_off(int world) { return (x_flags_off(world) + (size_t)2 * world * 8 + 255) / 256 * 256; }
inline size_t x_buffer_bytes(int world) { return x_arena_off(world) + 2 * kAxis0Arena; }

// One sharded axis-0 reduction's exchange over peer memory: this rank's
// partials are in its own arena of `parity`; the publish kernel stores `seq`
// into every peer's flag of (parity, rank), and the combine kernel waits
// (bounded) for every rank's flag in this rank's buffer, then reads every
// rank's partials in rank order.
struct Axis0Exchange {
  unsigned long long* const* peers = nullptr;  // device array: rank r's exchange buffer
  int world = 0;
  int rank = 0;
  unsigned long long seq = 0;
  int parity = 0;
  size_t flags_off = 0, arena_off = 0;         // bytes into every buffer
  int* err = nullptr;
};
Error run_axis0_publish(const Axis0Exchange& x, cudaStream_t stream);
Error run_axis0_sum_combine(int dtype, const Axis0Exchange& x, const trs_view* out, cudaStream_t stream);
Error run_axis0_max_combine(int dtype, const Axis0Exchange& x, int first_rank, const trs_view* out, bool argmax,
                            cudaStream_t stream);

// Element-wise program over `in`; writes `out` unless it is null, and the sum
// of the results to `sum` when it is non-null.
Error run_elementwise(const trs_ew_program& prog, const trs_view* in,
                      const trs_view* out, const SumTarget* sum, cudaStream_t stream);

// trs_elementwise_row_sums in one pass (rowsum.cu): Y = prog(in) into the
// contiguous `out`, its sums along the last axis into `rows_out` (contiguous,
// or null) and its total into `total` (or null).  Views are validated by the
// caller.  *taken is false, with nothing launched, when the layout is not one
// the fused kernel serves (fewer than 256 rows, a strided or transposed
// operand, integer division); the caller then runs the three passes.
Error run_row_sums_fused(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                         const trs_view* rows_out, const trs_view* total, cudaStream_t stream, bool* taken);

// Plan only (trs_plan_elementwise).
Error plan_elementwise(const trs_ew_program& prog, const trs_view* in,
                       const trs_view* out, EwFold* fold, EwChoice* choice);

// Writes a raw accumulator (f64 for floats, wrapping unsigned for integers)
// into a one-element view of `dtype`, rounding once.
Error run_acc_to_value(int dtype, const void* acc, const trs_view* out, cudaStream_t stream);

Error run_fill(trs_view* out, uint64_t seed, uint64_t first, double lo, double hi, bool normal,
               cudaStream_t stream);

// Sharded axis-0 reductions (shard.cu): round `n = numel(out)` all-reduced
// accumulators into `out`; fold `nranks` gathered max records per output
// (`first_rank`: the lowest rank that holds rows, whose first row is global
// row 0).
Error run_accs_to_view(int dtype, const void* acc, const trs_view* out, cudaStream_t stream);
Error run_max_records(int dtype, const void* records, int nranks, int first_rank, const trs_view* out,
                      bool argmax, cudaStream_t stream);
size_t max_record_size(int dtype);

// True when a program needs no transcendental (no powf, exp, tanh, ln).
inline bool is_simple_program(const trs_ew_program& p) {
  if (p.n_in >= 2 && p.op1 == TRS_POW) return false;
  if (p.n_in >= 3 && p.op2 == TRS_POW) return false;
  switch (p.epilogue) {
    case TRS_UN_SIGMOID: case TRS_UN_TANH: case TRS_UN_ELU: case TRS_UN_SELU: case TRS_UN_EXP:
    case TRS_UN_LN: case TRS_UN_POW_SCALAR: case TRS_UN_RPOW_SCALAR:
      return false;
  }
  return true;
}

// The compile-time program code (ProgCode in device_ops.cuh) of a program:
// a specialised code for the hot fused patterns, else a runtime code.
int program_code(const trs_ew_program& p, bool is_float_dtype);

// Per-dtype launch of a prepared element-wise op (ew_<dtype>.cu).
struct EwPrepared {
  EwFold fold;
  EwChoice choice;
  int dtype = TRS_F32;
};
template <class T>
Error ew_launch(const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                const SumTarget* sum, const EwPrepared& pr, cudaStream_t stream);

}  // namespace trs
