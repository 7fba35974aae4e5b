// comm.cpp -- several GPUs: each rank holds a leading-dimension shard; the
// element-wise part needs no communication and the full sum combines per-rank
// f64 partials over NVLink.
//
// The full sum's combine is fused into the kernel that folds this rank's
// partials (sum_exchange_kernel): at communicator creation every rank
// allocates a small slot buffer, exports it as a CUDA IPC handle, the handles
// travel by one NCCL all-gather, and every rank maps its peers' buffers; a
// sharded sum then writes its accumulator straight into every peer's buffer
// and reads the others' from its own, with no collective launch.  When the
// mapping cannot be made on some rank (peers not visible to the process, no
// peer access), every rank agrees (an all-reduce of a flag) to combine with
// ncclAllReduce instead; TRS_PEER_EXCHANGE=0 in the environment forces that.
// Axis-0 reductions (many values) keep NCCL.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2), so a process that never
// creates a communicator does not need it, and a process that already loaded
// NCCL (e.g. through PyTorch) shares that copy.  Communicators are created
// non-blocking and polled against a deadline; a rank that never joins makes
// the others return TRS_ERR_TIMEOUT instead of hanging.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/trs.h"
#include "launch.h"
#include "reduce.h"
#include "runtime.h"

using namespace trs;

struct trs_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int timeout_ms = 0;
  // peer exchange of the sharded sums (xpeers null: combine through NCCL)
  unsigned long long* xbuf = nullptr;    // this rank's slot buffer
  unsigned long long** xpeers = nullptr; // device array: every rank's buffer, mapped here
  std::vector<void*> xopened;            // IPC mappings of the peers' buffers
  unsigned long long xseq = 0;           // sequence number of the last sharded sum
  unsigned long long xseq_a0 = 0;        // ... and of the last sharded axis-0 exchange
};

namespace {

struct Nccl {
  bool loaded = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      n.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "");
      return;
    }
#define TRS_SYM(field, name)                                              \
  n.field = reinterpret_cast<decltype(n.field)>(dlsym(h, name));          \
  if (!n.field) { n.why = std::string("missing NCCL symbol ") + name; return; }
    TRS_SYM(GetUniqueId, "ncclGetUniqueId");
    TRS_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    TRS_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    TRS_SYM(CommAbort, "ncclCommAbort");
    TRS_SYM(CommDestroy, "ncclCommDestroy");
    TRS_SYM(AllReduce, "ncclAllReduce");
    TRS_SYM(AllGather, "ncclAllGather");
    TRS_SYM(GetErrorString, "ncclGetErrorString");
#undef TRS_SYM
    n.loaded = true;
  });
  return n;
}

trs_status finish(const Error& e) {
  if (!e.ok()) set_last_error(e.msg);
  return e.status;
}

Error nccl_error(ncclResult_t r, const char* what) {
  Nccl& n = nccl();
  return make_error(TRS_ERR_NCCL, std::string(what) + ": " +
                                      (n.GetErrorString ? n.GetErrorString(r) : "nccl error"));
}

// Waits until a non-blocking communicator leaves ncclInProgress: a few
// thousand yielding polls first (an enqueue that is merely busy clears in
// microseconds, and a sleep here would starve the GPU's queue), then polls
// 200 us apart until the deadline.
Error wait_ready(trs_comm* c, const char* what) {
  Nccl& n = nccl();
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (int polls = 0;; ++polls) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return nccl_error(r, "ncclCommGetAsyncError");
    if (st == ncclSuccess) return Error{};
    if (st != ncclInProgress) return nccl_error(st, what);
    if (std::chrono::steady_clock::now() > deadline)
      return make_error(TRS_ERR_TIMEOUT, std::string(what) + ": timed out");
    if (polls < 4096)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// ---- the peer exchange ------------------------------------------------------

Error nccl_call(trs_comm* c, ncclResult_t r, const char* what);

// Unmaps the peers' buffers and frees this rank's, after this device's work
// has finished (an exchange kernel of this rank may still be writing into a
// peer's buffer).  A peer writes into this rank's buffer only inside calls
// this rank also makes, before this rank's kernel of that call can finish.
void teardown_exchange(trs_comm* c) {
  if (c->xbuf || c->xpeers || !c->xopened.empty()) cudaDeviceSynchronize();
  for (void* p : c->xopened) cudaIpcCloseMemHandle(p);
  c->xopened.clear();
  if (c->xpeers) cudaFree(c->xpeers);
  if (c->xbuf) cudaFree(c->xbuf);
  c->xpeers = nullptr;
  c->xbuf = nullptr;
  cudaGetLastError();
}

// Called by every rank of a new communicator (a collective: one all-gather
// and one all-reduce).  Leaves c->xpeers set when every rank mapped every
// peer's slot buffer, null (NCCL combine) otherwise.
Error setup_exchange(trs_comm* c) {
  const int R = c->nranks;
  const char* env = std::getenv("TRS_PEER_EXCHANGE");
  const bool wanted = !(env && env[0] == '0');
  if (R < 2 || R > kMaxExchangeRanks) return Error{};
  Nccl& n = nccl();
  cudaStream_t s = nullptr;
  cudaError_t ce = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (ce != cudaSuccess) return cuda_error(ce, "cudaStreamCreateWithFlags");
  int ok = wanted ? 1 : 0;
  const size_t bytes = x_buffer_bytes(R);  // sum slots, axis-0 flags and arenas
  if (ok && cudaMalloc(&c->xbuf, bytes) != cudaSuccess) ok = 0;
  if (ok && cudaMemset(c->xbuf, 0, bytes) != cudaSuccess) ok = 0;
  cudaIpcMemHandle_t mine;
  std::memset(&mine, 0, sizeof(mine));
  if (ok && cudaIpcGetMemHandle(&mine, c->xbuf) != cudaSuccess) ok = 0;
  cudaGetLastError();
  // every rank's handle (an all-gather every rank takes part in, ok or not),
  // then the agreement flag
  const size_t hs = sizeof(cudaIpcMemHandle_t);
  char* dev = nullptr;
  ce = cudaMalloc(&dev, hs * (size_t)(R + 1) + 16);
  if (ce != cudaSuccess) {
    cudaStreamDestroy(s);
    teardown_exchange(c);
    return cuda_error(ce, "cudaMalloc (exchange set-up)");
  }
  std::vector<char> all(hs * (size_t)R);
  Error e;
  ce = cudaMemcpy(dev + hs * R, &mine, hs, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) e = cuda_error(ce, "cudaMemcpy");
  if (e.ok()) e = nccl_call(c, n.AllGather(dev + hs * R, dev, hs, ncclUint8, c->comm, s), "ncclAllGather (handles)");
  if (e.ok()) {
    ce = cudaMemcpyAsync(all.data(), dev, hs * R, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) e = cuda_error(ce, "reading the handles");
  }
  std::vector<unsigned long long*> table(R, nullptr);
  if (e.ok() && ok) {
    table[c->rank] = c->xbuf;
    for (int r = 0; r < R && ok; ++r) {
      if (r == c->rank) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, all.data() + hs * r, hs);
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
        break;
      }
      c->xopened.push_back(p);
      table[r] = static_cast<unsigned long long*>(p);
    }
  }
  // agreement: the exchange is used only if every rank mapped every peer
  int32_t* flag = reinterpret_cast<int32_t*>(dev + hs * (R + 1));
  int32_t agreed = 0;
  if (e.ok()) {
    ce = cudaMemcpy(flag, &ok, sizeof(int32_t), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) e = cuda_error(ce, "cudaMemcpy");
  }
  if (e.ok()) e = nccl_call(c, n.AllReduce(flag, flag, 1, ncclInt32, ncclMin, c->comm, s), "ncclAllReduce (agreement)");
  if (e.ok()) {
    ce = cudaMemcpyAsync(&agreed, flag, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) e = cuda_error(ce, "reading the agreement");
  }
  if (e.ok() && agreed) {
    ce = cudaMalloc(&c->xpeers, sizeof(unsigned long long*) * R);
    if (ce == cudaSuccess)
      ce = cudaMemcpy(c->xpeers, table.data(), sizeof(unsigned long long*) * R, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) e = cuda_error(ce, "the peer table");
  }
  cudaFree(dev);
  cudaStreamDestroy(s);
  if (!e.ok() || !agreed) teardown_exchange(c);
  return e;
}

ncclDataType_t acc_type(int dtype) {
  switch (dtype) {
    case TRS_I32: return ncclUint32;
    case TRS_I64: return ncclUint64;
    default: return ncclFloat64;
  }
}

Error sharded_sum(trs_comm* c, const trs_ew_program& prog, const trs_view* in, const trs_view* out,
                  trs_view* sum_out, cudaStream_t stream) {
  if (!c || !c->comm) return make_error(TRS_ERR_ARG, "null communicator");
  Error e = validate_view(sum_out, "sum output");
  if (!e.ok()) return e;
  if (numel_of(sum_out->shape, sum_out->ndim) != 1) return make_error(TRS_ERR_SHAPE, "sum output must hold one element");
  if (c->xpeers) {  // the combine fused into the partials' fold, over NVLink
    PeerExchange x;
    x.peers = c->xpeers;
    x.world = c->nranks;
    x.rank = c->rank;
    x.seq = ++c->xseq;
    x.err = async_error_word();
    SumTarget t;
    t.view = sum_out;
    t.exchange = &x;
    return run_elementwise(prog, in, out, &t, stream);
  }
  Scratch acc;
  e = acc.alloc(8, stream);
  if (!e.ok()) return e;
  SumTarget t;
  t.raw_acc = acc.get();
  e = run_elementwise(prog, in, out, &t, stream);
  if (!e.ok()) return e;
  Nccl& n = nccl();
  ncclResult_t r = n.AllReduce(acc.get(), acc.get(), 1, acc_type(in[0].dtype), ncclSum, c->comm, stream);
  if (r == ncclInProgress) {
    e = wait_ready(c, "ncclAllReduce");
    if (!e.ok()) return e;
  } else if (r != ncclSuccess) {
    return nccl_error(r, "ncclAllReduce");
  }
  return run_acc_to_value(in[0].dtype, acc.get(), sum_out, stream);
}

// A collective call on a non-blocking communicator.
Error nccl_call(trs_comm* c, ncclResult_t r, const char* what) {
  if (r == ncclInProgress) return wait_ready(c, what);
  if (r != ncclSuccess) return nccl_error(r, what);
  return Error{};
}

enum Axis0Op { kAxis0Sum, kAxis0Max, kAxis0Argmax };

// This rank's partials of sum_axis(0) / max_axis(0) / argmax_axis(0) (f64 or
// wrapping accumulators, or max records with global indices from `base`),
// unrounded, contiguous at `dst`.
Error axis0_local(int op, const trs_view* shard, const trs_view* out, int64_t base, void* dst, int64_t nout,
                  cudaStream_t stream) {
  if (nout == 0) return Error{};
  trs_view pv;
  std::memset(&pv, 0, sizeof(pv));
  pv.data = dst;
  pv.dtype = shard->dtype;
  pv.ndim = out->ndim;
  pv.storage_len = nout;
  int64_t step = 1;
  for (int i = out->ndim - 1; i >= 0; --i) {
    pv.shape[i] = out->shape[i];
    pv.strides[i] = step;
    step *= out->shape[i];
  }
  RedRequest q;
  q.mode = op == kAxis0Sum ? kRedSum : (op == kAxis0Max ? kRedMax : kRedArgmax);
  q.raw = true;
  q.idx_base = base;
  q.reduce_mask = 1u;
  q.in[0] = shard;
  for (int i = 0; i < shard->ndim; ++i) q.op_strides[0][i] = shard->strides[i];
  q.out[0] = &pv;
  for (int i = 1; i < shard->ndim; ++i) q.out_strides[0][i] = pv.strides[i - 1];
  return run_reduce(q, stream);
}

// The combine through NCCL: an all-reduce of the f64 partials, or an
// all-gather of every rank's max records folded in rank order.
Error axis0_combine_nccl(trs_comm* c, int op, const trs_view* shard, const trs_view* out, int64_t base,
                         int first_rank, int64_t nout, cudaStream_t stream) {
  Nccl& n = nccl();
  const int R = c->nranks;
  const int dt = shard->dtype;
  const size_t rec = op == kAxis0Sum ? (dt == TRS_I32 ? 4 : 8) : max_record_size(dt);
  const size_t slots = op == kAxis0Sum ? 1 : (size_t)R;
  Scratch part;
  Error e = part.alloc(rec * (size_t)(nout > 0 ? nout : 1) * slots, stream);
  if (!e.ok()) return e;
  char* mine_at = part.as<char>() + (op == kAxis0Sum ? 0 : rec * (size_t)nout * (size_t)c->rank);
  e = axis0_local(op, shard, out, base, mine_at, nout, stream);
  if (!e.ok()) return e;
  if (op == kAxis0Sum) {
    e = nccl_call(c, n.AllReduce(part.get(), part.get(), (size_t)nout, acc_type(dt), ncclSum, c->comm, stream),
                  "ncclAllReduce (partial sums)");
    if (!e.ok()) return e;
    return run_accs_to_view(dt, part.get(), out, stream);
  }
  e = nccl_call(c, n.AllGather(mine_at, part.get(), rec * (size_t)nout, ncclUint8, c->comm, stream),
                "ncclAllGather (max records)");
  if (!e.ok()) return e;
  return run_max_records(dt, part.get(), R, first_rank, out, op == kAxis0Argmax, stream);
}

// The combine over NVLink peer memory: this rank's partials go into its own
// arena of the call's parity, the publish kernel tells every peer, and the
// combine kernel reads every rank's partials in rank order (the same order
// on every rank) once every rank has published.  A rank cannot start call
// c + 2 (the same parity) before every rank has published call c + 1, which
// each does only after finishing call c, so no arena is overwritten while a
// peer still reads it.
Error axis0_combine_peers(trs_comm* c, int op, const trs_view* shard, const trs_view* out, int64_t base,
                          int first_rank, int64_t nout, cudaStream_t stream) {
  Axis0Exchange x;
  x.peers = c->xpeers;
  x.world = c->nranks;
  x.rank = c->rank;
  x.seq = ++c->xseq_a0;
  x.parity = (int)(x.seq & 1u);
  x.flags_off = x_flags_off(c->nranks);
  x.arena_off = x_arena_off(c->nranks);
  x.err = async_error_word();
  char* mine = reinterpret_cast<char*>(c->xbuf) + x.arena_off + (size_t)x.parity * kAxis0Arena;
  Error e = axis0_local(op, shard, out, base, mine, nout, stream);
  if (!e.ok()) return e;
  e = run_axis0_publish(x, stream);
  if (!e.ok()) return e;
  if (op == kAxis0Sum) return run_axis0_sum_combine(shard->dtype, x, out, stream);
  return run_axis0_max_combine(shard->dtype, x, first_rank, out, op == kAxis0Argmax, stream);
}

// sum_axis(0) / max_axis(0) / argmax_axis(0) of a tensor split on axis 0.
Error sharded_axis0(trs_comm* c, int op, const trs_view* shard, const trs_view* out, cudaStream_t stream) {
  if (!c || !c->comm) return make_error(TRS_ERR_ARG, "null communicator");
  Error e = validate_view(shard, "shard");
  if (!e.ok()) return e;
  e = validate_view(out, "output");
  if (!e.ok()) return e;
  if (shard->ndim < 1) return make_error(TRS_ERR_AXIS, "!!!Axis index out of range!!!");
  const int dt = shard->dtype;
  if (out->dtype != (op == kAxis0Argmax ? (int)TRS_I64 : dt))
    return make_error(TRS_ERR_DTYPE, op == kAxis0Argmax ? "argmax output must be i64" : "output dtype differs");
  bool ok = out->ndim == shard->ndim - 1;
  for (int i = 1; ok && i < shard->ndim; ++i) ok = out->shape[i - 1] == shard->shape[i];
  if (!ok) return make_error(TRS_ERR_SHAPE, "output shape must be the shard shape without axis 0");
  const int R = c->nranks;
  const int64_t nout = numel_of(out->shape, out->ndim);
  const size_t rec = op == kAxis0Sum ? (dt == TRS_I32 ? 4 : 8) : max_record_size(dt);
  // the same choice on every rank (it depends on the output's shape only)
  const bool peers = c->xpeers != nullptr && (size_t)nout * rec <= kAxis0Arena;
  int64_t base = 0;
  int first_rank = 0;
  if (op != kAxis0Sum) {
    // every rank's row count: the global index offset of this shard, the
    // lowest rank holding rows, and the empty-axis check of max/argmax (a sum
    // needs none of them)
    Nccl& n = nccl();
    Scratch counts;
    e = counts.alloc(sizeof(int64_t) * (R + 1), stream);
    if (!e.ok()) return e;
    int64_t* cnt = counts.as<int64_t>();
    const int64_t mine = shard->shape[0];
    cudaError_t ce = cudaMemcpyAsync(cnt + R, &mine, sizeof(int64_t), cudaMemcpyHostToDevice, stream);
    if (ce != cudaSuccess) return cuda_error(ce, "cudaMemcpyAsync");
    e = nccl_call(c, n.AllGather(cnt + R, cnt, 1, ncclInt64, c->comm, stream), "ncclAllGather (row counts)");
    if (!e.ok()) return e;
    std::vector<int64_t> all(R);
    ce = cudaMemcpyAsync(all.data(), cnt, sizeof(int64_t) * R, cudaMemcpyDeviceToHost, stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(stream);
    if (ce != cudaSuccess) return cuda_error(ce, "reading the row counts");
    int64_t total = 0;
    first_rank = -1;
    for (int r = 0; r < R; ++r) {
      if (r < c->rank) base += all[r];
      if (first_rank < 0 && all[r] > 0) first_rank = r;
      total += all[r];
    }
    if (op != kAxis0Sum && total == 0) return make_error(TRS_ERR_EMPTY_AXIS, "!!!Cannot reduce an empty axis!!!");
  }
  if (nout == 0) return Error{};
  if (peers) return axis0_combine_peers(c, op, shard, out, base, first_rank, nout, stream);
  return axis0_combine_nccl(c, op, shard, out, base, first_rank, nout, stream);
}

}  // namespace

extern "C" {

trs_status trs_comm_unique_id(uint8_t id[128]) {
  Nccl& n = nccl();
  if (!n.loaded) return finish(make_error(TRS_ERR_UNAVAILABLE, n.why));
  ncclUniqueId u;
  ncclResult_t r = n.GetUniqueId(&u);
  if (r != ncclSuccess) return finish(nccl_error(r, "ncclGetUniqueId"));
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id, &u, 128);
  return TRS_OK;
}

trs_status trs_comm_init_rank(const uint8_t id[128], int32_t nranks, int32_t rank, int32_t timeout_ms,
                              trs_comm** comm) {
  if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks || timeout_ms <= 0)
    return finish(make_error(TRS_ERR_ARG, "bad communicator arguments"));
  Nccl& n = nccl();
  if (!n.loaded) return finish(make_error(TRS_ERR_UNAVAILABLE, n.why));
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  trs_comm* c = new trs_comm;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return finish(nccl_error(r, "ncclCommInitRankConfig"));
  }
  Error e = wait_ready(c, "ncclCommInitRankConfig");
  if (e.ok()) e = setup_exchange(c);
  if (!e.ok()) {
    teardown_exchange(c);
    n.CommAbort(c->comm);
    delete c;
    return finish(e);
  }
  *comm = c;
  return TRS_OK;
}

trs_status trs_comm_destroy(trs_comm* comm) {
  if (!comm) return TRS_OK;
  Nccl& n = nccl();
  teardown_exchange(comm);
  ncclResult_t r = n.CommDestroy(comm->comm);
  delete comm;
  if (r != ncclSuccess && r != ncclInProgress) return finish(nccl_error(r, "ncclCommDestroy"));
  return TRS_OK;
}

trs_status trs_comm_abort(trs_comm* comm) {
  if (!comm) return TRS_OK;
  Nccl& n = nccl();
  teardown_exchange(comm);
  ncclResult_t r = n.CommAbort(comm->comm);
  delete comm;
  if (r != ncclSuccess) return finish(nccl_error(r, "ncclCommAbort"));
  return TRS_OK;
}

trs_status trs_comm_peer_exchange(const trs_comm* comm, int32_t* active) {
  if (!comm || !active) return finish(make_error(TRS_ERR_ARG, "null argument"));
  *active = comm->xpeers ? 1 : 0;
  return TRS_OK;
}

trs_status trs_sharded_sum(trs_comm* comm, const trs_view* shard, trs_view* out, trs_stream stream) {
  if (!shard || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  trs_ew_program p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = 1;
  return finish(sharded_sum(comm, p, shard, nullptr, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_sharded_elementwise_sum(trs_comm* comm, const trs_ew_program* prog, const trs_view* in,
                                       trs_view* out, trs_view* sum_out, trs_stream stream) {
  if (!prog || !in || !sum_out) return finish(make_error(TRS_ERR_ARG, "null argument"));
  return finish(sharded_sum(comm, *prog, in, out, sum_out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_sharded_sum_axis0(trs_comm* comm, const trs_view* shard, trs_view* out, trs_stream stream) {
  if (!shard || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(sharded_axis0(comm, kAxis0Sum, shard, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_sharded_max_axis0(trs_comm* comm, const trs_view* shard, trs_view* out, trs_stream stream) {
  if (!shard || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(sharded_axis0(comm, kAxis0Max, shard, out, static_cast<cudaStream_t>(stream)));
}

trs_status trs_sharded_argmax_axis0(trs_comm* comm, const trs_view* shard, trs_view* out, trs_stream stream) {
  if (!shard || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  return finish(sharded_axis0(comm, kAxis0Argmax, shard, out, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
