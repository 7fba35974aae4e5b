// noalloc.cu -- trs_sum_noalloc: sum() whose scratch lives in a static device
// array instead of coming from an allocator.
//
// Some callers cannot allocate device memory while they run: a host that owns
// all device memory through its own arena (and forbids other allocations after
// start-up), or a code path that must not enter the CUDA allocator at all.
// trs_sum needs scratch for its per-block partial sums and takes it from a
// stream-ordered pool; this variant keeps them in g_noalloc_scratch, a
// file-scope device array that every GPU loading the library holds until the
// process exits.  It calls no cudaMalloc, cudaFree or stream-ordered
// allocation.
//
// In host code `g_noalloc_scratch` only names a host-side stand-in for the
// array, not a device address; its device address is looked up once per
// device with cudaGetSymbolAddress (on the first call on that device, with
// that device current) and passed to the kernels.  CUDA loads a library's
// device code lazily, so that first lookup may be what loads this module and
// commits the array's memory: a host that reserves all device memory for its
// own arena makes its first call at start-up, before the reservation (and
// before any stream capture).  Every call shares the one array, so calls that
// overlap on the GPU (on different streams) race on it.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../include/trs.h"
#include "launch.h"
#include "runtime.h"

namespace trs {
namespace {

// Room for 8192 per-block partials of 8 bytes: far more blocks than one
// sum launches on a B200 (at most a few thousand, even for inputs that take
// several launches).
constexpr size_t kNoAllocScratchBytes = 64 * 1024;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.
void* noalloc_scratch(Error* err) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();  // leave no stale error for a later launch check
    *err = cuda_error(e != cudaSuccess ? e : cudaErrorInvalidDevice, "cudaGetDevice");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      *err = cuda_error(e, "cudaGetSymbolAddress of the no-alloc scratch");
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace
}  // namespace trs

extern "C" trs_status trs_sum_noalloc(const trs_view* x, trs_view* out, trs_stream stream) {
  using namespace trs;
  auto finish = [](const Error& e) {
    if (!e.ok()) set_last_error(e.msg);
    return e.status;
  };
  if (!x || !out) return finish(make_error(TRS_ERR_ARG, "null view"));
  Error err;
  void* scratch = noalloc_scratch(&err);
  if (!scratch) return finish(err);
  trs_ew_program p;
  std::memset(&p, 0, sizeof(p));
  p.n_in = 1;
  p.epilogue = TRS_UN_NONE;
  SumTarget t;
  t.view = out;
  t.partials = scratch;
  t.partials_bytes = kNoAllocScratchBytes;
  return finish(run_elementwise(p, x, nullptr, &t, static_cast<cudaStream_t>(stream)));
}
