// kernels.cuh -- launch descriptors and launcher declarations shared by the
// .cu files and the C ABI layer.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "bulk.cuh"
#include "device_ops.cuh"
#include "launch.h"
#include "plan.h"
#include "runtime.h"

namespace trs {

constexpr int kThreads = 256;

// Unsigned 32-bit division by a divisor fixed at launch (the round-up method
// of Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994): q = (umulhi(n, m) + n) >> s.
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
};
FastDiv make_fastdiv(uint32_t d);

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)__umulhi(n, f.m) + n) >> f.s);
}

// Per-kernel launch set-up done once per process: the dynamic shared memory
// a kernel may use (raised only upward), and the CTAs of it an SM keeps
// resident with a given dynamic shared memory (each kernel here has one block
// size), queried once per pair.
inline void allow_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done[kernel] >= bytes) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess)
    done[kernel] = bytes;
  else
    cudaGetLastError();
}

inline int resident_blocks_smem(const void* kernel, int threads, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;  // (kernel, shared bytes)
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(kernel, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, smem) != cudaSuccess || b < 1) {
    cudaGetLastError();
    b = 1;
  }
  cache[key] = b;
  return b;
}

// Element-wise launch descriptor (passed by value as a kernel parameter).
struct EwDev {
  int nd;
  int64_t shape[kMaxDims];
  int64_t st[kMaxOperands][kMaxDims];
  int64_t off[kMaxOperands];
  const void* in[3];
  void* out;
  int64_t n;
  // vector kernel
  int vec;
  uint64_t n_chunks;           // chunks of this launch (< 2^31)
  uint64_t row0;               // first row of this launch
  FastDiv f_cpr;               // chunks per row
  FastDiv f_dim[kMaxDims];     // shape[d] of the outer dimensions
  int stream[3];               // input k is read once: streaming loads
  // bulk-copy stream kernel
  uint64_t n_tiles_s;          // tiles of this launch
  FastDiv f_tpr;               // tiles per row
  int64_t inner;               // row length (innermost folded dimension)
  int bulk_slot[3];            // shared-memory slot of input k, or -1
  int* err;                    // async-error word of this device
  // tile kernel
  int ti;                      // tiled dimension i (unit stride in the transposed inputs)
  int transposed[3];           // input k is read through shared memory
  int tslot[3];                // ew_tr_kernel: shared-memory tile of transposed input k, or -1
  int n_batch;                 // dimensions other than i and j
  int batch_dim[kMaxDims];
  uint64_t tiles_i, tiles_j, n_tiles;
  // ew_tr_kernel: 32-bit tile decode when n_tiles < 2^32 and every batch
  // dimension is below 2^32 (f_dim then holds the batch dimensions' sizes)
  int tile32;
  FastDiv f_tj, f_ti;
};

}  // namespace trs
