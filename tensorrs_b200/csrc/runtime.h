// runtime.h -- host-side CUDA plumbing shared by the launchers: error state,
// the launch counter, per-device properties and stream-ordered scratch.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>

#include "plan.h"

namespace trs {

// Last failure text of the calling thread (trs_last_error).
void set_last_error(const std::string& msg);
const std::string& last_error();

// Kernels launched by this library (trs_launch_count).
extern std::atomic<uint64_t> g_launch_count;
inline void count_launch(uint64_t n = 1) { g_launch_count.fetch_add(n, std::memory_order_relaxed); }

// Successful Scratch::alloc calls (trs_scratch_alloc_count).
extern std::atomic<uint64_t> g_scratch_alloc_count;

Error cuda_error(cudaError_t e, const char* what);

// Checks the launch that was just issued.
inline Error check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return Error{};
}

struct DeviceInfo {
  int device = -1;
  int sm_count = 148;
  int max_smem_optin = 0;
  int cluster_launch = 0;
};
// Properties of the current device (cached per device).
const DeviceInfo& current_device_info();

// Scratch memory from this library's stream-ordered pool on the current
// device (created once per device with a release threshold that keeps freed
// blocks cached across synchronisations), released on the same stream when
// the object goes out of scope (after the work that uses it).
class Scratch {
 public:
  Scratch() = default;
  ~Scratch();
  Error alloc(size_t bytes, cudaStream_t stream);
  void* get() const { return ptr_; }
  template <class P> P* as() const { return static_cast<P*>(ptr_); }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;

 private:
  void* ptr_ = nullptr;
  cudaStream_t stream_ = nullptr;
};

// Address of the current device's async-error word (set by a kernel that gave
// up waiting for its own bulk copies), or null if it cannot be found.
int* async_error_word();

}  // namespace trs
