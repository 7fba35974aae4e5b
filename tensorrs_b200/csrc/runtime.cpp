// runtime.cpp -- see runtime.h.
#include "runtime.h"

#include <mutex>

namespace trs {

std::atomic<uint64_t> g_launch_count{0};
std::atomic<uint64_t> g_scratch_alloc_count{0};

namespace {
thread_local std::string t_last_error;
}

void set_last_error(const std::string& msg) { t_last_error = msg; }
const std::string& last_error() { return t_last_error; }

Error cuda_error(cudaError_t e, const char* what) {
  return make_error(TRS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + ": " +
                                      cudaGetErrorString(e));
}

const DeviceInfo& current_device_info() {
  static DeviceInfo infos[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    static DeviceInfo fallback;
    return fallback;
  }
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = infos[dev];
  if (d.device != dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) d.sm_count = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
      d.max_smem_optin = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrClusterLaunch, dev) == cudaSuccess) d.cluster_launch = v;
    d.device = dev;
  }
  return d;
}

// This library's stream-ordered pool on the current device, created on first
// use with a release threshold that keeps freed blocks cached across
// synchronisations (null if it cannot be created).
static cudaMemPool_t device_pool() {
  static cudaMemPool_t pools[64] = {};
  static bool tried[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!tried[dev]) {
    tried[dev] = true;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    if (cudaMemPoolCreate(&pools[dev], &props) == cudaSuccess) {
      uint64_t keep = ~0ull;
      cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
    } else {
      cudaGetLastError();
      pools[dev] = nullptr;
    }
  }
  return pools[dev];
}

Scratch::~Scratch() {
  if (ptr_) cudaFreeAsync(ptr_, stream_);
}

Error Scratch::alloc(size_t bytes, cudaStream_t stream) {
  stream_ = stream;
  if (bytes == 0) bytes = 16;
  cudaMemPool_t pool = device_pool();
  cudaError_t e = pool ? cudaMallocFromPoolAsync(&ptr_, bytes, pool, stream) : cudaMallocAsync(&ptr_, bytes, stream);
  if (e != cudaSuccess) {
    ptr_ = nullptr;
    cudaGetLastError();
    return make_error(e == cudaErrorMemoryAllocation ? TRS_ERR_OOM : TRS_ERR_CUDA,
                      std::string("scratch allocation of ") + std::to_string(bytes) +
                          " bytes: " + cudaGetErrorString(e));
  }
  g_scratch_alloc_count.fetch_add(1, std::memory_order_relaxed);
  return Error{};
}

}  // namespace trs
