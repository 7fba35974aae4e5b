// tma.cuh -- tensor-map (TMA) copies: the driver's cuTensorMapEncodeTiled,
// looked up once through the runtime, and the tiled global->shared loads.
//
// Every load completes on an mbarrier of the issuing CTA (bulk.cuh), lands in
// that CTA's own shared memory, reads this GPU's own global memory, and uses
// no cluster multicast.  A box's innermost start coordinate times the element
// size is always a multiple of 16 bytes; the other coordinates may lie
// outside the tensor, where the box reads zeros.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "bulk.cuh"
#include "kernels.cuh"

namespace trs {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's encoder, or nullptr with *err set when the driver has none.
inline EncodeTiled encode_fn(Error* err) {
  static std::once_flag once;
  static EncodeTiled fn = nullptr;
  static std::string why;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
    else
      why = "cuTensorMapEncodeTiled is not available from the driver";
    cudaGetLastError();
  });
  if (!fn) *err = make_error(TRS_ERR_UNAVAILABLE, why);
  return fn;
}

template <class T> constexpr CUtensorMapDataType tma_dtype();
template <> constexpr CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <> constexpr CUtensorMapDataType tma_dtype<double>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT64; }
template <> constexpr CUtensorMapDataType tma_dtype<int32_t>() { return CU_TENSOR_MAP_DATA_TYPE_INT32; }
template <> constexpr CUtensorMapDataType tma_dtype<int64_t>() { return CU_TENSOR_MAP_DATA_TYPE_INT64; }

// A 4-D tensor map over `base` (extents innermost first, byte strides of the
// outer three), boxes `box`, zeros outside.
template <class T>
inline Error make_map_4d(const char* fn, const void* base, const cuuint64_t (&dims)[4], const cuuint64_t (&strides)[3],
                  const cuuint32_t (&box)[4], CUtensorMap* map) {
  Error e;
  EncodeTiled enc = encode_fn(&e);
  if (!enc) return e;
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, tma_dtype<T>(), 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return make_error(TRS_ERR_CUDA, std::string(fn) + ": cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return Error{};
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace trs
