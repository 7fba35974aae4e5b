// ew_i32.cu -- element-wise kernels instantiated for int32_t.
#include "ew_kernels.cuh"

namespace trs {
template Error ew_launch<int32_t>(const trs_ew_program&, const trs_view*, const trs_view*,
                              const SumTarget*, const EwPrepared&, cudaStream_t);
}  // namespace trs
