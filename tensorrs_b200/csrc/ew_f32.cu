// ew_f32.cu -- element-wise kernels instantiated for float.
#include "ew_kernels.cuh"

namespace trs {
template Error ew_launch<float>(const trs_ew_program&, const trs_view*, const trs_view*,
                              const SumTarget*, const EwPrepared&, cudaStream_t);
}  // namespace trs
