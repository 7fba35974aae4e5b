// ew_f64.cu -- element-wise kernels instantiated for double.
#include "ew_kernels.cuh"

namespace trs {
template Error ew_launch<double>(const trs_ew_program&, const trs_view*, const trs_view*,
                              const SumTarget*, const EwPrepared&, cudaStream_t);
}  // namespace trs
