// reduce_f64.cu -- reduction kernels instantiated for double.
#include "reduce_kernels.cuh"

namespace trs {
template Error red_launch<double>(RedDev&, const RedChoice&, cudaStream_t);
}  // namespace trs
