// reduce_f64.cu -- reduction kernels instantiated for double.
#include "reduce_kernels.cuh"

namespace trs {
template Error red_launch<double>(RedDev&, const RedChoice&, cudaStream_t);
template bool red_stream_available<double>(int, int);
template bool red_cstream_available<double>(int, int);
}  // namespace trs
