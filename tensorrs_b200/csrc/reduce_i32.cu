// reduce_i32.cu -- reduction kernels instantiated for int32_t.
#include "reduce_kernels.cuh"

namespace trs {
template Error red_launch<int32_t>(RedDev&, const RedChoice&, cudaStream_t);
template bool red_stream_available<int32_t>(int, int);
template bool red_cstream_available<int32_t>(int, int);
}  // namespace trs
