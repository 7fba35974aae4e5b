// reduce_f32.cu -- reduction kernels instantiated for float.
#include "reduce_kernels.cuh"

namespace trs {
template Error red_launch<float>(RedDev&, const RedChoice&, cudaStream_t);
template bool red_stream_available<float>(int, int);
template bool red_cstream_available<float>(int, int);
}  // namespace trs
