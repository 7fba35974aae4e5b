// reduce_i64.cu -- reduction kernels instantiated for int64_t.
#include "reduce_kernels.cuh"

namespace trs {
template Error red_launch<int64_t>(RedDev&, const RedChoice&, cudaStream_t);
template bool red_stream_available<int64_t>(int, int);
template bool red_cstream_available<int64_t>(int, int);
}  // namespace trs
