// Instantiations of the frame kernels for the r <= 8 capacity classes.
#include "frame_qr_kernels.cuh"

namespace gfst {

template int launch_update<8, 8, 4, 2>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<8, 8, 4, 2>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<32, 8, 8, 1>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<32, 8, 8, 1>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<64, 8, 8, 1>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<64, 8, 8, 1>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<128, 8, 16, 1>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<128, 8, 16, 1>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<256, 8, 32, 1>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<256, 8, 32, 1>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);

}  // namespace gfst
