// Instantiations of the frame kernels for the r <= 16 capacity classes.
#include "frame_qr_kernels.cuh"

namespace gfst {

template int launch_update<16, 16, 8, 2>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<16, 16, 8, 2>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<32, 16, 8, 2>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<32, 16, 8, 2>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<64, 16, 8, 4>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<64, 16, 8, 4>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<128, 16, 8, 4>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<128, 16, 8, 4>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<256, 16, 16, 2>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<256, 16, 16, 2>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);

}  // namespace gfst
