// Instantiations of the frame kernels for the r <= 32 capacity classes.
#include "frame_qr_kernels.cuh"

namespace gfst {

template int launch_update<32, 32, 8, 4>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<32, 32, 8, 4>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<64, 32, 8, 4>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<64, 32, 8, 4>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);
template int launch_update<128, 32, 8, 4>(const float*, const float*, const float*, float, float*, int64_t, int, int, int, float, int, cudaStream_t);
template int launch_stream<128, 32, 8, 4>(float*, const float*, const float*, float, int64_t, int, int, int, int, float, int, float*, int, int, cudaStream_t);

}  // namespace gfst
