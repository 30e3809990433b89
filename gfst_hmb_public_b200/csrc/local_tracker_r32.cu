// Instantiations of the local-tracker kernel for the r <= 32 capacity classes.
#include "local_tracker.cuh"

namespace gfst {

template <int DMAX, int RMAX, int RG, int CG>
int launch_tracker_dispatch(float* U, float* nested, const float* X, int64_t n, int T, int d, int r,
                            const TrackerParams& prm, float* features, float* proj_sum, float* red_sum,
                            cudaStream_t stream) {
  return launch_tracker<DMAX, RMAX, RG, CG>(U, nested, X, n, T, d, r, prm, features, proj_sum, red_sum, stream);
}

template int launch_tracker_dispatch<32, 32, 8, 4>(float*, float*, const float*, int64_t, int, int, int, const TrackerParams&, float*, float*, float*, cudaStream_t);
template int launch_tracker_dispatch<64, 32, 8, 4>(float*, float*, const float*, int64_t, int, int, int, const TrackerParams&, float*, float*, float*, cudaStream_t);
template int launch_tracker_dispatch<128, 32, 8, 4>(float*, float*, const float*, int64_t, int, int, int, const TrackerParams&, float*, float*, float*, cudaStream_t);

}  // namespace gfst
