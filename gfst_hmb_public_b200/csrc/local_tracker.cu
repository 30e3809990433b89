// C-ABI entry of the per-token local tracker (largest flag basis, nested flag
// levels, alignment features).
#include "frame_qr_launch.h"
#include "local_tracker.cuh"

namespace gfst {

template <int DMAX, int RMAX, int RG, int CG>
int launch_tracker_dispatch(float* U, float* nested, const float* X, int64_t n, int T, int d, int r,
                            const TrackerParams& prm, float* features, float* proj_sum, float* red_sum,
                            cudaStream_t stream);

}  // namespace gfst

extern "C" int gfst_local_tracker_stream(float* U, float* nested, const float* x, int64_t n_streams, int T, int d,
                                         int r, int n_levels, const int32_t* dims, const double* rates, double eps,
                                         double eps_update, float eps_sign, int sign_mode, float* features,
                                         cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && T >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(r >= 1 && r <= d && r <= 32, GFST_ERR_SHAPE, "need 1 <= r <= min(d, 32) (d=%d r=%d)", d, r);
  GFST_REQUIRE(pick_shape(d, r) >= 0, GFST_ERR_SHAPE, "d=%d r=%d outside the supported classes", d, r);
  GFST_REQUIRE(d % 4 == 0, GFST_ERR_ALIGN, "d=%d must be a multiple of 4", d);
  GFST_REQUIRE(n_levels >= 0 && n_levels <= kMaxTrackerLevels, GFST_ERR_SHAPE, "n_levels=%d outside [0, %d]",
               n_levels, kMaxTrackerLevels);
  GFST_REQUIRE(n_levels == 0 || dims != nullptr, GFST_ERR_ARG, "dims must be given");
  GFST_REQUIRE(rates != nullptr, GFST_ERR_ARG, "rates must be given");
  GFST_REQUIRE(sign_mode == GFST_SIGN_FIRST_SIGNIFICANT || sign_mode == GFST_SIGN_R_DIAG_POSITIVE, GFST_ERR_ARG,
               "unknown sign_mode %d", sign_mode);
  TrackerParams prm{};
  prm.n_levels = n_levels;
  int off = 0;
  for (int l = 0; l < n_levels; ++l) {
    GFST_REQUIRE(dims[l] >= 1 && dims[l] < r && (l == 0 || dims[l] > dims[l - 1]), GFST_ERR_SHAPE,
                 "nested dims must increase strictly inside [1, r) (level %d: %d)", l, dims[l]);
    prm.dims[l] = dims[l];
    prm.voff[l] = off;
    off += r * dims[l];
  }
  for (int l = 0; l <= n_levels; ++l) {
    GFST_REQUIRE(rates[l] >= 0.0 && rates[l] <= 1.0, GFST_ERR_ARG, "rate %d outside [0, 1]", l);
    prm.rate[l] = (float)rates[l];
    prm.one_minus[l] = (float)(1.0 - rates[l]);
  }
  prm.eps = (float)eps;
  prm.eps_update_sq = (float)(eps_update * eps_update);
  prm.eps_sign = eps_sign;
  prm.sign_mode = sign_mode;
  if (n_streams == 0 || T == 0) return GFST_OK;
  GFST_REQUIRE(U && x && (n_levels == 0 || nested), GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(aligned16(x), GFST_ERR_ALIGN, "x must be 16-byte aligned");
  switch (pick_shape(d, r)) {
#define X(idx, D, R, RG, CG) \
  case idx:                  \
    return launch_tracker_dispatch<D, R, RG, CG>(U, nested, x, n_streams, T, d, r, prm, features, nullptr, nullptr, \
                                                 stream);
    GFST_SHAPE_CASES(X)
#undef X
    default:
      break;
  }
  set_last_error("no kernel for d=%d r=%d", d, r);
  return GFST_ERR_SHAPE;
}

extern "C" int gfst_block_tracker_stream(float* U, float* projector_sum, float* reduced_sum, const float* x,
                                         int64_t n_streams, int T, int d, int r, double rate, double eps_update,
                                         float eps_sign, int sign_mode, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && T >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(r >= 1 && r <= d && r <= 32 && r % 4 == 0, GFST_ERR_SHAPE,
               "need r in [1, min(d, 32)], r %% 4 == 0 (d=%d r=%d)", d, r);
  GFST_REQUIRE(d <= 64 && d % 4 == 0, GFST_ERR_SHAPE, "block tracker needs d <= 64, d %% 4 == 0 (d=%d)", d);
  GFST_REQUIRE(pick_shape(d, r) >= 0, GFST_ERR_SHAPE, "d=%d r=%d outside the supported classes", d, r);
  GFST_REQUIRE(rate >= 0.0 && rate <= 1.0, GFST_ERR_ARG, "rate outside [0, 1]");
  GFST_REQUIRE(sign_mode == GFST_SIGN_FIRST_SIGNIFICANT || sign_mode == GFST_SIGN_R_DIAG_POSITIVE, GFST_ERR_ARG,
               "unknown sign_mode %d", sign_mode);
  if (n_streams == 0 || T == 0) return GFST_OK;
  GFST_REQUIRE(U && projector_sum && reduced_sum && x, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(aligned16(x), GFST_ERR_ALIGN, "x must be 16-byte aligned");
  TrackerParams prm{};
  prm.n_levels = 0;
  prm.rate[0] = (float)rate;
  prm.one_minus[0] = (float)(1.0 - rate);
  prm.eps = 1e-6f;  // features are not produced
  prm.eps_update_sq = (float)(eps_update * eps_update);
  prm.eps_sign = eps_sign;
  prm.sign_mode = sign_mode;
  switch (pick_shape(d, r)) {
#define X(idx, D, R, RG, CG)                                                                                      \
  case idx:                                                                                                       \
    return launch_tracker_dispatch<D, R, RG, CG>(U, nullptr, x, n_streams, T, d, r, prm, nullptr, projector_sum, \
                                                 reduced_sum, stream);
    GFST_SHAPE_CASES(X)
#undef X
    default:
      break;
  }
  set_last_error("no kernel for d=%d r=%d", d, r);
  return GFST_ERR_SHAPE;
}
