// Shape dispatch and C-ABI entry points of the frame kernels.
#include "gfst_common.cuh"
#include "frame_qr_launch.h"

namespace gfst {

// ---------------------------------------------------------------------------
// shape dispatch
// ---------------------------------------------------------------------------
struct Shape {
  int dmax, rmax;
};

// Capacity classes (rows x columns), smallest first.  A frame runs in the
// first class with dmax >= d and rmax >= r.  Each class fixes the lane grid
// (row groups x column groups) in GFST_SHAPE_CASES below.
constexpr Shape kShapes[] = {
    {8, 8},   {32, 8},   {64, 8},   {128, 8},   {256, 8},
    {16, 16}, {32, 16},  {64, 16},  {128, 16},  {256, 16},
    {32, 32}, {64, 32},  {128, 32},
};

int pick_shape(int d, int r) {
  const int rcap = r <= 8 ? 8 : (r <= 16 ? 16 : 32);
  for (int i = 0; i < (int)(sizeof(kShapes) / sizeof(kShapes[0])); ++i) {
    if (kShapes[i].rmax == rcap && kShapes[i].dmax >= d) return i;
  }
  return -1;
}

int check_frame_args(int64_t n, int d, int r, int m, int sign_mode) {
  GFST_REQUIRE(n >= 0, GFST_ERR_ARG, "n_frames must be >= 0 (got %lld)", (long long)n);
  GFST_REQUIRE(r >= 1 && r <= d, GFST_ERR_SHAPE, "need 1 <= r <= d (d=%d r=%d)", d, r);
  GFST_REQUIRE(r <= 32, GFST_ERR_SHAPE, "r=%d exceeds 32", r);
  GFST_REQUIRE(pick_shape(d, r) >= 0, GFST_ERR_SHAPE, "d=%d r=%d outside the supported classes", d, r);
  GFST_REQUIRE(m >= 0 && m <= kMaxRank, GFST_ERR_SHAPE, "update rank m=%d outside [0, %d]", m, kMaxRank);
  GFST_REQUIRE(sign_mode == GFST_SIGN_FIRST_SIGNIFICANT || sign_mode == GFST_SIGN_R_DIAG_POSITIVE, GFST_ERR_ARG,
               "unknown sign_mode %d", sign_mode);
  return GFST_OK;
}

}  // namespace gfst

extern "C" int gfst_frame_update_qr(const float* U, const float* A, const float* B, float beta, float* Uout,
                                    int64_t n_frames, int d, int r, int m, float eps_sign, int sign_mode,
                                    cudaStream_t stream) {
  using namespace gfst;
  int st = check_frame_args(n_frames, d, r, m, sign_mode);
  if (st != GFST_OK) return st;
  if (n_frames == 0) return GFST_OK;
  GFST_REQUIRE(U != nullptr && Uout != nullptr, GFST_ERR_ARG, "U and Uout must be non-null");
  GFST_REQUIRE(m == 0 || (A != nullptr && B != nullptr), GFST_ERR_ARG, "A and B must be non-null when m > 0");
  switch (pick_shape(d, r)) {
#define X(idx, D, R, RG, CG) \
  case idx:                  \
    return launch_update<D, R, RG, CG>(U, A, B, beta, Uout, n_frames, d, r, m, eps_sign, sign_mode, stream);
    GFST_SHAPE_CASES(X)
#undef X
    default:
      break;
  }
  set_last_error("no kernel for d=%d r=%d", d, r);
  return GFST_ERR_SHAPE;
}

extern "C" int gfst_frame_stream_ex(float* U, const float* A, const float* B, float beta, int64_t n_frames, int T,
                                    int d, int r, int m, float eps_sign, int sign_mode, float* frames_out,
                                    int out_every, int qr_method, cudaStream_t stream) {
  using namespace gfst;
  int st = check_frame_args(n_frames, d, r, m, sign_mode);
  if (st != GFST_OK) return st;
  GFST_REQUIRE(qr_method == GFST_QR_AUTO || qr_method == GFST_QR_HOUSEHOLDER || qr_method == GFST_QR_CHOLESKY2 ||
                   qr_method == GFST_QR_CHOLESKY2_SPLIT,
               GFST_ERR_ARG, "unknown qr_method %d", qr_method);
  GFST_REQUIRE(T >= 0, GFST_ERR_ARG, "T must be >= 0 (got %d)", T);
  GFST_REQUIRE(m >= 1, GFST_ERR_SHAPE, "streaming needs an update rank m >= 1");
  if (n_frames == 0 || T == 0) return GFST_OK;
  GFST_REQUIRE(U != nullptr && A != nullptr && B != nullptr, GFST_ERR_ARG, "U, A and B must be non-null");
  GFST_REQUIRE(frames_out == nullptr || out_every > 0, GFST_ERR_ARG, "out_every must be > 0 with frames_out");
  GFST_REQUIRE((d * m) % 4 == 0 && (r * m) % 4 == 0, GFST_ERR_ALIGN,
               "streaming needs d*m and r*m to be multiples of 4 (d=%d r=%d m=%d)", d, r, m);
  GFST_REQUIRE(aligned16(A) && aligned16(B), GFST_ERR_ALIGN, "A and B must be 16-byte aligned");
  switch (pick_shape(d, r)) {
#define X(idx, D, R, RG, CG)                                                                                \
  case idx:                                                                                                 \
    return launch_stream<D, R, RG, CG>(U, A, B, beta, n_frames, T, d, r, m, eps_sign, sign_mode, frames_out, \
                                    out_every, qr_method, stream);
    GFST_SHAPE_CASES(X)
#undef X
    default:
      break;
  }
  set_last_error("no kernel for d=%d r=%d", d, r);
  return GFST_ERR_SHAPE;
}

extern "C" int gfst_frame_stream(float* U, const float* A, const float* B, float beta, int64_t n_frames, int T,
                                 int d, int r, int m, float eps_sign, int sign_mode, float* frames_out,
                                 int out_every, cudaStream_t stream) {
  return gfst_frame_stream_ex(U, A, B, beta, n_frames, T, d, r, m, eps_sign, sign_mode, frames_out, out_every,
                              GFST_QR_AUTO, stream);
}
