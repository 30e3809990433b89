// Host-side declarations of the frame-kernel launchers.  Each capacity class
// (DMAX, RMAX, RG, CG) is explicitly instantiated in one of frame_qr_r{8,16,32}.cu
// so the classes compile in parallel.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gfst {

constexpr int kMaxRank = 8;  // largest update rank m

template <int DMAX, int RMAX, int RG, int CG>
int launch_update(const float* U, const float* A, const float* B, float beta, float* Uout, int64_t n, int d, int r,
                  int m, float eps_sign, int sign_mode, cudaStream_t stream);

// qr_method: GFST_QR_AUTO (CholeskyQR2 where the class has it, else
// Householder), GFST_QR_HOUSEHOLDER, GFST_QR_CHOLESKY2 or
// GFST_QR_CHOLESKY2_SPLIT (classes with 8 < r <= 32 only).
template <int DMAX, int RMAX, int RG, int CG>
int launch_stream(float* U, const float* A, const float* B, float beta, int64_t n, int T, int d, int r, int m,
                  float eps_sign, int sign_mode, float* frames_out, int out_every, int qr_method,
                  cudaStream_t stream);

// Capacity class index for (d, r): the first class with dmax >= d and the
// column capacity of r; -1 if none (frame_qr.cu).
int pick_shape(int d, int r);

// (index, DMAX, RMAX, RG, CG): RG row groups x CG column groups of lanes per frame
#define GFST_SHAPE_CASES(X) \
  X(0, 8, 8, 4, 2)          \
  X(1, 32, 8, 8, 1)         \
  X(2, 64, 8, 8, 1)         \
  X(3, 128, 8, 16, 1)       \
  X(4, 256, 8, 32, 1)       \
  X(5, 16, 16, 8, 2)        \
  X(6, 32, 16, 8, 2)        \
  X(7, 64, 16, 8, 4)        \
  X(8, 128, 16, 8, 4)       \
  X(9, 256, 16, 16, 2)      \
  X(10, 32, 32, 8, 4)       \
  X(11, 64, 32, 8, 4)       \
  X(12, 128, 32, 8, 4)

}  // namespace gfst
