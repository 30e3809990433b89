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

template <int DMAX, int RMAX, int RG, int CG>
int launch_stream(float* U, const float* A, const float* B, float beta, int64_t n, int T, int d, int r, int m,
                  float eps_sign, int sign_mode, float* frames_out, int out_every, cudaStream_t stream);

}  // namespace gfst
