// Frame kernels: one-step rank-m update + thin QR, and the T-token streaming
// pass that keeps every frame in registers across tokens.  Templated on the
// capacity class (DMAX, RMAX, RG, CG); the classes are instantiated in
// frame_qr_r8.cu / frame_qr_r16.cu / frame_qr_r32.cu and dispatched in frame_qr.cu.
//
// Reference behaviour (paths relative to pkhairkh/gfst-hmb-public):
//   src/gfst_hmb_mpuc/gfst.py:26-46      canonical_qr_batched + canonicalize_qr_column_signs
//   src/gfst_hmb_mpuc/gfst.py:115-140    update_basis_candidate_batched (beta*U + A B^T form)
//   src/gfst_hmb_mpuc/modeling.py:2299-2423  per-token largest-level tracker update
#pragma once
#include "frame_chol.cuh"
#include "frame_chol_mw.cuh"
#include "frame_chol_small.cuh"
#include "frame_qr.cuh"
#include "frame_qr_launch.h"

namespace gfst {

constexpr int kWarps = 4;  // warps per CTA

// Register budget per capacity class: frames holding >= 128 values per lane get
// the register file share of 2 CTAs per SM (no spills; 8 frames per SM);
// smaller ones pack 4.
template <int DMAX, int RMAX, int RG, int CG>
constexpr int min_blocks() {
  return (DMAX / RG) * (RMAX / CG) >= 128 ? 2 : 4;
}

// Classes whose QR takes CholeskyQR2 in the Householder kernels' lane layout
// (frame_chol_small.cuh, with the Householder code as its fallback): up to 8
// columns, 9 to 128 rows.  The one-step kernel always takes it; the streaming
// kernel unless GFST_QR_HOUSEHOLDER is asked for.
template <int DMAX, int RMAX, int CG>
constexpr bool kCholSmall = RMAX == 8 && CG == 1 && DMAX >= 32 && DMAX <= 128;

// ---------------------------------------------------------------------------
// one step: Uout = QR(beta * U + A B^T)
// ---------------------------------------------------------------------------
template <int DMAX, int RMAX, int RG, int CG, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, (min_blocks<DMAX, RMAX, RG, CG>()))
    frame_update_qr_kernel(const float* __restrict__ U, const float* __restrict__ A, const float* __restrict__ B,
                           float beta, float* __restrict__ Uout, int64_t n_frames, int d, int r, int m,
                           float eps_sign, int sign_mode, bool vec4) {
  using QR = FrameQR<DMAX, RMAX, RG, CG>;
  constexpr int TPF = QR::TPF;
  constexpr int GPW = 32 / TPF;
  __shared__ typename QR::Smem qsm[WARPS * GPW];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = lane % TPF;
  const int g = warp * GPW + lane / TPF;
  const int64_t f = (int64_t)blockIdx.x * (WARPS * GPW) + g;
  const bool valid = f < n_frames;
  const int64_t fs = valid ? f : 0;
  const size_t frame_elems = (size_t)d * r;

  typename QR::Frame a;
  QR::load(a, U + fs * frame_elems, t, d, r, valid, vec4);
  if (beta != 1.f) QR::scale(a, beta);
  if (m > 0 && valid) QR::rank_update(a, A + fs * (size_t)d * m, B + fs * (size_t)r * m, t, d, r, m);
  if constexpr (kCholSmall<DMAX, RMAX, CG>) {
    FrameCholSmall<DMAX, RG>::qr(a, lane, t, qsm[g], eps_sign, sign_mode, r, valid);
  } else {
    QR::qr(a, lane, t, qsm[g], eps_sign, sign_mode, r);
  }
  QR::store(a, Uout + fs * frame_elems, t, d, r, valid, vec4);
}

// ---------------------------------------------------------------------------
// streaming: for t in [0, T): U <- QR(beta * U + A_t B_t^T)
// A_t and B_t are staged per frame group in shared memory with cp.async,
// double-buffered so token t+1's inputs load while token t factorises.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all_but_one() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}

template <int DMAX, int RMAX, int RG, int CG, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, (min_blocks<DMAX, RMAX, RG, CG>()))
    frame_stream_kernel(float* __restrict__ U, const float* __restrict__ A, const float* __restrict__ B, float beta,
                        int64_t n_frames, int T, int d, int r, int m, float eps_sign, int sign_mode,
                        float* __restrict__ frames_out, int out_every, bool vec4, bool chol) {
  using QR = FrameQR<DMAX, RMAX, RG, CG>;
  constexpr int TPF = QR::TPF;
  constexpr int GPW = 32 / TPF;
  __shared__ typename QR::Smem qsm[WARPS * GPW];
  extern __shared__ __align__(16) float stage[];  // [WARPS*GPW][2][d*m + r*m]

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = lane % TPF;
  const int g = warp * GPW + lane / TPF;
  const int64_t f = (int64_t)blockIdx.x * (WARPS * GPW) + g;
  const bool valid = f < n_frames;
  const int64_t fs = valid ? f : 0;
  const size_t frame_elems = (size_t)d * r;
  const int a_elems = d * m, b_elems = r * m;
  const int tok_elems = a_elems + b_elems;  // multiple of 4 (host-checked)
  float* my_stage = stage + (size_t)g * 2 * tok_elems;

  const float* Af = A + fs * (size_t)T * a_elems;
  const float* Bf = B + fs * (size_t)T * b_elems;

  auto issue = [&](int tok) {
    if (valid && tok < T) {
      float* dst = my_stage + (tok & 1) * tok_elems;
      const float* srcA = Af + (size_t)tok * a_elems;
      const float* srcB = Bf + (size_t)tok * b_elems;
      for (int c = t; c < a_elems / 4; c += TPF) cp_async16(dst + 4 * c, srcA + 4 * c);
      for (int c = t; c < b_elems / 4; c += TPF) cp_async16(dst + a_elems + 4 * c, srcB + 4 * c);
    }
    cp_async_commit();
  };

  typename QR::Frame a;
  QR::load(a, U + fs * frame_elems, t, d, r, valid, vec4);

  issue(0);
  for (int tok = 0; tok < T; ++tok) {
    issue(tok + 1);
    cp_async_wait_all_but_one();
    __syncwarp();
    const float* sA = my_stage + (tok & 1) * tok_elems;
    if (beta != 1.f) QR::scale(a, beta);
    if (valid) QR::rank_update(a, sA, sA + a_elems, t, d, r, m);
    if constexpr (kCholSmall<DMAX, RMAX, CG>) {
      if (chol) {
        FrameCholSmall<DMAX, RG>::qr(a, lane, t, qsm[g], eps_sign, sign_mode, r, valid);
      } else {
        QR::qr(a, lane, t, qsm[g], eps_sign, sign_mode, r);
      }
    } else {
      QR::qr(a, lane, t, qsm[g], eps_sign, sign_mode, r);
    }
    if (frames_out != nullptr && ((tok + 1) % out_every) == 0) {
      const int64_t snap = (tok + 1) / out_every - 1;
      QR::store(a, frames_out + (snap * n_frames + fs) * frame_elems, t, d, r, valid, vec4);
    }
    __syncwarp();  // every lane is done with this stage buffer before it is refilled
  }
  QR::store(a, U + fs * frame_elems, t, d, r, valid, vec4);
}

// ---------------------------------------------------------------------------
// streaming with CholeskyQR2 (frame_chol.cuh): one frame per warp in block
// rows, the Gram copy and R in shared memory next to the staged factors.
// ---------------------------------------------------------------------------
template <int DMAX, int RMAX, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 2)
    frame_stream_chol_kernel(float* __restrict__ U, const float* __restrict__ A, const float* __restrict__ B,
                             float beta, int64_t n_frames, int T, int d, int r, int m, float eps_sign, int sign_mode,
                             float* __restrict__ frames_out, int out_every, bool vec4) {
  using CQ = FrameChol<DMAX, RMAX>;
  extern __shared__ __align__(16) unsigned char chol_smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  typename CQ::Smem& sm = reinterpret_cast<typename CQ::Smem*>(chol_smem)[warp];
  const int a_elems = d * m, b_elems = r * m;
  const int tok_elems = a_elems + b_elems;  // multiple of 4 (host-checked)
  float* my_stage = reinterpret_cast<float*>(chol_smem + WARPS * sizeof(typename CQ::Smem)) +
                    (size_t)warp * 2 * tok_elems;

  const int64_t f = (int64_t)blockIdx.x * WARPS + warp;
  const bool valid = f < n_frames;
  const int64_t fs = valid ? f : 0;
  const size_t frame_elems = (size_t)d * r;
  const float* Af = A + fs * (size_t)T * a_elems;
  const float* Bf = B + fs * (size_t)T * b_elems;

  auto issue = [&](int tok) {
    if (valid && tok < T) {
      float* dst = my_stage + (tok & 1) * tok_elems;
      const float* srcA = Af + (size_t)tok * a_elems;
      const float* srcB = Bf + (size_t)tok * b_elems;
      for (int c = lane; c < a_elems / 4; c += 32) cp_async16(dst + 4 * c, srcA + 4 * c);
      for (int c = lane; c < b_elems / 4; c += 32) cp_async16(dst + a_elems + 4 * c, srcB + 4 * c);
    }
    cp_async_commit();
  };

  typename CQ::Frame fr;
  CQ::load(fr, U + fs * frame_elems, lane, d, r, valid, vec4);

  issue(0);
  for (int tok = 0; tok < T; ++tok) {
    issue(tok + 1);
    cp_async_wait_all_but_one();
    __syncwarp();
    const float* sA = my_stage + (tok & 1) * tok_elems;
    if (beta != 1.f) CQ::scale(fr, beta);
    if (valid) CQ::rank_update(fr, sA, sA + a_elems, lane, d, r, m);
    CQ::qr(fr, sm, lane, eps_sign, sign_mode, r);
    if (frames_out != nullptr && ((tok + 1) % out_every) == 0) {
      const int64_t snap = (tok + 1) / out_every - 1;
      CQ::store(fr, frames_out + (snap * n_frames + fs) * frame_elems, lane, d, r, valid, vec4);
    }
    __syncwarp();  // every lane is done with this stage buffer before it is refilled
  }
  CQ::store(fr, U + fs * frame_elems, lane, d, r, valid, vec4);
}

// ---------------------------------------------------------------------------
// streaming with CholeskyQR2, one frame per CTA split over d/32 warps
// (frame_chol_mw.cuh): for batches that leave most SMs idle with one frame
// per warp.  Each warp stages its own 32 rows of A_t and all of B_t.
// ---------------------------------------------------------------------------
template <int DMAX, int RMAX>
__global__ void __launch_bounds__(DMAX, 256 / DMAX)
    frame_stream_chol_mw_kernel(float* __restrict__ U, const float* __restrict__ A, const float* __restrict__ B,
                                float beta, int64_t n_frames, int T, int d, int r, int m, float eps_sign,
                                int sign_mode, float* __restrict__ frames_out, int out_every, bool vec4) {
  using MW = FrameCholMW<DMAX, RMAX>;
  extern __shared__ __align__(16) unsigned char mw_smem[];
  typename MW::Smem& sm = *reinterpret_cast<typename MW::Smem*>(mw_smem);
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int row = 32 * w + lane;
  const int64_t f = blockIdx.x;
  const int a_rows = max(0, min(32, d - 32 * w));
  const int a_elems = a_rows * m, b_elems = r * m;
  const int stage_elems = 32 * m + b_elems;  // a multiple of 4 (r * m is, host-checked)
  float* stage = reinterpret_cast<float*>(mw_smem + sizeof(typename MW::Smem)) + (size_t)w * 2 * stage_elems;
  const size_t frame_elems = (size_t)d * r;
  const float* Af = A + f * (size_t)T * d * m + (size_t)32 * w * m;
  const float* Bf = B + f * (size_t)T * b_elems;

  auto issue = [&](int tok) {
    if (tok < T) {
      float* dst = stage + (tok & 1) * stage_elems;
      const float* srcA = Af + (size_t)tok * d * m;
      const float* srcB = Bf + (size_t)tok * b_elems;
      for (int c = lane; c < a_elems / 4; c += 32) cp_async16(dst + 4 * c, srcA + 4 * c);
      for (int c = lane; c < b_elems / 4; c += 32) cp_async16(dst + 32 * m + 4 * c, srcB + 4 * c);
    }
    cp_async_commit();
  };

  float fr[RMAX];
  MW::load(fr, U + f * frame_elems, row, d, r, vec4);
  issue(0);
  for (int tok = 0; tok < T; ++tok) {
    issue(tok + 1);
    cp_async_wait_all_but_one();
    __syncwarp();
    const float* sA = stage + (tok & 1) * stage_elems;
    if (beta != 1.f) {
#pragma unroll
      for (int c = 0; c < RMAX; ++c) fr[c] *= beta;
    }
    if (row < d) MW::rank_update(fr, sA + lane * m, sA + 32 * m, r, m);
    MW::qr(fr, sm, w, lane, eps_sign, sign_mode, r);
    if (frames_out != nullptr && ((tok + 1) % out_every) == 0) {
      const int64_t snap = (tok + 1) / out_every - 1;
      MW::store(fr, frames_out + (snap * n_frames + f) * frame_elems, row, d, r, vec4);
    }
    __syncwarp();  // every lane is done with this stage buffer before it is refilled
  }
  MW::store(fr, U + f * frame_elems, row, d, r, vec4);
}

// ---------------------------------------------------------------------------
// launchers (host)
// ---------------------------------------------------------------------------

template <int DMAX, int RMAX, int RG, int CG>
int launch_update(const float* U, const float* A, const float* B, float beta, float* Uout, int64_t n, int d, int r,
                  int m, float eps_sign, int sign_mode, cudaStream_t stream) {
  constexpr int GPW = 32 / (RG * CG);
  const int64_t per_block = kWarps * GPW;
  const int64_t blocks = (n + per_block - 1) / per_block;
  GFST_REQUIRE(blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many frames: %lld", (long long)n);
  const bool vec4 = (r % 4 == 0) && aligned16(U) && aligned16(Uout);
  frame_update_qr_kernel<DMAX, RMAX, RG, CG, kWarps><<<(unsigned)blocks, kWarps * 32, 0, stream>>>(
      U, A, B, beta, Uout, n, d, r, m, eps_sign, sign_mode, vec4);
  return check_launch("frame_update_qr_kernel");
}

template <int DMAX, int RMAX>
int launch_stream_chol(float* U, const float* A, const float* B, float beta, int64_t n, int T, int d, int r, int m,
                       float eps_sign, int sign_mode, float* frames_out, int out_every, cudaStream_t stream) {
  using CQ = FrameChol<DMAX, RMAX>;
  const int64_t blocks = (n + kWarps - 1) / kWarps;
  GFST_REQUIRE(blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many frames: %lld", (long long)n);
  const bool vec4 = (r % 4 == 0) && aligned16(U) && (frames_out == nullptr || aligned16(frames_out));
  const size_t smem = kWarps * (sizeof(typename CQ::Smem) + 2 * (size_t)(d * m + r * m) * sizeof(float));
  auto kern = frame_stream_chol_kernel<DMAX, RMAX, kWarps>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)blocks, kWarps * 32, smem, stream>>>(U, A, B, beta, n, T, d, r, m, eps_sign, sign_mode,
                                                         frames_out, out_every, vec4);
  return check_launch("frame_stream_chol_kernel");
}

template <int DMAX, int RMAX>
int launch_stream_chol_mw(float* U, const float* A, const float* B, float beta, int64_t n, int T, int d, int r,
                          int m, float eps_sign, int sign_mode, float* frames_out, int out_every,
                          cudaStream_t stream) {
  using MW = FrameCholMW<DMAX, RMAX>;
  GFST_REQUIRE(n <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many frames: %lld", (long long)n);
  const bool vec4 = (r % 4 == 0) && aligned16(U) && (frames_out == nullptr || aligned16(frames_out));
  const size_t smem = sizeof(typename MW::Smem) + (size_t)MW::W * 2 * (size_t)(32 * m + r * m) * sizeof(float);
  auto kern = frame_stream_chol_mw_kernel<DMAX, RMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)n, DMAX, smem, stream>>>(U, A, B, beta, n, T, d, r, m, eps_sign, sign_mode, frames_out,
                                            out_every, vec4);
  return check_launch("frame_stream_chol_mw_kernel");
}

// The automatic choice splits each frame over d/32 warps while every split
// CTA is resident at once (256 / DMAX CTAs per SM by registers: 2 per SM for
// d = 128, 296 frames on B200): one frame per warp would leave most SMs idle
// and run each frame's dependency chain on one warp.  Measured on B200, 64
// tokens of 128 x 32 frames with rank-4 updates: 256 frames 0.66 ms split
// against 1.00 ms one per warp; past the resident count the split kernel
// needs a second wave (512 frames: 1.40 against 1.07 ms).
inline int64_t split_frames_max(int dmax) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int64_t)(256 / dmax) * sms;
}

template <int DMAX, int RMAX, int RG, int CG>
int launch_stream(float* U, const float* A, const float* B, float beta, int64_t n, int T, int d, int r, int m,
                  float eps_sign, int sign_mode, float* frames_out, int out_every, int qr_method,
                  cudaStream_t stream) {
  constexpr bool kChol = (DMAX == 64 || DMAX == 128) && (RMAX == 16 || RMAX == 32) && RG == 8 && CG == 4;
  if constexpr (kChol) {
    const bool split =
        qr_method == GFST_QR_CHOLESKY2_SPLIT || (qr_method == GFST_QR_AUTO && n <= split_frames_max(DMAX));
    if (split)
      return launch_stream_chol_mw<DMAX, RMAX>(U, A, B, beta, n, T, d, r, m, eps_sign, sign_mode, frames_out,
                                               out_every, stream);
    if (qr_method != GFST_QR_HOUSEHOLDER)
      return launch_stream_chol<DMAX, RMAX>(U, A, B, beta, n, T, d, r, m, eps_sign, sign_mode, frames_out,
                                            out_every, stream);
  } else if constexpr (kCholSmall<DMAX, RMAX, CG>) {
    GFST_REQUIRE(qr_method != GFST_QR_CHOLESKY2_SPLIT, GFST_ERR_SHAPE,
                 "the split CholeskyQR2 kernel covers d in (32, 128] with 8 < r <= 32 (d=%d r=%d)", d, r);
  } else {
    GFST_REQUIRE(qr_method != GFST_QR_CHOLESKY2 && qr_method != GFST_QR_CHOLESKY2_SPLIT, GFST_ERR_SHAPE,
                 "CholeskyQR2 streaming covers d in (8, 128] with r <= 32 (d=%d r=%d)", d, r);
  }
  const bool chol_small = kCholSmall<DMAX, RMAX, CG> && qr_method != GFST_QR_HOUSEHOLDER;
  constexpr int GPW = 32 / (RG * CG);
  const int64_t per_block = kWarps * GPW;
  const int64_t blocks = (n + per_block - 1) / per_block;
  GFST_REQUIRE(blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many frames: %lld", (long long)n);
  const bool vec4 = (r % 4 == 0) && aligned16(U) && (frames_out == nullptr || aligned16(frames_out));
  const size_t smem = (size_t)per_block * 2 * (size_t)(d * m + r * m) * sizeof(float);
  auto kern = frame_stream_kernel<DMAX, RMAX, RG, CG, kWarps>;
  {
    // static scratch + the staged factors can pass 48 KB together: always opt in
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  kern<<<(unsigned)blocks, kWarps * 32, smem, stream>>>(U, A, B, beta, n, T, d, r, m, eps_sign, sign_mode,
                                                         frames_out, out_every, vec4, chol_small);
  return check_launch("frame_stream_kernel");
}

}  // namespace gfst
