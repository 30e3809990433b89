// CholeskyQR2 of narrow frames (r <= 8 columns) in the lane layout of the
// Householder kernel FrameQR<DMAX, 8, RG, 1>: a frame is RG consecutive lanes,
// lane t owns rows t, t + RG, t + 2 RG, ... of all 8 columns (float2 row
// pairs), so 32 / RG frames share a warp.
//
// Why: a Householder QR of a 64 x 8 frame is 16 dependent reflector steps,
// each a column norm and up to 8 dot products reduced across the frame's
// lanes; the batched one-QR-per-frame launch is then issue-bound (about twice
// the time its 4 KB of HBM traffic per frame needs).  CholeskyQR2 replaces the
// reflectors by two passes of
//     G = C^T C  (36 independent dot products, one butterfly reduction),
//     G = R^T R  (an 8 x 8 Cholesky, computed redundantly by every lane of
//                 the frame, so no broadcast is needed),
//     C <- C R^{-1}  (right-looking, each lane on its own rows),
// a fifth of the instructions.  The second pass runs on the nearly
// orthonormal result of the first and sets the final factor: the thin Q of
// the input with a positive R diagonal, the matrix Householder QR with the
// R-diagonal-positive rule produces (the factorisation is unique for a
// full-rank input).  Cholesky's backward error is componentwise in the
// column scaling, so frames whose columns differ in scale by 1e3 or more
// (the batched-QR workload scales column j by 10^(-j/2)) factor as accurately
// as equilibrated ones.
//
// The pivot test of FrameChol applies: a pivot R_jj^2 below kPivotTol * G_jj
// (column j within about 6 degrees of the span of the columns before it), a
// non-finite pivot or a zero column sends the whole warp through Householder
// on its current pass input (the second pass's input has the same Q as the
// original), so the near-collinear and rank-deficient frames take exactly the
// path they took before.
#pragma once

#include "frame_chol.cuh"
#include "frame_qr.cuh"

namespace gfst {

template <int DMAX, int RG>
struct FrameCholSmall {
  static constexpr int RMAX = 8;
  using QR = FrameQR<DMAX, RMAX, RG, 1>;
  using Frame = typename QR::Frame;  // a[p][c] = rows (t + 2p RG, t + (2p + 1) RG) of column c
  static constexpr int RP = QR::RP;
  static_assert(QR::CPT == RMAX, "one column group: every lane holds all columns");

  // Upper triangle of G = C^T C, summed over the frame's RG lanes.  The xor
  // butterfly gives every lane of the frame the same bits (each level adds
  // the same two partial sums, in either order).
  __device__ static __forceinline__ void gram(const Frame& a, float (&g)[RMAX][RMAX]) {
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
#pragma unroll
      for (int j = i; j < RMAX; ++j) {
        float2 acc = __fmul2_rn(a[0][i], a[0][j]);
#pragma unroll
        for (int p = 1; p < RP; ++p) acc = ffma2(a[p][i], a[p][j], acc);
        g[i][j] = acc.x + acc.y;
      }
    }
#pragma unroll
    for (int off = 1; off < RG; off <<= 1) {
#pragma unroll
      for (int i = 0; i < RMAX; ++i)
#pragma unroll
        for (int j = i; j < RMAX; ++j) g[i][j] += __shfl_xor_sync(0xffffffffu, g[i][j], off);
    }
  }

  // In place: g (upper triangle) <- R with R[k][k] replaced by 1 / R[k][k].
  // Columns >= r are zero padding: they get a unit diagonal (R = I there).
  // Returns this lane's pivot test over the real columns.
  __device__ static __forceinline__ bool cholesky(float (&g)[RMAX][RMAX], int r) {
    float dg[RMAX];
#pragma unroll
    for (int j = 0; j < RMAX; ++j) {
      if (j >= r) g[j][j] = 1.f;
      dg[j] = g[j][j];
    }
    bool ok = true;
#pragma unroll
    for (int k = 0; k < RMAX; ++k) {
      const float piv = g[k][k];
      // NaN fails every comparison; an infinite Gram gives a NaN or infinite pivot
      if (k < r) ok = ok && dg[k] > 0.f && piv > kPivotTol * dg[k] && piv <= 3.0e38f;
      // the second pass's R is I + O(1e-6): an rsqrt within a few ulp moves a
      // column's norm by a few 1e-7, far inside the orthogonality bar
      const float inv = rsqrtf(piv);
      g[k][k] = inv;
#pragma unroll
      for (int j = k + 1; j < RMAX; ++j) g[k][j] *= inv;
#pragma unroll
      for (int i = k + 1; i < RMAX; ++i)
#pragma unroll
        for (int j = i; j < RMAX; ++j) g[i][j] = fmaf(-g[k][i], g[k][j], g[i][j]);
    }
    return ok;
  }

  // a <- a R^{-1}, right-looking: column i is finished (times 1/R[i][i]), then
  // removed from every later column.
  // The column loop is a static_for: as a plain unrolled loop its triangular
  // inner loop kept a dynamic index and the frame went to local memory.
  __device__ static __forceinline__ void solve(Frame& a, const float (&g)[RMAX][RMAX]) {
    static_for<0, RMAX>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      const float2 s = make_float2(g[i][i], g[i][i]);
#pragma unroll
      for (int p = 0; p < RP; ++p) a[p][i] = __fmul2_rn(a[p][i], s);
#pragma unroll
      for (int j = i + 1; j < RMAX; ++j) {
        const float2 nr = make_float2(-g[i][j], -g[i][j]);
#pragma unroll
        for (int p = 0; p < RP; ++p) a[p][j] = ffma2(a[p][i], nr, a[p][j]);
      }
    });
  }

  // One pass; false (a unchanged) when a frame of the warp fails the pivot
  // test.  `valid` is false for the padding frames of the last warp (all
  // zero), which must not send their warp to Householder.
  __device__ static __forceinline__ bool pass(Frame& a, int r, bool valid) {
    float g[RMAX][RMAX];
    gram(a, g);
    const bool ok = cholesky(g, r) || !valid;
    if (!__all_sync(0xffffffffu, ok)) return false;
    solve(a, g);
    return true;
  }

  // In place: a <- sign-fixed thin Q.
  __device__ static __forceinline__ void qr(Frame& a, int lane, int t, typename QR::Smem& sm, float eps_sign,
                                            int sign_mode, int r, bool valid) {
    // the two passes run as one rolled loop (the unrolled pass code is large
    // enough to thrash the instruction cache), and the fallback is called once,
    // after it, so that the frame stays in registers through the passes
    bool done = true;
#pragma unroll 1
    for (int ps = 0; ps < 2 && done; ++ps) done = pass(a, r, valid);
    if (!done) {
      QR::qr(a, lane, t, sm, eps_sign, sign_mode, r);
      return;
    }
    // R = R2 R1 has a positive diagonal: the R-diagonal rule needs no flips
    if (sign_mode == GFST_SIGN_FIRST_SIGNIFICANT) {
      const uint32_t mask = r >= 32 ? 0xffffffffu : ((1u << r) - 1u);
      const uint32_t flip = QR::first_significant_flips(a, lane, 0, eps_sign, mask & 0xffu);
#pragma unroll
      for (int p = 0; p < RP; ++p)
#pragma unroll
        for (int c = 0; c < RMAX; ++c)
          if ((flip >> c) & 1u) a[p][c] = make_float2(-a[p][c].x, -a[p][c].y);
    }
  }
};

}  // namespace gfst
