// CholeskyQR2 of one d x r fp32 frame per CTA, split over d/32 warps: the
// streaming pass for batches too small to fill the GPU with one frame per
// warp (frame_chol.cuh).  Same arithmetic as FrameChol -- pass 1: G = C^T C
// (3xTF32 tensor-core products, FP32 sums), G = R^T R, C <- C R^{-1}; pass 2:
// G = C^T C, then the first-order correction C (I - F), or a full Cholesky
// pass when |G - I| > kFirstOrderTol; Householder when a pivot test fails --
// so the result is the same thin Q to FP32 rounding.  What changes is who
// does what:
//
//   * warp w owns rows [32w, 32w + 32) and lane l one row of them, so the
//     rank-m update, the triangular solve and the correction each do a 32nd
//     of a frame's work per lane instead of an 8th, and the per-token
//     dependency chain of a frame shortens by about that much;
//   * each warp forms the Gram of its own 32 rows (its block of the
//     column-major copy stays inside the warp: the chunk swizzle only permutes
//     4-row chunks within a 32-row block), the partial Grams meet in shared
//     memory and every warp adds them in the same fixed order (deterministic);
//   * warp 0 adds the partials and runs the 32-step Cholesky (or takes the
//     first-order correction) while the other warps wait at the barrier that
//     publishes its decision and R; every warp then solves (or corrects) its
//     own rows.  Two CTA barriers per pass (partials written / R published).
// The frame row is not live across the Cholesky (it waits in the shared copy),
// and the Householder fallback keeps its matrix in shared memory (one row per
// thread).  The kernel is compiled for up to 255 registers (two 128-thread
// CTAs per SM): at 128 it spilled to local memory on every token, and the
// split form only runs while all of its CTAs are resident anyway.  Measured on
// B200, 256 frames of 128 x 32 x 64 tokens: 0.66 ms against 0.76 ms at 128
// registers; inside the 256-stream step 0.84 against 1.00 ms per block, since
// two frame CTAs now fill an SM's registers and the readout's CTAs run beside
// fewer of them.
#pragma once

#include "frame_chol.cuh"

namespace gfst {

template <int DMAX, int RMAX>
struct FrameCholMW {
  static_assert(DMAX == 64 || DMAX == 128, "32 rows per warp: 2 or 4 warps per frame");
  static_assert(RMAX == 16 || RMAX == 32, "Gram tiles of FrameChol");
  static constexpr int W = DMAX / 32;   // warps per frame
  static constexpr int GS = RMAX + 4;   // Gram row stride (floats)
  using One = FrameChol<DMAX, RMAX>;    // swizzled layout, TF32 helpers
  using Row = float[RMAX];              // this lane's row of the frame

  struct __align__(16) Smem {
    float mt[RMAX * DMAX];              // column-major, chunk-swizzled copy of the pass input
    float part[W][RMAX * GS];           // warp w's partial Gram
    float area[RMAX * GS];              // warp 0's R rows (or the Gram rows for the correction)
    float red2[W][RMAX];                // Householder fallback: per-warp column sums
    float red[W];                       // Householder fallback: per-warp scalar sums
    float tau[RMAX], beta[RMAX];        // Householder fallback: reflector scales, R diagonal
    uint32_t sign_bits[W][2];           // first-significant search: found / negative bits
    int action;                         // warp 0's decision for the pass (kSolve / kCorrect / kFallback)
  };
  static constexpr int kSolve = 0, kCorrect = 1, kFallback = 2;

  __device__ static __forceinline__ void write_mt(const Row& f, Smem& sm, int row) {
#pragma unroll
    for (int c = 0; c < RMAX; ++c) sm.mt[One::mt_at(c, row)] = f[c];
  }
  __device__ static __forceinline__ void read_mt(Row& f, const Smem& sm, int row) {
#pragma unroll
    for (int c = 0; c < RMAX; ++c) f[c] = sm.mt[One::mt_at(c, row)];
  }

  // Partial Gram of rows [32w, 32w + 32): FrameChol::gram restricted to the
  // warp's four k-steps, stored transposed in part[w] (row j holds G[i][j]
  // for i <= j; entries below the computed tiles are not written).
  __device__ static __forceinline__ void gram_partial(Smem& sm, int w, int lane) {
    constexpr int NQ = RMAX / 8;
    constexpr int NT = RMAX == 32 ? 6 : 2;
    constexpr int MQ[6] = {0, 0, 0, 0, 2, 2}, NQI[6] = {0, 1, 2, 3, 2, 3};
    const int g = lane >> 2, t = lane & 3;
    int off[NQ], swz[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      off[q] = (8 * q + g) * DMAX + t;
      swz[q] = One::sw(8 * q + g);
    }
    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int ks = 4 * w + kk;
      uint32_t h0[NQ], l0[NQ], h1[NQ], l1[NQ];
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        One::split_tf32(sm.mt[off[q] + 4 * ((2 * ks) ^ swz[q])], h0[q], l0[q]);
        One::split_tf32(sm.mt[off[q] + 4 * ((2 * ks + 1) ^ swz[q])], h1[q], l1[q]);
      }
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int a = MQ[i], b = NQI[i];
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        One::mma_tf32(c, l0[a], l0[a + 1], l1[a], l1[a + 1], h0[b], h1[b]);
        One::mma_tf32(c, h0[a], h0[a + 1], h1[a], h1[a + 1], l0[b], l1[b]);
        One::mma_tf32(c, h0[a], h0[a + 1], h1[a], h1[a + 1], h0[b], h1[b]);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] += c[e];
      }
    }
    float* pg = sm.part[w];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int m0 = 8 * MQ[i] + g, n0 = 8 * NQI[i] + 2 * t;
      pg[n0 * GS + m0] = acc[i][0];
      pg[(n0 + 1) * GS + m0] = acc[i][1];
      pg[n0 * GS + m0 + 8] = acc[i][2];
      pg[(n0 + 1) * GS + m0 + 8] = acc[i][3];
    }
  }

  // Row j of the Gram (lane j < RMAX): the warps' partials added in warp
  // order.  Lanes >= RMAX read row 0 (unused).
  __device__ static __forceinline__ void sum_partials(Row& gr, const Smem& sm, int lane) {
    const int row = lane < RMAX ? lane : 0;
#pragma unroll
    for (int q = 0; q < RMAX; q += 4) {
      float4 s = *reinterpret_cast<const float4*>(sm.part[0] + row * GS + q);
#pragma unroll
      for (int w = 1; w < W; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(sm.part[w] + row * GS + q);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      gr[q] = s.x;
      gr[q + 1] = s.y;
      gr[q + 2] = s.z;
      gr[q + 3] = s.w;
    }
  }

  // FrameChol::cholesky on a Gram held in registers (lane j: column j),
  // writing R row k to row k of `area` (1/R[k][k] on the diagonal, -R[k][j]
  // right of it).  Returns this lane's pivot test.
  __device__ static __forceinline__ bool cholesky(Row& g, float* area, int lane, int r) {
    const bool own = lane < RMAX;
    // the diagonal entry g[lane], picked with static indices: a register array
    // indexed by a run-time value would be moved to local memory
    float gjj = 1.f;
#pragma unroll
    for (int i = 0; i < RMAX; ++i)
      if (i == lane) gjj = g[i];
    if (lane >= r) {
#pragma unroll
      for (int i = 0; i < RMAX; ++i) g[i] = (i == lane) ? 1.f : 0.f;
      gjj = 1.f;
    }
    float piv = 1.f, dn = 0.f;
#pragma unroll
    for (int k = 0; k < RMAX; ++k) {
      const float dk = __shfl_sync(0xffffffffu, k == 0 ? g[0] : dn, k);
      const float inv = rsqrtf(dk);
      float rkj = g[k] * inv;
      if (lane == k) piv = dk;
      if (lane < k) rkj = 0.f;
      if (own) area[k * GS + lane] = (lane == k) ? inv : -rkj;
      if (k + 1 < RMAX) {
        dn = fmaf(-rkj, rkj, g[k + 1]);
        const float rn = __shfl_sync(0xffffffffu, rkj, k + 1);
        g[k + 1] = fmaf(-rn, rkj, g[k + 1]);
        __syncwarp();
        const int Q0 = ((k + 2) / 4) * 4;
#pragma unroll
        for (int q = Q0; q < RMAX; q += 4) {
          const float4 v = *reinterpret_cast<const float4*>(area + k * GS + q);  // -R[k][q..q+3]
          if (q + 0 >= k + 2) g[q + 0] = fmaf(v.x, rkj, g[q + 0]);
          if (q + 1 >= k + 2) g[q + 1] = fmaf(v.y, rkj, g[q + 1]);
          if (q + 2 >= k + 2) g[q + 2] = fmaf(v.z, rkj, g[q + 2]);
          if (q + 3 >= k + 2) g[q + 3] = fmaf(v.w, rkj, g[q + 3]);
        }
      }
    }
    return gjj > 0.f && piv > kPivotTol * gjj && piv <= 3.0e38f;
  }

  // f <- f R^{-1} on this lane's row, right-looking; column pairs issue packed FMAs.
  __device__ static __forceinline__ void solve(Row& f, const float* area) {
    static_for<0, RMAX>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      constexpr int Q0 = (i / 4) * 4;
      float rr[RMAX];
#pragma unroll
      for (int q = Q0; q < RMAX; q += 4) {
        const float4 v = *reinterpret_cast<const float4*>(area + i * GS + q);
        rr[q] = v.x;
        rr[q + 1] = v.y;
        rr[q + 2] = v.z;
        rr[q + 3] = v.w;
      }
      f[i] *= rr[i];
      const float fi = f[i];
      constexpr int J0 = i + 1;
      if constexpr (J0 < RMAX && (J0 & 1)) f[J0] = fmaf(fi, rr[J0], f[J0]);
#pragma unroll
      for (int j = J0 + (J0 & 1); j < RMAX; j += 2) {
        const float2 s = ffma2(make_float2(fi, fi), make_float2(rr[j], rr[j + 1]), make_float2(f[j], f[j + 1]));
        f[j] = s.x;
        f[j + 1] = s.y;
      }
    });
  }

  // Largest |E_ij| (i <= j) of E = G - I over the warp, from the Gram rows
  // in registers (lane j: row j).
  __device__ static __forceinline__ float gram_defect(const Row& g, int lane, int r) {
    float e = 0.f;
    if (lane < RMAX && lane < r) {
#pragma unroll
      for (int i = 0; i < RMAX; ++i) {
        const float x = fabsf(i == lane ? g[i] - 1.f : g[i]);
        if (i <= lane) e = (x > e || x != x) ? x : e;
      }
    }
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(e)));
  }

  // f <- f (I - F), F = triu(E) - diag(E)/2, with row j of `area` holding
  // G[i][j] (i <= j): column j becomes f_j (1 - E_jj/2) - sum_{i<j} f_i E_ij,
  // the columns from the last down.
  __device__ static __forceinline__ void correct(Row& f, const float* area) {
    static_for_down<0, RMAX>([&](auto jc) {
      constexpr int j = decltype(jc)::value;
      float e[((j + 4) / 4) * 4];
#pragma unroll
      for (int q = 0; q <= j; q += 4) {
        const float4 v = *reinterpret_cast<const float4*>(area + j * GS + q);
        e[q] = v.x;
        e[q + 1] = v.y;
        e[q + 2] = v.z;
        e[q + 3] = v.w;
      }
      float s = f[j] * fmaf(-0.5f, e[j] - 1.f, 1.f);
#pragma unroll
      for (int i = 0; i < j; ++i) s = fmaf(f[i], -e[i], s);
      f[j] = s;
    });
  }

  __device__ static __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
  }

  // Sum of x over the CTA (every thread gets it).
  __device__ static __forceinline__ float block_sum(float x, Smem& sm, int w, int lane) {
    x = warp_sum(x);
    if (lane == 0) sm.red[w] = x;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < W; ++v) s += sm.red[v];
    __syncthreads();  // red is free again
    return s;
  }

  // w_j = sum over rows of v * A[row][j] for j in (k, r) into red2 (warp sums;
  // the caller adds the W warps' entries after a barrier).
  __device__ static __forceinline__ void column_dots(Smem& sm, float v, int k, int r, int row, int w, int lane) {
    for (int j = k + 1; j < r; ++j) {
      const float c = warp_sum(v * sm.mt[One::mt_at(j, row)]);
      if (lane == 0) sm.red2[w][j] = c;
    }
  }
  __device__ static __forceinline__ void column_update(Smem& sm, float tv, int k, int r, int row) {
    for (int j = k + 1; j < r; ++j) {
      float wj = 0.f;
#pragma unroll
      for (int v = 0; v < W; ++v) wj += sm.red2[v][j];
      sm.mt[One::mt_at(j, row)] -= tv * wj;
    }
  }

  // Householder QR of the matrix in mt -- LAPACK's sgeqr2 then sorg2r, with the
  // formulas of FrameQR (slarfg: xnorm == 0 gives tau = 0 and beta = alpha;
  // else beta = -sign(alpha) sqrt(alpha^2 + xnorm^2), tau = (beta - alpha) /
  // beta, v = x / (alpha - beta)) -- one row per thread, the matrix kept in
  // shared memory; the R-diagonal rule applied (the first-significant rule is
  // the caller's).  The fallback for frames whose Gram fails the pivot test:
  // written to hold few registers, not for speed.  Called by every thread of
  // the CTA after the pass input is in mt; the thin Q replaces it.
  __device__ static void householder(Smem& sm, int w, int lane, int r, int sign_mode) {
    const int row = 32 * w + lane;
#pragma unroll 1
    for (int k = 0; k < r; ++k) {
      const float xk = sm.mt[One::mt_at(k, row)];
      const float ssq = block_sum(row > k ? xk * xk : 0.f, sm, w, lane);
      const float alpha = sm.mt[One::mt_at(k, k)];
      float beta = alpha, tau = 0.f, scale = 0.f;
      if (ssq != 0.f) {
        const float nrm = sqrtf(fmaf(alpha, alpha, ssq));
        beta = alpha >= 0.f ? -nrm : nrm;
        tau = (beta - alpha) / beta;
        scale = 1.f / (alpha - beta);
      }
      const float v = row > k ? xk * scale : (row == k ? 1.f : 0.f);
      if (row == 0) {
        sm.tau[k] = tau;
        sm.beta[k] = beta;
      }
      column_dots(sm, v, k, r, row, w, lane);
      __syncthreads();  // dots written; alpha and column k read by everyone
      if (row > k) sm.mt[One::mt_at(k, row)] = v;
      if (row == k) sm.mt[One::mt_at(k, k)] = beta;
      column_update(sm, tau * v, k, r, row);
      __syncthreads();  // red2 free, the trailing columns updated
    }
#pragma unroll 1
    for (int i = r - 1; i >= 0; --i) {
      const float vi = row > i ? sm.mt[One::mt_at(i, row)] : (row == i ? 1.f : 0.f);
      const float tau = sm.tau[i];
      column_dots(sm, vi, i, r, row, w, lane);
      __syncthreads();
      column_update(sm, tau * vi, i, r, row);
      sm.mt[One::mt_at(i, row)] = row > i ? -tau * vi : (row == i ? 1.f - tau : 0.f);
      __syncthreads();
    }
    if (sign_mode == GFST_SIGN_R_DIAG_POSITIVE) {
      for (int k = 0; k < r; ++k)
        if (sm.beta[k] < 0.f) sm.mt[One::mt_at(k, row)] = -sm.mt[One::mt_at(k, row)];
    }
  }

  // Reference sign rule (gfst.py:35-46) across the warps: the first row of each
  // column with |q| > eps_sign decides; rows are ordered warp by warp.
  __device__ static __forceinline__ void first_significant(Row& f, Smem& sm, int w, int lane, float eps_sign) {
    uint32_t hs = 0u, ng = 0u;
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      const uint32_t b = __ballot_sync(0xffffffffu, fabsf(f[c]) > eps_sign);
      const float v0 = __shfl_sync(0xffffffffu, f[c], b ? __ffs(b) - 1 : 0);
      hs |= (b ? 1u : 0u) << c;
      ng |= (b && v0 < 0.f ? 1u : 0u) << c;
    }
    if (lane == 0) {
      sm.sign_bits[w][0] = hs;
      sm.sign_bits[w][1] = ng;
    }
    __syncthreads();
    uint32_t decided = 0u, flip = 0u;
#pragma unroll
    for (int v = 0; v < W; ++v) {
      const uint32_t h = sm.sign_bits[v][0] & ~decided;
      flip |= sm.sign_bits[v][1] & h;
      decided |= h;
    }
    __syncthreads();  // the bits are read before the next token writes them again
#pragma unroll
    for (int c = 0; c < RMAX; ++c)
      if ((flip >> c) & 1u) f[c] = -f[c];
  }

  // In place: f (this lane's row) <- the row of the sign-fixed thin Q.  Warp 0
  // adds the partial Grams and runs the Cholesky (or decides on the
  // first-order correction) while the other warps wait at the barrier that
  // publishes its decision and R.
  __device__ static __forceinline__ void qr(Row& f, Smem& sm, int w, int lane, float eps_sign, int sign_mode,
                                            int r) {
    const int row = 32 * w + lane;
#pragma unroll 1
    for (int ps = 0; ps < 2; ++ps) {
      write_mt(f, sm, row);
      __syncwarp();
      gram_partial(sm, w, lane);
      __syncthreads();  // every partial is written; everyone is done with the last area
      if (w == 0) {
        Row g;
        sum_partials(g, sm, lane);
        int action;
        if (ps == 1 && gram_defect(g, lane, r) <= kFirstOrderTol) {
          if (lane < RMAX) {
#pragma unroll
            for (int q = 0; q < RMAX; q += 4)
              *reinterpret_cast<float4*>(sm.area + lane * GS + q) = make_float4(g[q], g[q + 1], g[q + 2], g[q + 3]);
          }
          action = kCorrect;
        } else {
          action = __all_sync(0xffffffffu, cholesky(g, sm.area, lane, r)) ? kSolve : kFallback;
        }
        if (lane == 0) sm.action = action;
      }
      __syncthreads();  // the decision and R (or G) are published; the partials are free
      const int action = sm.action;
      if (action == kCorrect) {
        correct(f, sm.area);
        break;
      }
      if (action == kFallback) {
        householder(sm, w, lane, r, sign_mode);
        read_mt(f, sm, row);
        if (sign_mode == GFST_SIGN_FIRST_SIGNIFICANT) first_significant(f, sm, w, lane, eps_sign);
        return;
      }
      read_mt(f, sm, row);  // the row waited in mt across the Cholesky
      solve(f, sm.area);
    }
    if (sign_mode == GFST_SIGN_FIRST_SIGNIFICANT) first_significant(f, sm, w, lane, eps_sign);
  }

  // ---- global memory and the rank-m update (one row per lane) -------------
  __device__ static __forceinline__ void load(Row& f, const float* __restrict__ src, int row, int d, int r,
                                              bool vec4) {
    if (row < d && vec4 && r == RMAX) {
#pragma unroll
      for (int c = 0; c < RMAX; c += 4) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(src + (size_t)row * RMAX + c));
        f[c] = x.x;
        f[c + 1] = x.y;
        f[c + 2] = x.z;
        f[c + 3] = x.w;
      }
      return;
    }
#pragma unroll
    for (int c = 0; c < RMAX; ++c) f[c] = (row < d && c < r) ? __ldg(src + (size_t)row * r + c) : 0.f;
  }

  __device__ static __forceinline__ void store(const Row& f, float* __restrict__ dst, int row, int d, int r,
                                               bool vec4) {
    if (row >= d) return;
    if (vec4 && r == RMAX) {
#pragma unroll
      for (int c = 0; c < RMAX; c += 4)
        *reinterpret_cast<float4*>(dst + (size_t)row * RMAX + c) = make_float4(f[c], f[c + 1], f[c + 2], f[c + 3]);
      return;
    }
#pragma unroll
    for (int c = 0; c < RMAX; ++c)
      if (c < r) dst[(size_t)row * r + c] = f[c];
  }

  // f += a B^T for this lane's row a = A[row, :m] (staged) and B [r, m] (staged).
  __device__ static __forceinline__ void rank_update(Row& f, const float* a_row, const float* B, int r, int m) {
    for (int u = 0; u < m; ++u) {
      const float au = a_row[u];
#pragma unroll
      for (int c = 0; c < RMAX; ++c) f[c] = fmaf(au, c < r ? B[c * m + u] : 0.f, f[c]);
    }
  }
};

}  // namespace gfst
