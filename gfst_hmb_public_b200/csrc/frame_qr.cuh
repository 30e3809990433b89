// Register-resident Householder thin QR of one d x r fp32 frame per lane group.
//
// Layout (2-D cyclic): a frame group is TPF = RG * CG consecutive lanes of one
// warp.  Group lane t is (rg, cg) = (t % RG, t / RG); it owns rows
// rg + s*RG (s < RPT = DMAX/RG) of columns cg + c*CG (c < CPT = RMAX/CG), all in
// registers, stored as float2 row pairs (slots 2i, 2i+1) so the update and the
// dot products issue packed fma.f32x2.  Cyclic columns keep every column group
// busy until the last reflector; the dot products of a step only need a
// reduction over the RG lanes of one column group.  Rows >= d and columns >= r
// are zero padding: a zero row adds nothing to any reflector and zero trailing
// columns leave the leading columns of Q unchanged, so the leading d x r block
// of the padded result is the QR of the unpadded frame.
//
// Arithmetic follows LAPACK's unblocked sgeqr2/slarfg + sorg2r (the path that
// torch.linalg.qr takes for these sizes; gfst.py:26-32 of the reference) and the
// reference's own fixed-order device kernel
// (src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:447-549):
//   step k:  alpha = A[k,k], xnorm^2 = sum_{i>k} A[i,k]^2
//            xnorm == 0      -> tau = 0, beta = alpha (H_k = I, as slarfg)
//            otherwise       beta = -sign(alpha) * sqrt(alpha^2 + xnorm^2)
//                            tau  = (beta - alpha) / beta,  v = [1; x / (alpha - beta)]
//   trailing update A[k:, j] -= tau * v * (v^T A[k:, j]).
// The step's reduction carries the "Gram row" c_j = sum_{i>k} x_i A[i,j], so
// v^T A[k:,j] = A[k,j] + c_j / (alpha - beta) needs no second pass.  Q is then
// accumulated backward from the identity in place (sorg2r order).
#pragma once

#include "gfst_common.cuh"

namespace gfst {

template <int DMAX, int RMAX, int RG, int CG>
struct FrameQR {
  static constexpr int TPF = RG * CG;
  static constexpr int RPT = DMAX / RG;  // row slots per lane
  static constexpr int RP = RPT / 2;     // row pairs per lane
  static constexpr int CPT = RMAX / CG;  // local columns per lane
  static_assert(TPF >= 2 && TPF <= 32 && (TPF & (TPF - 1)) == 0, "TPF must be a power of two <= 32");
  static_assert((RG & (RG - 1)) == 0 && (CG & (CG - 1)) == 0, "RG, CG powers of two");
  static_assert(DMAX % (2 * RG) == 0, "each lane needs an even number of row slots");
  static_assert(RMAX % CG == 0 && (CPT & (CPT - 1)) == 0, "CPT must be a power of two");
  static_assert(RMAX <= 32 && RMAX <= DMAX, "thin QR needs r <= d, r <= 32");
  static constexpr int XS = RPT + 4;     // padded row stride of the broadcast buffer (floats)

  // a[i][c] = rows (slot 2i, slot 2i+1) of local column c
  using Frame = float2[RP][CPT];

  // Per-group shared scratch (double-buffered by step parity).
  struct __align__(16) Smem {
    float xb[2][RG][XS];   // column K of this step (reflector source), by row group
    float piv[2][CG][CPT]; // pivot row K, by column group
    float red[2][CG][CPT]; // reduced dot products, by column group
    float tau[RMAX];
  };

  __device__ static __forceinline__ float get(const Frame& a, int s, int c) {
    return (s & 1) ? a[s >> 1][c].y : a[s >> 1][c].x;
  }
  __device__ static __forceinline__ void set(Frame& a, int s, int c, float v) {
    if (s & 1) {
      a[s >> 1][c].y = v;
    } else {
      a[s >> 1][c].x = v;
    }
  }

  // Reflectors are processed in groups of CG consecutive steps K = C0*CG + j
  // (j < CG): within a group the local column index (C0) and the row slot
  // holding row K (SK) are compile-time constants, so the group's code is a
  // rolled loop over j.  This keeps the unrolled code CG times smaller than a
  // fully unrolled factorisation (instruction-cache bound otherwise).
  static_assert(RG % CG == 0, "a group of CG steps must fall inside one row slot");

  // row of slot s is > K, for K in group C0 (compile-time except slot SK)
  template <int C0>
  __device__ static __forceinline__ bool below(int s, int rg, int K) {
    constexpr int SK = (C0 * CG) / RG;
    if (s > SK) return true;
    if (s < SK) return false;
    return rg + s * RG > K;
  }

  // Read column K (written by its column group) from the broadcast buffer,
  // zeroing rows <= K.
  template <int C0>
  __device__ static __forceinline__ void read_column(float2 (&x)[RP], const float* xb, int rg, int K) {
#pragma unroll
    for (int i = 0; i < RP; i += 2) {
      if (i + 1 < RP) {
        const float4 q = *reinterpret_cast<const float4*>(xb + rg * XS + 2 * i);
        x[i] = make_float2(q.x, q.y);
        x[i + 1] = make_float2(q.z, q.w);
      } else {
        x[i] = *reinterpret_cast<const float2*>(xb + rg * XS + 2 * i);
      }
    }
#pragma unroll
    for (int i = 0; i < RP; ++i) {
      if (!below<C0>(2 * i, rg, K)) x[i].x = 0.f;
      if (!below<C0>(2 * i + 1, rg, K)) x[i].y = 0.f;
    }
  }

  template <int C0>
  __device__ static __forceinline__ void write_column(const Frame& a, float* xb, int rg) {
#pragma unroll
    for (int i = 0; i < RP; i += 2) {
      if (i + 1 < RP) {
        *reinterpret_cast<float4*>(xb + rg * XS + 2 * i) =
            make_float4(a[i][C0].x, a[i][C0].y, a[i + 1][C0].x, a[i + 1][C0].y);
      } else {
        *reinterpret_cast<float2*>(xb + rg * XS + 2 * i) = a[i][C0];
      }
    }
  }

  // Dot products of the (masked) column x with local columns c in [C0, CPT) --
  // c == C0 counts only for column groups right of K's (cg > j) -- reduced over
  // the RG lanes of the column group and published to red[0 ..).
  template <int C0>
  __device__ static __forceinline__ void column_dots(const Frame& a, const float2 (&x)[RP], int rg, bool first_live,
                                                     float* red) {
    constexpr int NV = CPT - C0;
    constexpr int P = pow2_ceil(NV);
    float v[P];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int p = 0; p < RP; ++p) acc = ffma2(x[p], a[p][C0 + i], acc);
      v[i] = acc.x + acc.y;
    }
#pragma unroll
    for (int i = NV; i < P; ++i) v[i] = 0.f;
    if (!first_live) v[0] = 0.f;
    subgroup_reduce_scatter<P, RG>(v, rg);
    subgroup_publish<P, RG>(v, rg, red);
  }

  static_assert(CPT % 4 == 0, "local column rows move as float4");

  // this lane's slot-SK row (row K when the lane owns it) -> dst[0..CPT)
  template <int SK>
  __device__ static __forceinline__ void write_row(const Frame& a, float* dst) {
#pragma unroll
    for (int c = 0; c < CPT; c += 4)
      *reinterpret_cast<float4*>(dst + c) = make_float4(get(a, SK, c), get(a, SK, c + 1), get(a, SK, c + 2),
                                                        get(a, SK, c + 3));
  }
  __device__ static __forceinline__ void read_row(float (&v)[CPT], const float* src) {
#pragma unroll
    for (int c = 0; c < CPT; c += 4) {
      const float4 q = *reinterpret_cast<const float4*>(src + c);
      v[c] = q.x;
      v[c + 1] = q.y;
      v[c + 2] = q.z;
      v[c + 3] = q.w;
    }
  }

  // a[:, C0 + i] -= g[i] * x for i < NV (packed, two columns' scalars at a time)
  template <int C0>
  __device__ static __forceinline__ void rank1_update(Frame& a, const float2 (&x)[RP], const float (&g)[CPT]) {
    constexpr int NV = CPT - C0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float2 ng = make_float2(-g[i], -g[i]);
#pragma unroll
      for (int p = 0; p < RP; ++p) a[p][C0 + i] = ffma2(ng, x[p], a[p][C0 + i]);
    }
  }

  template <int C0>
  __device__ static __forceinline__ void geqrf_group(Frame& a, int rg, int cg, Smem& sm, uint32_t& rneg) {
    constexpr int NV = CPT - C0, SK = (C0 * CG) / RG;
#pragma unroll 1
    for (int j = 0; j < CG; ++j) {
      const int K = C0 * CG + j;
      float* xb = &sm.xb[K & 1][0][0];
      float* piv = &sm.piv[K & 1][0][0];
      float* red = &sm.red[K & 1][cg][0];
      const bool own_pivot = (rg == K - SK * RG);  // this lane holds row K (slot SK)
      const bool first_live = cg > j;              // local column C0 is right of K
      if (cg == j) write_column<C0>(a, xb, rg);
      if (own_pivot) write_row<SK>(a, piv + cg * CPT);
      __syncwarp();
      float2 x[RP];
      read_column<C0>(x, xb, rg, K);
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int p = 0; p < RP; ++p) acc = ffma2(x[p], x[p], acc);
      const float xn2 = subgroup_allreduce<RG>(acc.x + acc.y);
      column_dots<C0>(a, x, rg, first_live, red);
      __syncwarp();

      const float alpha = piv[j * CPT + C0];
      float pv[CPT], rv[CPT];
      read_row(pv, piv + cg * CPT);
      read_row(rv, red);
      float beta, tau, scal;
      if (xn2 == 0.f) {
        beta = alpha;
        tau = 0.f;
        scal = 0.f;
      } else {
        // sigma = sqrt(alpha^2 + xnorm^2), beta = -sign(alpha) sigma,
        // tau = (beta - alpha) / beta = 1 + |alpha| / sigma, scal = 1 / (alpha - beta);
        // correctly rounded rsqrt / rcp keep the per-step chain short
        const float ss = fmaf(alpha, alpha, xn2);
        const float rs = __frsqrt_rn(ss);
        const float sigma = ss * rs;
        beta = alpha >= 0.f ? -sigma : sigma;
        tau = fmaf(fabsf(alpha), rs, 1.f);
        scal = __frcp_rn(alpha - beta);
      }
      rneg |= (beta < 0.f ? 1u : 0u) << K;
      if (rg == 0 && cg == 0) sm.tau[K] = tau;

      // g_i = tau * (piv_i + scal * c_i) * scal, zero for column K / finished columns
      float g[CPT];
#pragma unroll
      for (int i = 0; i < NV; i += 2) {
        if (i + 1 < NV) {
          const float2 w = ffma2(make_float2(scal, scal), make_float2(rv[i], rv[i + 1]),
                                 make_float2(pv[C0 + i], pv[C0 + i + 1]));
          const float2 gg = __fmul2_rn(__fmul2_rn(w, make_float2(tau, tau)), make_float2(scal, scal));
          g[i] = gg.x;
          g[i + 1] = gg.y;
        } else {
          g[i] = tau * fmaf(scal, rv[i], pv[C0 + i]) * scal;
        }
      }
      if (!first_live) g[0] = 0.f;
      // row K takes A[K, j] -= tau * w_j: with x_K = alpha - beta the packed
      // update g * x_K gives exactly that term (g = tau w scal, scal = 1/(alpha-beta))
      if (own_pivot) {
        if (SK & 1) {
          x[SK >> 1].y = alpha - beta;
        } else {
          x[SK >> 1].x = alpha - beta;
        }
      }
      rank1_update<C0>(a, x, g);
      if (cg == j) {
        // column K: v = x * scal below the diagonal, beta on it
#pragma unroll
        for (int p = 0; p < RP; ++p) {
          if (below<C0>(2 * p, rg, K)) a[p][C0].x *= scal;
          if (below<C0>(2 * p + 1, rg, K)) a[p][C0].y *= scal;
        }
        if (own_pivot) set(a, SK, C0, beta);
      }
    }
  }

  // Backward accumulation of the explicit thin Q (sorg2r order), in place.
  template <int C0>
  __device__ static __forceinline__ void orgqr_group(Frame& a, int rg, int cg, Smem& sm) {
    constexpr int NV = CPT - C0, SK = (C0 * CG) / RG;
#pragma unroll 1
    for (int j = CG - 1; j >= 0; --j) {
      const int K = C0 * CG + j;
      const float tau = sm.tau[K];
      const bool own_pivot = (rg == K - SK * RG);
      const bool first_live = cg > j;
      if (K + 1 < RMAX) {
        float* xb = &sm.xb[K & 1][0][0];
        float* red = &sm.red[K & 1][cg][0];
        if (cg == j) write_column<C0>(a, xb, rg);
        __syncwarp();
        float2 v[RP];
        read_column<C0>(v, xb, rg, K);
        column_dots<C0>(a, v, rg, first_live, red);
        __syncwarp();
        float rv[CPT], g[CPT];
        read_row(rv, red);
#pragma unroll
        for (int i = 0; i < NV; i += 2) {
          if (i + 1 < NV) {
            const float2 tp = __fmul2_rn(make_float2(tau, tau), make_float2(rv[i], rv[i + 1]));
            g[i] = tp.x;
            g[i + 1] = tp.y;
          } else {
            g[i] = tau * rv[i];
          }
        }
        if (!first_live) g[0] = 0.f;
        // v_K = 1: row K of each trailing column (zeroed at that column's own
        // step) becomes -tau * (v^T Q[:, column]) through the packed update
        if (own_pivot) {
          if (SK & 1) {
            v[SK >> 1].y = 1.f;
          } else {
            v[SK >> 1].x = 1.f;
          }
        }
        rank1_update<C0>(a, v, g);
      }
      if (cg == j) {
#pragma unroll
        for (int s = 0; s < RPT; ++s) {
          if (below<C0>(s, rg, K)) {
            set(a, s, C0, get(a, s, C0) * -tau);
          } else if (s == SK && own_pivot) {
            set(a, s, C0, 1.f - tau);
          } else {
            set(a, s, C0, 0.f);  // rows < K: discard R
          }
        }
      }
    }
  }

  // Columns to negate under the reference's first-significant-entry rule
  // (gfst.py:35-46): first row (in row order) with |q| > eps_sign, negative ->
  // flip.  Bit c of the result refers to local column c.
  __device__ static __forceinline__ uint32_t first_significant_flips(const Frame& a, int lane, int cg,
                                                                     float eps_sign, uint32_t local_mask) {
    const int sub = (lane / TPF) * TPF + cg * RG;  // first lane of my column group
    const uint32_t gmask = RG == 32 ? 0xffffffffu : ((1u << RG) - 1u);
    uint32_t flip = 0u, found = 0u;
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const float q = get(a, s, c);
        const uint32_t sig = (__ballot_sync(0xffffffffu, fabsf(q) > eps_sign) >> sub) & gmask;
        const uint32_t neg = (__ballot_sync(0xffffffffu, q < 0.f) >> sub) & gmask;
        if (!((found >> c) & 1u) && sig != 0u) {
          found |= 1u << c;
          flip |= ((neg >> (__ffs(sig) - 1)) & 1u) << c;
        }
      }
      if (!__any_sync(0xffffffffu, (found & local_mask) != local_mask)) break;
    }
    return flip;
  }

  // In place: a <- sign-fixed thin Q.  r = number of real columns.
  __device__ static __forceinline__ void qr(Frame& a, int lane, int t, Smem& sm, float eps_sign, int sign_mode,
                                            int r) {
    const int rg = t % RG, cg = t / RG;
    uint32_t rneg = 0u;
    static_for<0, CPT>([&](auto cc) { geqrf_group<decltype(cc)::value>(a, rg, cg, sm, rneg); });
    __syncwarp();  // tau[] writes before any orgqr read
    static_for_down<0, CPT>([&](auto cc) { orgqr_group<decltype(cc)::value>(a, rg, cg, sm); });
    uint32_t flip = 0u;
    if (sign_mode == GFST_SIGN_R_DIAG_POSITIVE) {
#pragma unroll
      for (int c = 0; c < CPT; ++c) flip |= ((rneg >> (cg + c * CG)) & 1u) << c;
    } else {
      uint32_t local_mask = 0u;
#pragma unroll
      for (int c = 0; c < CPT; ++c) local_mask |= (cg + c * CG < r ? 1u : 0u) << c;
      flip = first_significant_flips(a, lane, cg, eps_sign, local_mask);
    }
#pragma unroll
    for (int p = 0; p < RP; ++p) {
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        if ((flip >> c) & 1u) a[p][c] = make_float2(-a[p][c].x, -a[p][c].y);
      }
    }
  }

  // Load a dense row-major [d, r] frame, zero padded.  With one column group
  // (CG == 1) a lane owns whole rows and full-width frames load as float4
  // (vec4: the host checked 16-byte alignment of every row).
  __device__ static __forceinline__ void load(Frame& a, const float* __restrict__ src, int t, int d, int r,
                                              bool valid, bool vec4) {
    const int rg = t % RG, cg = t / RG;
    if constexpr (CG == 1 && RMAX % 4 == 0) {
      if (vec4 && r == RMAX) {
#pragma unroll
        for (int s = 0; s < RPT; ++s) {
          const int row = rg + s * RG;
#pragma unroll
          for (int c4 = 0; c4 < RMAX / 4; ++c4) {
            float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
            if (valid && row < d) q = __ldg(reinterpret_cast<const float4*>(src + (size_t)row * RMAX) + c4);
            set(a, s, 4 * c4 + 0, q.x);
            set(a, s, 4 * c4 + 1, q.y);
            set(a, s, 4 * c4 + 2, q.z);
            set(a, s, 4 * c4 + 3, q.w);
          }
        }
        return;
      }
    }
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const int row = rg + s * RG;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int col = cg + c * CG;
        set(a, s, c, (valid && row < d && col < r) ? __ldg(src + (size_t)row * r + col) : 0.f);
      }
    }
  }

  __device__ static __forceinline__ void store(const Frame& a, float* __restrict__ dst, int t, int d, int r,
                                               bool valid, bool vec4) {
    const int rg = t % RG, cg = t / RG;
    if (!valid) return;
    if constexpr (CG == 1 && RMAX % 4 == 0) {
      if (vec4 && r == RMAX) {
#pragma unroll
        for (int s = 0; s < RPT; ++s) {
          const int row = rg + s * RG;
          if (row >= d) continue;
#pragma unroll
          for (int c4 = 0; c4 < RMAX / 4; ++c4) {
            reinterpret_cast<float4*>(dst + (size_t)row * RMAX)[c4] =
                make_float4(get(a, s, 4 * c4), get(a, s, 4 * c4 + 1), get(a, s, 4 * c4 + 2), get(a, s, 4 * c4 + 3));
          }
        }
        return;
      }
    }
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const int row = rg + s * RG;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int col = cg + c * CG;
        if (row < d && col < r) dst[(size_t)row * r + col] = get(a, s, c);
      }
    }
  }

  // Rows of a d-vector owned by this lane, as row pairs (zero beyond d).
  __device__ static __forceinline__ void load_rows(float2 (&xr)[RP], const float* x, int t, int d) {
    const int rg = t % RG;
#pragma unroll
    for (int p = 0; p < RP; ++p) {
      const int r0 = rg + (2 * p) * RG, r1 = rg + (2 * p + 1) * RG;
      xr[p] = make_float2(r0 < d ? x[r0] : 0.f, r1 < d ? x[r1] : 0.f);
    }
  }

  // w[c] = a[:, c] . x for this lane's columns (all rows: reduced over the RG
  // lanes of the column group; every lane of the group gets the same bits).
  __device__ static __forceinline__ void col_dots(const Frame& a, const float2 (&xr)[RP], float (&w)[CPT]) {
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int p = 0; p < RP; ++p) acc = ffma2(a[p][c], xr[p], acc);
      w[c] = subgroup_allreduce<RG>(acc.x + acc.y);
    }
  }

  // proj[p] = a[rows of p, :] . w (all columns: reduced over the CG lanes that
  // share this lane's rows).
  __device__ static __forceinline__ void row_dots(const Frame& a, const float (&w)[CPT], float2 (&proj)[RP]) {
#pragma unroll
    for (int p = 0; p < RP; ++p) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < CPT; ++c) acc = ffma2(a[p][c], make_float2(w[c], w[c]), acc);
#pragma unroll
      for (int o = CG / 2; o >= 1; o >>= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o * RG);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o * RG);
      }
      proj[p] = acc;
    }
  }

  __device__ static __forceinline__ void scale(Frame& a, float beta) {
    const float2 b2 = make_float2(beta, beta);
#pragma unroll
    for (int p = 0; p < RP; ++p)
#pragma unroll
      for (int c = 0; c < CPT; ++c) a[p][c] = __fmul2_rn(a[p][c], b2);
  }

  // a += A B^T with A [d, m], B [r, m] row-major (global or shared memory).
  __device__ static __forceinline__ void rank_update(Frame& a, const float* A, const float* B, int t, int d, int r,
                                                     int m) {
    const int rg = t % RG, cg = t / RG;
    for (int mm = 0; mm < m; ++mm) {
      float2 ax[RP];
#pragma unroll
      for (int p = 0; p < RP; ++p) {
        const int r0 = rg + (2 * p) * RG, r1 = rg + (2 * p + 1) * RG;
        ax[p] = make_float2(r0 < d ? A[r0 * m + mm] : 0.f, r1 < d ? A[r1 * m + mm] : 0.f);
      }
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int col = cg + c * CG;
        const float b = col < r ? B[col * m + mm] : 0.f;
        const float2 b2 = make_float2(b, b);
#pragma unroll
        for (int p = 0; p < RP; ++p) a[p][c] = ffma2(ax[p], b2, a[p][c]);
      }
    }
  }
};

}  // namespace gfst
