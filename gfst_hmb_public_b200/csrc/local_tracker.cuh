// Per-token local tracker: the largest flag basis U [d, r] and the nested flag
// bases V_l [r, dim_l] of one stream, advanced token by token on chip.
//
// Reference (pkhairkh/gfst-hmb-public): GfstHmbSublayer._update_local_bases
// (src/gfst_hmb_mpuc/modeling.py:2299-2423) and _local_alignment_features
// (modeling.py:2425-2437), with the update rule residual_rank_one_v1 of
// update_basis_candidate (src/gfst_hmb_mpuc/gfst.py:91-112):
//   w = B^T v;  s = (v - B w) / sqrt(||v||^2 + eps_update^2)
//   B~ = (1 - a) B + a v w^T + a s e_last^T;  B <- canonical thin QR of B~
// per token x: U takes v = x at rate a_last; p = U^T x; V_l takes v = p at
// rate a_l (Q keeps dim_l columns); features are the (cumulative, increment)
// pairs of ||V_l^T p||^2 / max(||x||^2, eps) and ||p||^2 / max(||x||^2, eps).
//
// U lives in registers in the 2-D cyclic lane layout of FrameQR.  The nested
// bases live in shared memory between tokens; their QR runs column-per-lane
// (SmallQR: lane j holds column j, reflectors broadcast through shared memory).
// The candidate is formed with separately rounded products and sums in the
// reference's order ((1 - a) B + a (v w^T)) + a (s e^T).
#pragma once

#include "frame_qr.cuh"

namespace gfst {

constexpr int kMaxTrackerLevels = 4;  // nested flag levels (flag_dims[:-1])

struct TrackerParams {
  int n_levels;
  int dims[kMaxTrackerLevels];
  int voff[kMaxTrackerLevels];  // float offset of level l inside a group's nested buffer
  float one_minus[kMaxTrackerLevels + 1];  // (float)(1 - rate), nested levels then the largest
  float rate[kMaxTrackerLevels + 1];       // (float)rate
  float eps;                               // feature denominator floor
  float eps_update_sq;                     // (float)(eps_update^2)
  float eps_sign;
  int sign_mode;
};

constexpr int kTrackerWarps = 4;

// Frames of at least 128 values per lane are parked in shared memory while the
// nested levels run, so the nested columns do not spill.
template <int DMAX, int RMAX, int RG, int CG>
__host__ __device__ constexpr int tracker_stash_floats() {
  return (DMAX / RG) * (RMAX / CG) >= 128 ? DMAX * RMAX : 0;
}

// dynamic shared floats per frame group: QR scratch (`fixed`, a multiple of 4),
// x stage, nested bases, parked frame, and with block accumulation the frame
// rows [d][r] and the projector sum [d][d]
__host__ __device__ inline int tracker_group_floats(int d, int r, const TrackerParams& prm, int stash, int fixed,
                                                    bool accumulate) {
  const int nl = prm.n_levels;
  const int nested_floats = nl > 0 ? prm.voff[nl - 1] + r * prm.dims[nl - 1] : 0;
  return fixed + 2 * d + ((nested_floats + 3) & ~3) + stash + (accumulate ? d * r + d * d : 0);
}

// Column-per-lane Householder thin QR of an m x n matrix, m <= RMAX <= 32,
// n <= m: group lane j < n holds column j in c[0, RMAX) (rows >= m are zero).
// Same arithmetic as FrameQR (LAPACK sgeqr2 / slarfg, then sorg2r order).
template <int RMAX>
struct SmallQR {
  struct Smem {
    float v[RMAX][RMAX];  // reflector k: v[k][i], 0 above row k, 1 at row k
    float tau[RMAX];
  };

  // All lanes of the warp call (uniform m, n); lanes j >= n only synchronise.
  __device__ static __forceinline__ void qr(float (&c)[RMAX], int j, int n, Smem& sm, float eps_sign,
                                            int sign_mode) {
    bool neg = false;  // R_jj < 0 for this lane's column
    for (int k = 0; k < n; ++k) {
      if (j == k) {
        float alpha = 0.f, xn2 = 0.f;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) {
          if (i == k) alpha = c[i];
          if (i > k) xn2 = fmaf(c[i], c[i], xn2);
        }
        float beta, tau, scal;
        if (xn2 == 0.f) {
          beta = alpha;
          tau = 0.f;
          scal = 0.f;
        } else {
          const float ss = fmaf(alpha, alpha, xn2);
          const float rs = __frsqrt_rn(ss);
          const float sigma = ss * rs;
          beta = alpha >= 0.f ? -sigma : sigma;
          tau = fmaf(fabsf(alpha), rs, 1.f);
          scal = __frcp_rn(alpha - beta);
        }
#pragma unroll
        for (int i = 0; i < RMAX; ++i) sm.v[k][i] = i < k ? 0.f : (i == k ? 1.f : c[i] * scal);
        sm.tau[k] = tau;
        neg = beta < 0.f;
      }
      __syncwarp();
      if (j > k && j < n) {
        const float tau = sm.tau[k];
        float w = 0.f;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) w = fmaf(sm.v[k][i], c[i], w);
        const float g = tau * w;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) c[i] = fmaf(-g, sm.v[k][i], c[i]);
      }
    }
    // explicit Q, sorg2r order: column j is formed at k = j, then H_{j-1} .. H_0
    for (int k = n - 1; k >= 0; --k) {
      const float tau = sm.tau[k];
      if (j == k) {
#pragma unroll
        for (int i = 0; i < RMAX; ++i) c[i] = i < k ? 0.f : (i == k ? 1.f - tau : -tau * sm.v[k][i]);
      } else if (j > k && j < n) {
        float w = 0.f;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) w = fmaf(sm.v[k][i], c[i], w);
        const float g = tau * w;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) c[i] = fmaf(-g, sm.v[k][i], c[i]);
      }
    }
    bool flip = false;
    if (sign_mode == GFST_SIGN_R_DIAG_POSITIVE) {
      flip = neg;
    } else {
      bool found = false;
#pragma unroll
      for (int i = 0; i < RMAX; ++i) {
        if (!found && fabsf(c[i]) > eps_sign) {
          found = true;
          flip = c[i] < 0.f;
        }
      }
    }
    if (flip) {
#pragma unroll
      for (int i = 0; i < RMAX; ++i) c[i] = -c[i];
    }
    __syncwarp();  // reflector buffer free for the next call
  }
};

// ((1 - a) b + a (v w)) + a s, each product and sum rounded separately
__device__ __forceinline__ float tracker_candidate(float om, float a, float b, float v, float w, float s,
                                                   bool novelty) {
  const float t = __fadd_rn(__fmul_rn(om, b), __fmul_rn(a, __fmul_rn(v, w)));
  return novelty ? __fadd_rn(t, __fmul_rn(a, s)) : t;
}

template <int DMAX, int RMAX, int RG, int CG, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1)
    local_tracker_stream_kernel(float* __restrict__ U, float* __restrict__ nested, const float* __restrict__ X,
                                int64_t n_streams, int T, int d, int r, TrackerParams prm,
                                float* __restrict__ features, float* __restrict__ proj_sum,
                                float* __restrict__ red_sum) {
  using QR = FrameQR<DMAX, RMAX, RG, CG>;
  using SQ = SmallQR<RMAX>;
  constexpr int TPF = QR::TPF;
  constexpr int GPW = 32 / TPF;
  constexpr int NG = WARPS * GPW;
  constexpr int RP = QR::RP, CPT = QR::CPT;
  static_assert(TPF >= RMAX, "a frame group needs a lane per nested row and column");
  __shared__ float pbuf[NG][RMAX], wbuf[NG][RMAX], sbuf[NG][RMAX];
  __shared__ float featb[NG][kMaxTrackerLevels];
  // per group: QR scratch, small-QR scratch, x stage [2][d], nested [sum r*dim_l], parked frame
  extern __shared__ __align__(16) float dyn[];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = lane % TPF;
  const int g = warp * GPW + lane / TPF;
  const int rg = t % RG, cg = t / RG;
  const int64_t f = (int64_t)blockIdx.x * NG + g;
  const bool valid = f < n_streams;
  const int64_t fs = valid ? f : 0;
  const int NL = prm.n_levels;
  constexpr int STASH = tracker_stash_floats<DMAX, RMAX, RG, CG>();
  constexpr int FIXED = (int)((sizeof(typename QR::Smem) + sizeof(typename SQ::Smem)) / sizeof(float));
  static_assert(sizeof(typename QR::Smem) % 16 == 0 && sizeof(typename SQ::Smem) % 16 == 0, "16-byte parts");
  // block tracker (projector and token sums): frames of at most 64 rows only
  constexpr bool kCanAcc = DMAX <= 64;
  const bool acc = kCanAcc && proj_sum != nullptr;
  const int group_floats = tracker_group_floats(d, r, prm, STASH, FIXED, acc);
  float* gbase = dyn + (size_t)g * group_floats;
  typename QR::Smem& qsm_g = *reinterpret_cast<typename QR::Smem*>(gbase);
  typename SQ::Smem& ssm_g = *reinterpret_cast<typename SQ::Smem*>(gbase + sizeof(typename QR::Smem) / sizeof(float));
  float* xstage = gbase + FIXED;
  float* vs = xstage + 2 * d;
  const int acc_floats = acc ? d * r + d * d : 0;
  float2* park = reinterpret_cast<float2*>(dyn + (size_t)(g + 1) * group_floats - acc_floats - STASH);  // [RP*CPT][TPF]
  float* ubuf = dyn + (size_t)(g + 1) * group_floats - acc_floats;  // [d][r]
  float* pacc = ubuf + d * r;                                         // [d][d]
  const float* Xf = X + fs * (size_t)T * d;

  auto issue = [&](int tok) {
    if (valid && tok < T) {
      float* dst = xstage + (tok & 1) * d;
      const float* src = Xf + (size_t)tok * d;
      for (int c = t; c < d / 4; c += TPF) {
        const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(dst + 4 * c));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(src + 4 * c) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  typename QR::Frame a;
  QR::load(a, U + fs * (size_t)d * r, t, d, r, valid, false);
  float2 racc[kCanAcc ? RP : 1];  // running token sum of this lane's rows (block tracker)
  if constexpr (kCanAcc) {
   if (acc) {
    const float* ps = proj_sum + fs * (size_t)d * d;
    for (int e = t; e < d * d; e += TPF) pacc[e] = valid ? ps[e] : 0.f;
#pragma unroll
    for (int p = 0; p < RP; ++p) {
      const int r0 = rg + (2 * p) * RG, r1 = rg + (2 * p + 1) * RG;
      racc[p] = make_float2(valid && r0 < d ? red_sum[fs * d + r0] : 0.f, valid && r1 < d ? red_sum[fs * d + r1] : 0.f);
    }
   }
  }
  for (int l = 0; l < NL; ++l) {
    const int n = prm.dims[l];
    const float* src = nested + ((size_t)fs * NL + l) * r * r;
    for (int e = t; e < r * n; e += TPF) vs[prm.voff[l] + e] = valid ? src[(e / n) * r + e % n] : 0.f;
  }
  __syncwarp();

  const float om_u = prm.one_minus[NL], a_u = prm.rate[NL];
  issue(0);
  for (int tok = 0; tok < T; ++tok) {
    issue(tok + 1);
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    __syncwarp();
    const float* x = xstage + (tok & 1) * d;

    // ---- largest basis: residual_rank_one_v1 candidate, canonical QR ----
    float2 xr[RP];
    QR::load_rows(xr, x, t, d);
    float2 sq2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int p = 0; p < RP; ++p) sq2 = ffma2(xr[p], xr[p], sq2);
    const float xsq = subgroup_allreduce<RG>(sq2.x + sq2.y);  // ||x||^2
    float w[CPT];
    QR::col_dots(a, xr, w);
    float2 proj[RP];
    QR::row_dots(a, w, proj);
    const float xnorm = sqrtf(xsq);
    const float den_u = sqrtf(__fadd_rn(__fmul_rn(xnorm, xnorm), prm.eps_update_sq));
#pragma unroll
    for (int p = 0; p < RP; ++p) {
      const float s0 = __fdiv_rn(__fsub_rn(xr[p].x, proj[p].x), den_u);
      const float s1 = __fdiv_rn(__fsub_rn(xr[p].y, proj[p].y), den_u);
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const bool nov = cg + c * CG == r - 1;
        a[p][c].x = tracker_candidate(om_u, a_u, a[p][c].x, xr[p].x, w[c], s0, nov);
        a[p][c].y = tracker_candidate(om_u, a_u, a[p][c].y, xr[p].y, w[c], s1, nov);
      }
    }
    QR::qr(a, lane, t, qsm_g, prm.eps_sign, prm.sign_mode, r);

    // ---- block tracker: projector_sum += U U^T, reduced_sum += x ----
    if constexpr (kCanAcc) {
     if (acc) {
#pragma unroll
      for (int p = 0; p < RP; ++p) racc[p] = __fadd2_rn(racc[p], xr[p]);
#pragma unroll
      for (int sl = 0; sl < QR::RPT; ++sl) {
        const int row = rg + sl * RG;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          const int col = cg + c * CG;
          if (row < d && col < r) ubuf[row * r + col] = QR::get(a, sl, c);
        }
      }
      __syncwarp();
      // 2 x 2 tiles of the upper triangle (row pairs i2 <= j2), each dot in column order
      const int h = d / 2, n_tiles = h * (h + 1) / 2;
      for (int e = t; e < n_tiles; e += TPF) {
        int i2 = 0, rem = e;
        while (rem >= h - i2) {
          rem -= h - i2;
          ++i2;
        }
        const int j2 = i2 + rem;
        const float4* u0 = reinterpret_cast<const float4*>(ubuf + (2 * i2) * r);
        const float4* u1 = reinterpret_cast<const float4*>(ubuf + (2 * i2 + 1) * r);
        const float4* v0 = reinterpret_cast<const float4*>(ubuf + (2 * j2) * r);
        const float4* v1 = reinterpret_cast<const float4*>(ubuf + (2 * j2 + 1) * r);
        float d00 = 0.f, d01 = 0.f, d10 = 0.f, d11 = 0.f;
        for (int c4 = 0; c4 < r / 4; ++c4) {
          const float4 a0 = u0[c4], a1 = u1[c4], b0 = v0[c4], b1 = v1[c4];
          d00 = fmaf(a0.x, b0.x, d00); d00 = fmaf(a0.y, b0.y, d00); d00 = fmaf(a0.z, b0.z, d00); d00 = fmaf(a0.w, b0.w, d00);
          d01 = fmaf(a0.x, b1.x, d01); d01 = fmaf(a0.y, b1.y, d01); d01 = fmaf(a0.z, b1.z, d01); d01 = fmaf(a0.w, b1.w, d01);
          d10 = fmaf(a1.x, b0.x, d10); d10 = fmaf(a1.y, b0.y, d10); d10 = fmaf(a1.z, b0.z, d10); d10 = fmaf(a1.w, b0.w, d10);
          d11 = fmaf(a1.x, b1.x, d11); d11 = fmaf(a1.y, b1.y, d11); d11 = fmaf(a1.z, b1.z, d11); d11 = fmaf(a1.w, b1.w, d11);
        }
        const int i = 2 * i2, j = 2 * j2;
        pacc[i * d + j] += d00;
        pacc[i * d + j + 1] += d01;
        pacc[(i + 1) * d + j + 1] += d11;
        if (i2 != j2) {
          pacc[(i + 1) * d + j] += d10;
          pacc[j * d + i] += d00;
          pacc[(j + 1) * d + i] += d01;
          pacc[j * d + i + 1] += d10;
          pacc[(j + 1) * d + i + 1] += d11;
        } else {
          pacc[(i + 1) * d + j] += d01;  // the tile's transposed corner: same dot, same bits
        }
      }
      __syncwarp();
     }
    }

    // ---- p = U^T x (new U) ----
    QR::col_dots(a, xr, w);
    if (rg == 0) {
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int col = cg + c * CG;
        if (col < r) pbuf[g][col] = w[c];
      }
    }
    __syncwarp();
    float psq = 0.f;  // ||p||^2, same order on every lane
    for (int i = 0; i < r; ++i) psq = fmaf(pbuf[g][i], pbuf[g][i], psq);
    const float pnorm = sqrtf(psq);
    const float den_n = sqrtf(__fadd_rn(__fmul_rn(pnorm, pnorm), prm.eps_update_sq));
    const float den_x = fmaxf(xsq, prm.eps);

    // ---- nested flag levels (column-per-lane) ----
    if constexpr (STASH > 0) {
#pragma unroll
      for (int p = 0; p < RP; ++p)
#pragma unroll
        for (int c = 0; c < CPT; ++c) park[(p * CPT + c) * TPF + t] = a[p][c];
    }
    for (int l = 0; l < NL; ++l) {
      const int n = prm.dims[l];
      float* V = vs + prm.voff[l];
      float c[RMAX];
      float wj = 0.f;
#pragma unroll
      for (int i = 0; i < RMAX; ++i) {
        c[i] = (t < n && i < r) ? V[i * n + t] : 0.f;
        wj = fmaf(c[i], i < r ? pbuf[g][i] : 0.f, wj);
      }
      if (t < n) wbuf[g][t] = wj;
      __syncwarp();
      if (t < r) {
        float pr = 0.f;
        for (int jj = 0; jj < n; ++jj) pr = fmaf(V[t * n + jj], wbuf[g][jj], pr);
        sbuf[g][t] = __fdiv_rn(__fsub_rn(pbuf[g][t], pr), den_n);
      }
      __syncwarp();
      if (t < n) {
        const float om = prm.one_minus[l], al = prm.rate[l];
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
          if (i < r) c[i] = tracker_candidate(om, al, c[i], pbuf[g][i], wj, sbuf[g][i], t == n - 1);
      }
      SQ::qr(c, t, n, ssm_g, prm.eps_sign, prm.sign_mode);
      float vp = 0.f;
      if (t < n) {
#pragma unroll
        for (int i = 0; i < RMAX; ++i) {
          if (i < r) {
            V[i * n + t] = c[i];
            vp = fmaf(c[i], pbuf[g][i], vp);
          }
        }
      }
      float vsq = t < n ? vp * vp : 0.f;
      vsq = subgroup_allreduce<TPF>(vsq);
      if (t == 0) featb[g][l] = __fdiv_rn(vsq, den_x);
      __syncwarp();
    }
    if constexpr (STASH > 0) {
#pragma unroll
      for (int p = 0; p < RP; ++p)
#pragma unroll
        for (int c = 0; c < CPT; ++c) a[p][c] = park[(p * CPT + c) * TPF + t];
    }
    if (features != nullptr && valid && t == 0) {
      float* fo = features + ((size_t)fs * T + tok) * 2 * (NL + 1);
      float prev = 0.f;
      for (int l = 0; l <= NL; ++l) {
        const float cum = l < NL ? featb[g][l] : __fdiv_rn(psq, den_x);
        fo[2 * l] = cum;
        fo[2 * l + 1] = __fsub_rn(cum, prev);
        prev = cum;
      }
    }
    __syncwarp();  // stage buffer and shared vectors free before the next token
  }
  QR::store(a, U + fs * (size_t)d * r, t, d, r, valid, false);
  if constexpr (kCanAcc) {
   if (acc && valid) {
    float* ps = proj_sum + fs * (size_t)d * d;
    for (int e = t; e < d * d; e += TPF) ps[e] = pacc[e];
    if (cg == 0) {
#pragma unroll
      for (int p = 0; p < RP; ++p) {
        const int r0 = rg + (2 * p) * RG, r1 = rg + (2 * p + 1) * RG;
        if (r0 < d) red_sum[fs * d + r0] = racc[p].x;
        if (r1 < d) red_sum[fs * d + r1] = racc[p].y;
      }
    }
   }
  }
  for (int l = 0; l < NL; ++l) {
    const int n = prm.dims[l];
    float* dst = nested + ((size_t)fs * NL + l) * r * r;
    if (valid)
      for (int e = t; e < r * r; e += TPF) dst[e] = (e % r) < n ? vs[prm.voff[l] + (e / r) * n + e % r] : 0.f;
  }
}

template <int DMAX, int RMAX, int RG, int CG>
int launch_tracker(float* U, float* nested, const float* X, int64_t n, int T, int d, int r, const TrackerParams& prm,
                   float* features, float* proj_sum, float* red_sum, cudaStream_t stream) {
  constexpr int NG = kTrackerWarps * (32 / (RG * CG));
  const int64_t blocks = (n + NG - 1) / NG;
  GFST_REQUIRE(blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many streams: %lld", (long long)n);
  const size_t smem =
      (size_t)NG *
      tracker_group_floats(d, r, prm, tracker_stash_floats<DMAX, RMAX, RG, CG>(),
                           (int)((sizeof(typename FrameQR<DMAX, RMAX, RG, CG>::Smem) +
                                  sizeof(typename SmallQR<RMAX>::Smem)) / sizeof(float)),
                           proj_sum != nullptr) *
      sizeof(float);
  GFST_REQUIRE(smem <= 200u * 1024u, GFST_ERR_SHAPE, "tracker state needs %zu bytes of shared memory", smem);
  auto kern = local_tracker_stream_kernel<DMAX, RMAX, RG, CG, kTrackerWarps>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)blocks, kTrackerWarps * 32, smem, stream>>>(U, nested, X, n, T, d, r, prm, features, proj_sum,
                                                                red_sum);
  return check_launch("local_tracker_stream_kernel");
}

}  // namespace gfst
