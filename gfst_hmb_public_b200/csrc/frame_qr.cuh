// Register-resident Householder thin QR of one d x r fp32 frame per lane group.
//
// Layout: TPF consecutive lanes of a warp (a "frame group", TPF a power of two
// <= 32) own one frame of capacity DMAX x RMAX.  Group lane t holds rows
// t, t + TPF, t + 2*TPF, ... (RPT = DMAX / TPF rows), all RMAX columns of each,
// in registers.  Rows >= d and columns >= r are zero padding: a zero row adds
// nothing to any reflector and a zero trailing column leaves the leading
// columns of Q unchanged, so the leading d x r block of the padded result is
// the QR of the unpadded frame.
//
// Arithmetic follows LAPACK's unblocked sgeqr2/slarfg + sorg2r (the path that
// torch.linalg.qr takes for these sizes, gfst.py:26-32 in the reference) and the
// reference's own fixed-order device kernel
// (src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:447-549):
//   step k:  alpha = A[k,k], xnorm^2 = sum_{i>k} A[i,k]^2
//            xnorm == 0      -> tau = 0, beta = alpha (H_k = I, as slarfg)
//            otherwise       beta = -sign(alpha) * sqrt(alpha^2 + xnorm^2)
//                            tau  = (beta - alpha) / beta,  v = [1; x / (alpha - beta)]
//   trailing update A[k:, j] -= tau * v * (v^T A[k:, j]).
// Every step needs one reduction across the group.  The reduction carries the
// "Gram row" c_j = sum_{i>k} x_i A[i,j] together with xnorm^2, so
// v^T A[k:,j] = A[k,j] + c_j / (alpha - beta) is known without a second pass.
// Reductions are recursive-halving butterflies over the group's lanes (each
// lane ends with a slice of the totals), followed by a shared-memory gather.
#pragma once

#include "gfst_common.cuh"

namespace gfst {

// Sum v[0..P) over the TPF lanes of a frame group (group lane index t).
// On return: if P >= TPF, v[0..P/TPF) holds the totals of values
// [t*P/TPF, (t+1)*P/TPF); if P < TPF, v[0] holds the total of value t/(TPF/P).
template <int S, int O, int P>
struct ReduceScatter {
  __device__ static __forceinline__ void run(float (&v)[P], int t) {
    if constexpr (O >= 1) {
      if constexpr (S > 1) {
        const bool upper = (t & O) != 0;
#pragma unroll
        for (int i = 0; i < S / 2; ++i) {
          const float send = upper ? v[i] : v[i + S / 2];
          const float keep = upper ? v[i + S / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
        }
        ReduceScatter<S / 2, O / 2, P>::run(v, t);
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
        ReduceScatter<1, O / 2, P>::run(v, t);
      }
    }
  }
};

template <int P, int TPF>
__device__ __forceinline__ void group_reduce_scatter(float (&v)[P], int t) {
  ReduceScatter<P, TPF / 2, P>::run(v, t);
}

// Write the totals left by group_reduce_scatter to red[0..P).
template <int P, int TPF>
__device__ __forceinline__ void group_publish(const float (&v)[P], int t, float* red) {
  if constexpr (P >= TPF) {
    constexpr int C = P / TPF;
#pragma unroll
    for (int i = 0; i < C; ++i) red[t * C + i] = v[i];
  } else {
    constexpr int G = TPF / P;
    if ((t % G) == 0) red[t / G] = v[0];
  }
}

template <int DMAX, int RMAX, int TPF>
struct FrameQR {
  static_assert(TPF >= 2 && TPF <= 32 && (TPF & (TPF - 1)) == 0, "TPF must be a power of two in [2, 32]");
  static_assert(DMAX % TPF == 0, "DMAX must be a multiple of TPF");
  static_assert(RMAX >= 1 && RMAX <= 32 && (RMAX & (RMAX - 1)) == 0, "RMAX must be a power of two <= 32");
  static_assert(RMAX <= DMAX, "thin QR needs r <= d");
  static constexpr int RPT = DMAX / TPF;

  // Per-group shared scratch: reduction totals and pivot row (double-buffered by
  // step parity) and the tau of every reflector.
  struct Smem {
    float red[2][RMAX];
    float piv[2][RMAX];
    float tau[RMAX];
  };

  // true when the row of slot s of group lane t is > K (folds at compile time
  // for every slot that lies entirely above or below K).
  template <int K>
  __device__ static __forceinline__ bool below(int s, int t) {
    if (s * TPF > K) return true;
    if (s * TPF + TPF - 1 <= K) return false;
    return t + s * TPF > K;
  }
  template <int K>
  __device__ static __forceinline__ bool at(int s, int t) {
    if (K < s * TPF || K >= s * TPF + TPF) return false;
    return t == K - s * TPF;
  }

  // Partial sums over this lane's rows (> K) of the values [I0, I0+N) of the
  // step-K list {c_{K+1}, ..., c_{RMAX-1}, xnorm^2}, reduced across the group and
  // published to red[I0 ..).  Chunks of <= 16 values keep the live partials small;
  // the butterfly costs about the same number of shuffles either way.
  template <int K, int I0, int N>
  __device__ static __forceinline__ void gram_chunk(const float (&a)[RPT][RMAX], int t, float* red) {
    constexpr int NC = RMAX - K - 1;
    constexpr int P = pow2_ceil(N);
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = 0.f;
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const float x = below<K>(s, t) ? a[s][K] : 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (I0 + i < NC) {
          v[i] = fmaf(x, a[s][K + 1 + I0 + i], v[i]);
        } else {
          v[i] = fmaf(x, x, v[i]);
        }
      }
    }
    group_reduce_scatter<P, TPF>(v, t);
    group_publish<P, TPF>(v, t, red + I0);
  }

  // Same for the orgqr step: values [I0, I0+N) of {v^T Q[:, K+1], ..., v^T Q[:, RMAX-1]}.
  template <int K, int I0, int N>
  __device__ static __forceinline__ void vq_chunk(const float (&a)[RPT][RMAX], int t, float* red) {
    constexpr int P = pow2_ceil(N);
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = 0.f;
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const float vi = below<K>(s, t) ? a[s][K] : 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = fmaf(vi, a[s][K + 1 + I0 + i], v[i]);
    }
    group_reduce_scatter<P, TPF>(v, t);
    group_publish<P, TPF>(v, t, red + I0);
  }

  static constexpr int kChunk = 16;

  template <int K>
  __device__ static __forceinline__ void geqrf_step(float (&a)[RPT][RMAX], int t, Smem& sm, uint32_t& rneg) {
    constexpr int NC = RMAX - K - 1;  // trailing columns
    constexpr int NV = NC + 1;        // c_{K+1..RMAX-1}, xnorm^2
    constexpr int NCH = (NV + kChunk - 1) / kChunk;
    float* red = sm.red[K & 1];
    float* piv = sm.piv[K & 1];

    // pivot row K: piv[j] = A[K, K+1+j], piv[NC] = A[K, K]
    constexpr int SK = K / TPF;
    if (t == K % TPF) {
#pragma unroll
      for (int j = 0; j < NC; ++j) piv[j] = a[SK][K + 1 + j];
      piv[NC] = a[SK][K];
    }
    static_for<0, NCH>([&](auto cc) {
      constexpr int C = decltype(cc)::value;
      constexpr int I0 = C * kChunk;
      constexpr int N = (NV - I0) < kChunk ? (NV - I0) : kChunk;
      gram_chunk<K, I0, N>(a, t, red);
    });
    __syncwarp();

    const float alpha = piv[NC];
    const float xn2 = red[NC];
    float beta, tau, scal;
    if (xn2 == 0.f) {
      beta = alpha;
      tau = 0.f;
      scal = 0.f;
    } else {
      const float sigma = sqrtf(fmaf(alpha, alpha, xn2));
      beta = alpha >= 0.f ? -sigma : sigma;
      tau = (beta - alpha) / beta;
      scal = 1.f / (alpha - beta);
    }
    rneg |= (beta < 0.f ? 1u : 0u) << K;
    if (t == 0) sm.tau[K] = tau;

#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const float w = fmaf(scal, red[j], piv[j]);  // v^T A[K:, K+1+j]
      const float tw = tau * w;
      const float g = tw * scal;
#pragma unroll
      for (int s = 0; s < RPT; ++s) {
        if (below<K>(s, t)) {
          a[s][K + 1 + j] = fmaf(-g, a[s][K], a[s][K + 1 + j]);
        } else if (at<K>(s, t)) {
          a[s][K + 1 + j] -= tw;
        }
      }
    }
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      if (below<K>(s, t)) {
        a[s][K] *= scal;  // v_i, i > K
      } else if (at<K>(s, t)) {
        a[s][K] = beta;   // R_KK
      }
    }
  }

  // Backward accumulation of the explicit thin Q (sorg2r order), in place.
  template <int K>
  __device__ static __forceinline__ void orgqr_step(float (&a)[RPT][RMAX], int t, Smem& sm) {
    constexpr int NC = RMAX - K - 1;
    const float tau = sm.tau[K];
    if constexpr (NC > 0) {
      constexpr int NCH = (NC + kChunk - 1) / kChunk;
      float* red = sm.red[K & 1];
      static_for<0, NCH>([&](auto cc) {
        constexpr int C = decltype(cc)::value;
        constexpr int I0 = C * kChunk;
        constexpr int N = (NC - I0) < kChunk ? (NC - I0) : kChunk;
        vq_chunk<K, I0, N>(a, t, red);
      });
      __syncwarp();
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const float tp = tau * red[j];
#pragma unroll
        for (int s = 0; s < RPT; ++s) {
          if (below<K>(s, t)) {
            a[s][K + 1 + j] = fmaf(-tp, a[s][K], a[s][K + 1 + j]);
          } else if (at<K>(s, t)) {
            a[s][K + 1 + j] = -tp;  // row K of column K+1+j was zeroed at its own step
          }
        }
      }
    }
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      if (below<K>(s, t)) {
        a[s][K] *= -tau;
      } else if (at<K>(s, t)) {
        a[s][K] = 1.f - tau;
      } else {
        a[s][K] = 0.f;  // rows < K: discard R
      }
    }
  }

  // Bitmask of columns whose sign must flip under the reference's
  // first-significant-entry rule (gfst.py:35-46): first row with |q| > eps_sign,
  // negative -> flip.  cols_mask selects the real (unpadded) columns.
  __device__ static __forceinline__ uint32_t first_significant_flips(const float (&a)[RPT][RMAX], int lane,
                                                                     float eps_sign, uint32_t cols_mask) {
    const int gbase = (lane / TPF) * TPF;
    const uint32_t gmask = TPF == 32 ? 0xffffffffu : ((1u << TPF) - 1u);
    uint32_t flip = 0u, found = 0u;
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
#pragma unroll
      for (int j = 0; j < RMAX; ++j) {
        const uint32_t sig = (__ballot_sync(0xffffffffu, fabsf(a[s][j]) > eps_sign) >> gbase) & gmask;
        const uint32_t neg = (__ballot_sync(0xffffffffu, a[s][j] < 0.f) >> gbase) & gmask;
        if (!((found >> j) & 1u) && sig != 0u) {
          found |= 1u << j;
          flip |= ((neg >> (__ffs(sig) - 1)) & 1u) << j;
        }
      }
      if (!__any_sync(0xffffffffu, (found & cols_mask) != cols_mask)) break;
    }
    return flip;
  }

  // Full thin QR in place: a <- sign-fixed Q.
  __device__ static __forceinline__ void qr(float (&a)[RPT][RMAX], int lane, int t, Smem& sm, float eps_sign,
                                            int sign_mode, uint32_t cols_mask) {
    uint32_t rneg = 0u;
    static_for<0, RMAX>([&](auto kc) { geqrf_step<decltype(kc)::value>(a, t, sm, rneg); });
    // tau[RMAX-1] is written by one lane in the last step, which has no
    // reduction (and so no __syncwarp) after it; order it before any reader.
    __syncwarp();
    static_for_down<0, RMAX>([&](auto kc) { orgqr_step<decltype(kc)::value>(a, t, sm); });
    const uint32_t flip = (sign_mode == GFST_SIGN_R_DIAG_POSITIVE)
                              ? rneg
                              : first_significant_flips(a, lane, eps_sign, cols_mask);
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
#pragma unroll
      for (int j = 0; j < RMAX; ++j) {
        if ((flip >> j) & 1u) a[s][j] = -a[s][j];
      }
    }
  }

  // Load a dense [d, r] frame (zero padded to DMAX x RMAX).
  __device__ static __forceinline__ void load(float (&a)[RPT][RMAX], const float* __restrict__ src, int t, int d,
                                              int r, bool valid, bool vec4) {
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const int row = t + s * TPF;
      const bool ok = valid && row < d;
      if (vec4) {
        // r == RMAX, RMAX % 4 == 0, src 16-byte aligned
#pragma unroll
        for (int c = 0; c < RMAX / 4; ++c) {
          float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
          if (ok) q = __ldg(reinterpret_cast<const float4*>(src + (size_t)row * RMAX) + c);
          a[s][4 * c + 0] = q.x;
          a[s][4 * c + 1] = q.y;
          a[s][4 * c + 2] = q.z;
          a[s][4 * c + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < RMAX; ++j) a[s][j] = (ok && j < r) ? __ldg(src + (size_t)row * r + j) : 0.f;
      }
    }
  }

  __device__ static __forceinline__ void store(const float (&a)[RPT][RMAX], float* __restrict__ dst, int t, int d,
                                               int r, bool valid, bool vec4) {
#pragma unroll
    for (int s = 0; s < RPT; ++s) {
      const int row = t + s * TPF;
      if (!(valid && row < d)) continue;
      if (vec4) {
#pragma unroll
        for (int c = 0; c < RMAX / 4; ++c) {
          reinterpret_cast<float4*>(dst + (size_t)row * RMAX)[c] =
              make_float4(a[s][4 * c + 0], a[s][4 * c + 1], a[s][4 * c + 2], a[s][4 * c + 3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < RMAX; ++j)
          if (j < r) dst[(size_t)row * r + j] = a[s][j];
      }
    }
  }
};

}  // namespace gfst
