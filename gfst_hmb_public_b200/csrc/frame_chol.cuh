// Cholesky QR, twice (CholeskyQR2), of one d x r fp32 frame per warp, for the
// streaming pass, with the Householder factorisation of frame_qr.cuh as the
// fallback for frames whose Gram matrix is not safely positive definite.
//
// Why: the streaming frames are C = beta*U + A B^T with U orthonormal and a
// rank-m update, so C is well conditioned.  Householder QR spends 2r dependent
// reflector steps (each a column norm and r dot products reduced across lanes)
// per token; CholeskyQR2 replaces them with two Gram products (independent
// dot products), an r x r Cholesky and a triangular solve per pass:
//     pass:  G = C^T C,  G = R^T R (Cholesky),  C <- C R^{-1}
// The first pass only has to make C well conditioned, so its Gram runs on
// the tensor cores in TF32 (mma.sync, FP32 accumulation; C R1^{-1} comes out
// orthonormal to about 1e-3); its solve is FP32, so C R1^{-1} keeps the
// column spans of C to FP32 rounding.  The second pass is FP32 throughout and
// sets the result: the thin Q of the QR of the input with a positive R
// diagonal -- the matrix Householder QR with the R-diagonal-positive rule
// produces (the factorisation is unique for a full-rank input) -- after which
// the reference's first-significant-entry sign rule (gfst.py:35-46) is
// applied when asked.  A pivot R_jj^2 below kPivotTol * G_jj (column j within
// about 6 degrees of the span of the columns before it), a non-finite pivot
// or a zero column sends the frame through Householder instead, on the input
// of the pass that failed (the second pass's input has the same Q).
//
// Layout: block rows.  Lane l owns rows RPL*l .. RPL*l + RPL - 1 of every
// column as float2 row pairs (packed fma.f32x2 in the update and the solve).
// The Gram products read a column-major copy in shared memory whose 4-row
// chunks are XOR-swizzled per column (conflict-free tile and fragment loads).
#pragma once

#include <type_traits>

#include "frame_qr.cuh"

namespace gfst {

constexpr float kPivotTol = 1e-2f;
constexpr float kFirstOrderTol = 3e-4f;  // |E| bound for the first-order second pass

template <int DMAX, int RMAX>
struct FrameChol {
  static_assert(DMAX == 64 || DMAX == 128, "block rows: 2 or 4 rows per lane");
  static_assert(RMAX == 16 || RMAX == 32, "Gram tiles are spread over 8 x 4 lanes");
  static constexpr int RPL = DMAX / 32;  // rows per lane
  static constexpr int RPP = RPL / 2;    // row pairs per lane
  static constexpr int TI = RMAX / 8;    // Gram tile rows per lane
  static constexpr int TJ = RMAX / 4;    // Gram tile columns per lane
  static constexpr int GS = RMAX + 4;    // Gram row stride (floats)
  static constexpr int NCH = DMAX / 4;   // 4-row chunks per column
  using Frame = float2[RPP][RMAX];       // f[p][c] = rows (RPL*lane + 2p, +1) of column c
  using HH = FrameQR<DMAX, RMAX, 8, 4>;  // Householder fallback, one frame per warp

  struct __align__(16) Smem {
    float mt[RMAX * DMAX];  // column-major copy of the pass input
    union {
      float g[RMAX * GS];   // Gram (row-major); then R row-major: 1/R[k][k] on the
                            // diagonal, -R[k][j] right of it
      typename HH::Smem hh; // fallback scratch
    };
  };

  // XOR swizzle of the 4-row chunks of column `col`, a bijection on the three
  // low column bits both for the FP32 Gram's row-tile loads (columns
  // TI*bi + ii over bi) and for the tensor-core fragment loads (columns
  // 8q + g over g), so either lands a quarter warp on distinct bank quads.
  __device__ static __forceinline__ int sw(int col) {
    if constexpr (RMAX == 32) return ((col ^ (col >> 3)) & 3) | (col & 4);
    else return (col & 6) | ((col ^ (col >> 3)) & 1);
  }
  __device__ static __forceinline__ int mt_at(int col, int row) {
    return col * DMAX + 4 * ((row >> 2) ^ sw(col)) + (row & 3);
  }

  __device__ static __forceinline__ void write_mt(const Frame& f, Smem& sm, int lane) {
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      if constexpr (RPL == 4) {
        *reinterpret_cast<float4*>(sm.mt + c * DMAX + 4 * (lane ^ sw(c))) =
            make_float4(f[0][c].x, f[0][c].y, f[1][c].x, f[1][c].y);
      } else {
        *reinterpret_cast<float2*>(sm.mt + c * DMAX + 4 * ((lane >> 1) ^ sw(c)) + 2 * (lane & 1)) = f[0][c];
      }
    }
  }
  __device__ static __forceinline__ void read_mt(Frame& f, const Smem& sm, int lane) {
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      if constexpr (RPL == 4) {
        const float4 v = *reinterpret_cast<const float4*>(sm.mt + c * DMAX + 4 * (lane ^ sw(c)));
        f[0][c] = make_float2(v.x, v.y);
        f[1][c] = make_float2(v.z, v.w);
      } else {
        f[0][c] = *reinterpret_cast<const float2*>(sm.mt + c * DMAX + 4 * ((lane >> 1) ^ sw(c)) + 2 * (lane & 1));
      }
    }
  }

  // G = C^T C on the tensor cores (mma.sync m16n8k8, TF32 operands): each
  // value x is split as hi + lo (hi = x rounded to TF32, lo = the rest rounded
  // to TF32, |x - hi - lo| <= 2^-22 |x|) and every product is taken as
  // lo*hi + hi*lo + hi*hi.  Each k-step (8 frame rows) sums its products in a
  // fresh accumulator, added to the running sums in FP32, so the tensor
  // cores' internal rounding applies to one step's partial sum only: G comes
  // out to a few 1e-7 relative, like an FP32 dot product.
  // A = C^T rows (frame columns) 16*mt + g and 16*mt + 8 + g, B = frame columns
  // 8*nt + g, K = frame rows.  Tiles (mt, nt) on or above the diagonal blocks
  // are computed and stored transposed (gT[n][m] = G[m][n]): row j of the
  // area then holds G[i][j] for every i <= j, which is all the Cholesky of
  // column j and the first-order correction read.
  __device__ static __forceinline__ uint32_t to_tf32(float x) {
    uint32_t y;
    asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(y) : "f"(x));
    return y;
  }
  __device__ static __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = to_tf32(x);
    lo = to_tf32(x - __uint_as_float(hi));
  }
  __device__ static __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ static __forceinline__ void gram(Smem& sm, int lane) {
    constexpr int NQ = RMAX / 8;            // frame-column groups of 8
    constexpr int NT = RMAX == 32 ? 6 : 2;  // tiles computed
    constexpr int MQ[6] = {0, 0, 0, 0, 2, 2}, NQI[6] = {0, 1, 2, 3, 2, 3};
    const int g = lane >> 2, t = lane & 3;
    int off[NQ], swz[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      off[q] = (8 * q + g) * DMAX + t;
      swz[q] = sw(8 * q + g);
    }
    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll 2
    for (int ks = 0; ks < NCH / 2; ++ks) {
      uint32_t h0[NQ], l0[NQ], h1[NQ], l1[NQ];  // frame column 8q+g at rows 8ks+t and 8ks+4+t
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        split_tf32(sm.mt[off[q] + 4 * ((2 * ks) ^ swz[q])], h0[q], l0[q]);
        split_tf32(sm.mt[off[q] + 4 * ((2 * ks + 1) ^ swz[q])], h1[q], l1[q]);
      }
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int a = MQ[i], b = NQI[i];
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tf32(c, l0[a], l0[a + 1], l1[a], l1[a + 1], h0[b], h1[b]);
        mma_tf32(c, h0[a], h0[a + 1], h1[a], h1[a + 1], l0[b], l1[b]);
        mma_tf32(c, h0[a], h0[a + 1], h1[a], h1[a + 1], h0[b], h1[b]);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] += c[e];
      }
    }
    // D fragment: (g, 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1) of each 16 x 8 tile
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int m0 = 8 * MQ[i] + g, n0 = 8 * NQI[i] + 2 * t;
      sm.g[n0 * GS + m0] = acc[i][0];
      sm.g[(n0 + 1) * GS + m0] = acc[i][1];
      sm.g[n0 * GS + m0 + 8] = acc[i][2];
      sm.g[(n0 + 1) * GS + m0 + 8] = acc[i][3];
    }
  }

  // Cholesky G = R^T R, lane j holding column j of the Schur complement
  // (G is symmetric: column j = row j).  Row k of R goes to row k of the Gram
  // area as it is produced (1/R[k][k], then -R[k][j]); the trailing update
  // reads it back.  Columns >= r are unit columns (R = I there; the padded
  // input columns are zero).  With RMAX = 16 lanes 16..31 only follow along.
  // Returns this lane's pivot test.
  __device__ static __forceinline__ bool cholesky(Smem& sm, int lane, int r) {
    const bool own = lane < RMAX;
    const int row = own ? lane : 0;
    float g[RMAX];
#pragma unroll
    for (int q = 0; q < RMAX; q += 4) {
      const float4 v = *reinterpret_cast<const float4*>(sm.g + row * GS + q);
      g[q] = v.x;
      g[q + 1] = v.y;
      g[q + 2] = v.z;
      g[q + 3] = v.w;
    }
    float gjj = sm.g[row * GS + row];
    __syncwarp();  // every row read before R overwrites the area
    if (lane >= r) {
#pragma unroll
      for (int i = 0; i < RMAX; ++i) g[i] = (i == lane) ? 1.f : 0.f;
      gjj = 1.f;
    }
    float piv = 1.f, dn = 0.f;
#pragma unroll
    for (int k = 0; k < RMAX; ++k) {
      // pivot of step k: lane k's diagonal, updated through step k - 1 (its own
      // update, computed one step ahead in dn)
      const float dk = __shfl_sync(0xffffffffu, k == 0 ? g[0] : dn, k);
      const float inv = rsqrtf(dk);
      float rkj = g[k] * inv;
      if (lane == k) piv = dk;
      if (lane < k) rkj = 0.f;
      if (own) sm.g[k * GS + lane] = (lane == k) ? inv : -rkj;
      if (k + 1 < RMAX) {
        dn = fmaf(-rkj, rkj, g[k + 1]);
        const float rn = __shfl_sync(0xffffffffu, rkj, k + 1);
        g[k + 1] = fmaf(-rn, rkj, g[k + 1]);
        __syncwarp();
        const int Q0 = ((k + 2) / 4) * 4;
#pragma unroll
        for (int q = Q0; q < RMAX; q += 4) {
          const float4 v = *reinterpret_cast<const float4*>(sm.g + k * GS + q);  // -R[k][q..q+3]
          if (q + 0 >= k + 2) g[q + 0] = fmaf(v.x, rkj, g[q + 0]);
          if (q + 1 >= k + 2) g[q + 1] = fmaf(v.y, rkj, g[q + 1]);
          if (q + 2 >= k + 2) g[q + 2] = fmaf(v.z, rkj, g[q + 2]);
          if (q + 3 >= k + 2) g[q + 3] = fmaf(v.w, rkj, g[q + 3]);
        }
      }
    }
    // NaN fails every comparison; an infinite Gram gives a NaN or infinite pivot
    return gjj > 0.f && piv > kPivotTol * gjj && piv <= 3.0e38f;
  }

  // f <- f R^{-1}, right-looking: column i is finished (times 1/R[i][i]), then
  // removed from every later column -- the later columns' updates are
  // independent of one another.
  __device__ static __forceinline__ void solve(Frame& f, const Smem& sm) {
    static_for<0, RMAX>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      constexpr int Q0 = (i / 4) * 4;
      float rr[RMAX];
#pragma unroll
      for (int q = Q0; q < RMAX; q += 4) {
        const float4 v = *reinterpret_cast<const float4*>(sm.g + i * GS + q);
        rr[q] = v.x;
        rr[q + 1] = v.y;
        rr[q + 2] = v.z;
        rr[q + 3] = v.w;
      }
#pragma unroll
      for (int p = 0; p < RPP; ++p) f[p][i] = __fmul2_rn(f[p][i], make_float2(rr[i], rr[i]));
#pragma unroll
      for (int j = i + 1; j < RMAX; ++j)
#pragma unroll
        for (int p = 0; p < RPP; ++p) f[p][j] = ffma2(f[p][i], make_float2(rr[j], rr[j]), f[p][j]);
    });
  }

  // Largest |E_ij| (i <= j, over this lane's column j < r) of E = G - I,
  // reduced over the warp (float bits order like the values; NaN is larger).
  __device__ static __forceinline__ float gram_defect(const Smem& sm, int lane, int r) {
    float e = 0.f;
    if (lane < RMAX && lane < r) {
#pragma unroll
      for (int q = 0; q < RMAX; q += 4) {
        const float4 v = *reinterpret_cast<const float4*>(sm.g + lane * GS + q);
        const float w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = q + u;
          const float x = fabsf(i == lane ? w[u] - 1.f : w[u]);
          if (i <= lane) e = (x > e || x != x) ? x : e;
        }
      }
    }
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(e)));
  }

  // Second pass on a nearly orthonormal f (G = f^T f = I + E, |E| small):
  // chol(I + E) = I + F + O(E^2) with F = triu(E) - diag(E)/2, so
  // f <- f (I - F): column j becomes f_j (1 - E_jj/2) - sum_{i<j} f_i E_ij.
  // Columns run from the last down (each reads only columns left of it), and
  // the columns are independent of one another.
  __device__ static __forceinline__ void correct(Frame& f, const Smem& sm) {
    static_for_down<0, RMAX>([&](auto jc) {
      constexpr int j = decltype(jc)::value;
      float e[((j + 4) / 4) * 4];
#pragma unroll
      for (int q = 0; q <= j; q += 4) {
        const float4 v = *reinterpret_cast<const float4*>(sm.g + j * GS + q);
        e[q] = v.x;
        e[q + 1] = v.y;
        e[q + 2] = v.z;
        e[q + 3] = v.w;
      }
      const float fac = fmaf(-0.5f, e[j] - 1.f, 1.f);
#pragma unroll
      for (int p = 0; p < RPP; ++p) {
        float2 s = __fmul2_rn(f[p][j], make_float2(fac, fac));
#pragma unroll
        for (int i = 0; i < j; ++i) s = ffma2(f[p][i], make_float2(-e[i], -e[i]), s);
        f[p][j] = s;
      }
    });
  }

  // Householder QR (sign rule included) of the matrix held in mt -> f.
  __device__ static __forceinline__ void householder(Frame& f, Smem& sm, int lane, float eps_sign, int sign_mode,
                                                     int r) {
    const int rg = lane & 7, cg = lane >> 3;
    typename HH::Frame a;
#pragma unroll
    for (int s = 0; s < DMAX / 8; ++s)
#pragma unroll
      for (int c = 0; c < RMAX / 4; ++c) HH::set(a, s, c, sm.mt[mt_at(cg + 4 * c, rg + 8 * s)]);
    __syncwarp();
    HH::qr(a, lane, lane, sm.hh, eps_sign, sign_mode, r);
#pragma unroll
    for (int s = 0; s < DMAX / 8; ++s)
#pragma unroll
      for (int c = 0; c < RMAX / 4; ++c) sm.mt[mt_at(cg + 4 * c, rg + 8 * s)] = HH::get(a, s, c);
    __syncwarp();
    read_mt(f, sm, lane);
  }

  // Reference sign rule on block rows: the first row (in row order) of each
  // column with |q| > eps_sign decides; negative -> negate the column.
  __device__ static __forceinline__ void first_significant(Frame& f, float eps_sign) {
    uint32_t hs = 0u, ng = 0u;
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      bool found = false, neg = false;
#pragma unroll
      for (int q = 0; q < RPL; ++q) {
        const float v = (q & 1) ? f[q >> 1][c].y : f[q >> 1][c].x;
        if (!found && fabsf(v) > eps_sign) {
          found = true;
          neg = v < 0.f;
        }
      }
      hs |= (found ? 1u : 0u) << c;
      ng |= (neg ? 1u : 0u) << c;
    }
    uint32_t flip = 0u;
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      const uint32_t b = __ballot_sync(0xffffffffu, (hs >> c) & 1u);
      const uint32_t src_ng = __shfl_sync(0xffffffffu, ng, b ? __ffs(b) - 1 : 0);
      if (b) flip |= ((src_ng >> c) & 1u) << c;
    }
#pragma unroll
    for (int p = 0; p < RPP; ++p)
#pragma unroll
      for (int c = 0; c < RMAX; ++c)
        if ((flip >> c) & 1u) f[p][c] = make_float2(-f[p][c].x, -f[p][c].y);
  }

  // In place: f <- sign-fixed thin Q.  Pass 1: Gram, Cholesky, solve.  Pass 2
  // on the nearly orthonormal result: Gram, then the first-order correction
  // when |E| <= kFirstOrderTol (its error is O(|E|^2)), else a full Cholesky
  // pass.  A failed pivot test sends the pass's input through Householder.
  __device__ static __forceinline__ void qr(Frame& f, Smem& sm, int lane, float eps_sign, int sign_mode, int r) {
#pragma unroll 1
    for (int ps = 0; ps < 2; ++ps) {  // one copy of the pass code
      __syncwarp();  // the previous reads of mt and the Gram area are done
      write_mt(f, sm, lane);
      __syncwarp();
      gram(sm, lane);
      __syncwarp();
      if (ps == 1 && gram_defect(sm, lane, r) <= kFirstOrderTol) {
        correct(f, sm);
        break;
      }
      const bool ok = __all_sync(0xffffffffu, cholesky(sm, lane, r));
      __syncwarp();
      if (!ok) {
        householder(f, sm, lane, eps_sign, sign_mode, r);
        return;
      }
      read_mt(f, sm, lane);
      solve(f, sm);
    }
    // R = R2 R1 has a positive diagonal: the R-diagonal rule needs no flips
    if (sign_mode == GFST_SIGN_FIRST_SIGNIFICANT) first_significant(f, eps_sign);
  }

  // ---- global memory and the rank-m update (block rows) ------------------
  __device__ static __forceinline__ void load(Frame& f, const float* __restrict__ src, int lane, int d, int r,
                                              bool valid, bool vec4) {
#pragma unroll
    for (int p = 0; p < RPP; ++p) {
      const int r0 = RPL * lane + 2 * p, r1 = r0 + 1;
      if (vec4 && r == RMAX) {
#pragma unroll
        for (int c = 0; c < RMAX; c += 4) {
          float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
          if (valid && r0 < d) x0 = __ldg(reinterpret_cast<const float4*>(src + (size_t)r0 * RMAX + c));
          if (valid && r1 < d) x1 = __ldg(reinterpret_cast<const float4*>(src + (size_t)r1 * RMAX + c));
          f[p][c] = make_float2(x0.x, x1.x);
          f[p][c + 1] = make_float2(x0.y, x1.y);
          f[p][c + 2] = make_float2(x0.z, x1.z);
          f[p][c + 3] = make_float2(x0.w, x1.w);
        }
      } else {
#pragma unroll
        for (int c = 0; c < RMAX; ++c) {
          const bool cv = valid && c < r;
          f[p][c] = make_float2(cv && r0 < d ? __ldg(src + (size_t)r0 * r + c) : 0.f,
                                cv && r1 < d ? __ldg(src + (size_t)r1 * r + c) : 0.f);
        }
      }
    }
  }

  __device__ static __forceinline__ void store(const Frame& f, float* __restrict__ dst, int lane, int d, int r,
                                               bool valid, bool vec4) {
    if (!valid) return;
#pragma unroll
    for (int p = 0; p < RPP; ++p) {
      const int r0 = RPL * lane + 2 * p, r1 = r0 + 1;
      if (vec4 && r == RMAX) {
#pragma unroll
        for (int c = 0; c < RMAX; c += 4) {
          if (r0 < d)
            *reinterpret_cast<float4*>(dst + (size_t)r0 * RMAX + c) =
                make_float4(f[p][c].x, f[p][c + 1].x, f[p][c + 2].x, f[p][c + 3].x);
          if (r1 < d)
            *reinterpret_cast<float4*>(dst + (size_t)r1 * RMAX + c) =
                make_float4(f[p][c].y, f[p][c + 1].y, f[p][c + 2].y, f[p][c + 3].y);
        }
      } else {
#pragma unroll
        for (int c = 0; c < RMAX; ++c) {
          if (c >= r) continue;
          if (r0 < d) dst[(size_t)r0 * r + c] = f[p][c].x;
          if (r1 < d) dst[(size_t)r1 * r + c] = f[p][c].y;
        }
      }
    }
  }

  __device__ static __forceinline__ void scale(Frame& f, float beta) {
    const float2 b2 = make_float2(beta, beta);
#pragma unroll
    for (int p = 0; p < RPP; ++p)
#pragma unroll
      for (int c = 0; c < RMAX; ++c) f[p][c] = __fmul2_rn(f[p][c], b2);
  }

  // f += A B^T, A [d, m] and B [r, m] row-major (shared memory).  m = 2, 4, 8:
  // one vector load per row of A and of B per group of <= 4 update columns.
  template <int MV>
  __device__ static __forceinline__ void rank_update_vec(Frame& f, const float* A, const float* B, int lane, int d,
                                                         int r, int m, int m0) {
    using V = typename std::conditional<MV == 4, float4, float2>::type;
    float av[RPL][MV];
#pragma unroll
    for (int q = 0; q < RPL; ++q) {
      const int row = RPL * lane + q;
      V v{};
      if (row < d) v = *reinterpret_cast<const V*>(A + row * m + m0);
      const float* pv = reinterpret_cast<const float*>(&v);
#pragma unroll
      for (int u = 0; u < MV; ++u) av[q][u] = pv[u];
    }
#pragma unroll
    for (int c = 0; c < RMAX; ++c) {
      V v{};
      if (c < r) v = *reinterpret_cast<const V*>(B + c * m + m0);
      const float* pb = reinterpret_cast<const float*>(&v);
#pragma unroll
      for (int p = 0; p < RPP; ++p) {
        float2 acc = f[p][c];
#pragma unroll
        for (int u = 0; u < MV; ++u)
          acc = ffma2(make_float2(av[2 * p][u], av[2 * p + 1][u]), make_float2(pb[u], pb[u]), acc);
        f[p][c] = acc;
      }
    }
  }

  __device__ static __forceinline__ void rank_update(Frame& f, const float* A, const float* B, int lane, int d, int r,
                                                     int m) {
    if (m % 4 == 0) {  // rows of A and B are 16-byte aligned in the stage
      for (int m0 = 0; m0 < m; m0 += 4) rank_update_vec<4>(f, A, B, lane, d, r, m, m0);
      return;
    }
    if (m == 2) {
      rank_update_vec<2>(f, A, B, lane, d, r, m, 0);
      return;
    }
    for (int mm = 0; mm < m; ++mm) {
      float2 a2[RPP];
#pragma unroll
      for (int p = 0; p < RPP; ++p) {
        const int r0 = RPL * lane + 2 * p, r1 = r0 + 1;
        a2[p] = make_float2(r0 < d ? A[r0 * m + mm] : 0.f, r1 < d ? A[r1 * m + mm] : 0.f);
      }
#pragma unroll
      for (int c = 0; c < RMAX; ++c) {
        const float b = c < r ? B[c * m + mm] : 0.f;
        const float2 b2 = make_float2(b, b);
#pragma unroll
        for (int p = 0; p < RPP; ++p) f[p][c] = ffma2(a2[p], b2, f[p][c]);
      }
    }
  }
};

}  // namespace gfst
