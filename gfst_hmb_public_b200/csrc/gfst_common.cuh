// Shared helpers for the GFST-HMB sm_100a kernels: status plumbing, compile-time
// loops, bf16 conversion and small warp utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "gfst_b200.h"

namespace gfst {

// ---------------------------------------------------------------------------
// host side: last-error text (thread local) and launch checks
// ---------------------------------------------------------------------------
void set_last_error(const char* fmt, ...);
int check_launch(const char* what);

#define GFST_REQUIRE(cond, code, ...)            \
  do {                                           \
    if (!(cond)) {                               \
      ::gfst::set_last_error(__VA_ARGS__);       \
      return (code);                             \
    }                                            \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// sticky device error words
// ---------------------------------------------------------------------------
// One word per translation unit: kernels record a status with atomicExch; the
// host reads it (and clears it when asked) in one atomic step through a
// one-thread kernel on the legacy default stream, whose result lands in a
// snapshot word that the following cudaMemcpyFromSymbol reads.  Callers
// synchronise the device first (gfst_check_device_errors does), so the word
// holds every report of work enqueued before the call.
#define GFST_DEFINE_ERROR_WORD(word, reader, what)                                                         \
  __device__ unsigned int word = 0;                                                                       \
  __device__ unsigned int word##_snapshot = 0;                                                            \
  __global__ void word##_take(int clear) {                                                                \
    word##_snapshot = clear ? atomicExch(&word, 0u) : atomicOr(&word, 0u);                                \
  }                                                                                                        \
  int reader(int clear, unsigned int* value) {                                                             \
    word##_take<<<1, 1, 0, cudaStreamLegacy>>>(clear);                                                     \
    cudaError_t e = cudaGetLastError();                                                                    \
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "reading the " what " error word: %s",                \
                 cudaGetErrorString(e));                                                                   \
    unsigned int v = 0;                                                                                    \
    e = cudaMemcpyFromSymbol(&v, word##_snapshot, sizeof(v));                                              \
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "reading the " what " error word: %s",                \
                 cudaGetErrorString(e));                                                                   \
    *value = v;                                                                                            \
    return GFST_OK;                                                                                        \
  }

// ---------------------------------------------------------------------------
// compile-time helpers usable in device code
// ---------------------------------------------------------------------------
template <int V>
struct IC {
  static constexpr int value = V;
};

// f(IC<B>), f(IC<B+1>), ..., f(IC<E-1>)
template <int B, int E, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (B < E) {
    f(IC<B>{});
    static_for<B + 1, E>(f);
  }
}

// f(IC<E-1>), f(IC<E-2>), ..., f(IC<B>)
template <int B, int E, typename F>
__device__ __forceinline__ void static_for_down(F&& f) {
  if constexpr (B < E) {
    f(IC<E - 1>{});
    static_for_down<B, E - 1>(f);
  }
}

__host__ __device__ constexpr int pow2_ceil(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

__host__ __device__ constexpr int ilog2(int n) {
  int l = 0;
  while ((1 << l) < n) ++l;
  return l;
}

// ---------------------------------------------------------------------------
// bf16 <-> fp32 (exact widening; narrowing rounds to nearest even)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }

// (score, index) total order used by every selection in this library:
// higher score first; equal scores -> lower index first.  NaN scores rank last.
__device__ __forceinline__ bool better(float sa, int ia, float sb, int ib) {
  if (sa > sb) return true;
  if (sa < sb) return false;
  if (sa == sb) return ia < ib;
  // at least one NaN: a non-NaN beats NaN, two NaNs compare by index
  const bool na = sa != sa, nb = sb != sb;
  if (na != nb) return nb;
  return ia < ib;
}

// ---------------------------------------------------------------------------
// warp-subgroup reductions
// ---------------------------------------------------------------------------
// Sum v[0..P) over the G lanes of a lane subgroup (subgroup lane index t; the
// subgroup is G consecutive lanes, G a power of two).  On return: if P >= G,
// v[0..P/G) holds the totals of values [t*P/G, (t+1)*P/G); if P < G, v[0]
// holds the total of value t/(G/P).
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

template <int P, int G>
__device__ __forceinline__ void subgroup_reduce_scatter(float (&v)[P], int t) {
  ReduceScatter<P, G / 2, P>::run(v, t);
}

// Write the totals left by subgroup_reduce_scatter to red[0..P).
template <int P, int G>
__device__ __forceinline__ void subgroup_publish(const float (&v)[P], int t, float* red) {
  if constexpr (P >= G) {
    constexpr int C = P / G;
#pragma unroll
    for (int i = 0; i < C; ++i) red[t * C + i] = v[i];
  } else {
    constexpr int Q = G / P;
    if ((t % Q) == 0) red[t / Q] = v[0];
  }
}

template <int G>
__device__ __forceinline__ float subgroup_allreduce(float x) {
#pragma unroll
  for (int o = G / 2; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

}  // namespace gfst
