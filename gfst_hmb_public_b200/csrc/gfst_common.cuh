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

}  // namespace gfst
