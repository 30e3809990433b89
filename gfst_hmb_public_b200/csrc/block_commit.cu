// Block commit: write an L-token block of keys / values into its slot of the
// block memory pool and store the block's summary key (mean of its keys).
//
// Reference (pkhairkh/gfst-hmb-public): the exact-token store commits a packed
// block every block_len tokens (src/gfst_hmb_mpuc/state.py:651-815) and the
// block summary is appended at the same boundary
// (src/gfst_hmb_mpuc/modeling.py:3482-3535).  The summary key here is the mean
// of the block's token keys.
//
// HBM-bound: every byte of K and V is read once and written once.  Key threads
// own a 16-byte column chunk of the block and walk its L rows in token order,
// so the fp32 sum is taken in token order (t = 0, 1, ..., L-1), divided by L and
// rounded once -- the same arithmetic as the CPU oracle, hence bit-identical.
#include "gfst_common.cuh"

namespace gfst {
namespace {

constexpr int kThreads = 128;

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
};

__device__ __forceinline__ void unpack(const uint4& v, float (&f)[4], float) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ void unpack(const uint4& v, float (&f)[8], __nv_bfloat16) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x);
  f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z);
  f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}
__device__ __forceinline__ uint4 pack(const float (&f)[4], float) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(f32_to_bf16(lo));
  const uint32_t h = __bfloat16_as_ushort(f32_to_bf16(hi));
  return l | (h << 16);
}
__device__ __forceinline__ uint4 pack(const float (&f)[8], __nv_bfloat16) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

// blockIdx.y == 0: keys + summary; each thread owns one 16-byte column chunk of
// one stream's block.  blockIdx.y == 1: plain copy of the value block.
template <typename T>
__global__ void __launch_bounds__(kThreads) block_commit_kernel(const T* __restrict__ K, const T* __restrict__ V,
                                                                T* __restrict__ pool_K, T* __restrict__ pool_V,
                                                                T* __restrict__ summary, int64_t n_streams,
                                                                int n_slots, int slot, int L, int d, int dv) {
  constexpr int N = Vec16<T>::N;
  if (blockIdx.y == 0) {
    const int chunks = d / N;
    const int64_t gid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (gid >= n_streams * chunks) return;
    const int64_t s = gid / chunks;
    const int c = (int)(gid % chunks);
    const uint4* src = reinterpret_cast<const uint4*>(K + (size_t)s * L * d) + c;
    uint4* dst = reinterpret_cast<uint4*>(pool_K + ((size_t)s * n_slots + slot) * L * d) + c;
    const int row_vecs = d / N;
    float acc[N];
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = 0.f;
    int t = 0;
    for (; t + 8 <= L; t += 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(src + (size_t)(t + u) * row_vecs);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        dst[(size_t)(t + u) * row_vecs] = v[u];
        float f[N];
        unpack(v[u], f, T());
#pragma unroll
        for (int i = 0; i < N; ++i) acc[i] += f[i];
      }
    }
    for (; t < L; ++t) {
      const uint4 v = __ldg(src + (size_t)t * row_vecs);
      dst[(size_t)t * row_vecs] = v;
      float f[N];
      unpack(v, f, T());
#pragma unroll
      for (int i = 0; i < N; ++i) acc[i] += f[i];
    }
    const float len = (float)L;
#pragma unroll
    for (int i = 0; i < N; ++i) acc[i] = acc[i] / len;
    reinterpret_cast<uint4*>(summary + ((size_t)s * n_slots + slot) * d)[c] = pack(acc, T());
  } else {
    const int64_t vecs_per_stream = (int64_t)L * dv / N;
    const int64_t total = n_streams * vecs_per_stream;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kThreads) {
      const int64_t s = i / vecs_per_stream;
      const int64_t o = i % vecs_per_stream;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(V + (size_t)s * L * dv) + o);
      reinterpret_cast<uint4*>(pool_V + ((size_t)s * n_slots + slot) * L * dv)[o] = v;
    }
  }
}

template <typename T>
int launch(const void* K, const void* V, void* pool_K, void* pool_V, void* summary, int64_t S, int n_slots,
           int slot, int L, int d, int dv, cudaStream_t stream) {
  constexpr int N = Vec16<T>::N;
  GFST_REQUIRE(d % N == 0 && (V == nullptr || dv % N == 0), GFST_ERR_ALIGN,
               "rows must be whole 16-byte chunks (d=%d dv=%d, %d elements per chunk)", d, dv, N);
  const int64_t key_threads = S * (d / N);
  const int64_t key_blocks = (key_threads + kThreads - 1) / kThreads;
  const int64_t val_vecs = V ? S * (int64_t)L * dv / N : 0;
  int64_t val_blocks = (val_vecs + kThreads - 1) / kThreads;
  if (val_blocks > 148 * 32) val_blocks = 148 * 32;
  const int64_t gx = key_blocks > val_blocks ? key_blocks : val_blocks;
  GFST_REQUIRE(gx <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many streams (%lld)", (long long)S);
  dim3 grid((unsigned)gx, V ? 2u : 1u);
  block_commit_kernel<T><<<grid, kThreads, 0, stream>>>(
      static_cast<const T*>(K), static_cast<const T*>(V), static_cast<T*>(pool_K), static_cast<T*>(pool_V),
      static_cast<T*>(summary), S, n_slots, slot, L, d, dv);
  return check_launch("block_commit_kernel");
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_block_commit_mean(const void* K, const void* V, void* pool_K, void* pool_V, void* summary,
                                      int64_t n_streams, int n_slots, int slot, int L, int d, int dv, int dtype,
                                      cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_slots >= 1 && L >= 1 && d >= 1, GFST_ERR_ARG,
               "bad sizes (n_streams=%lld n_slots=%d L=%d d=%d)", (long long)n_streams, n_slots, L, d);
  GFST_REQUIRE(slot >= 0 && slot < n_slots, GFST_ERR_ARG, "slot %d outside [0, %d)", slot, n_slots);
  GFST_REQUIRE((V == nullptr) == (pool_V == nullptr), GFST_ERR_ARG, "V and pool_V must both be set or both NULL");
  GFST_REQUIRE(V == nullptr || dv >= 1, GFST_ERR_ARG, "dv must be >= 1 with values");
  if (n_streams == 0) return GFST_OK;
  GFST_REQUIRE(K && pool_K && summary, GFST_ERR_ARG, "K, pool_K and summary must be non-null");
  GFST_REQUIRE(aligned16(K) && aligned16(pool_K) && aligned16(summary) && aligned16(V) && aligned16(pool_V),
               GFST_ERR_ALIGN, "buffers must be 16-byte aligned");
  if (dtype == GFST_F32) return launch<float>(K, V, pool_K, pool_V, summary, n_streams, n_slots, slot, L, d, dv, stream);
  if (dtype == GFST_BF16)
    return launch<__nv_bfloat16>(K, V, pool_K, pool_V, summary, n_streams, n_slots, slot, L, d, dv, stream);
  set_last_error("unsupported dtype %d", dtype);
  return GFST_ERR_DTYPE;
}
