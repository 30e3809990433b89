// Exact top-k of one query against a bank of keys, any k <= count: the
// drop-in for the reference's FaissGpuRetriever.exact_topk
// (pkhairkh/gfst-hmb-public, src/gfst_hmb_mpuc/retrieval.py:165-172:
// scores = keys @ q, torch.topk, scores returned as float32).
//
// A score and its key index travel as one 64-bit sort key: the high word is
// the score's bits mapped to an unsigned order (NaN -> 0, below -inf), the low
// word is ~index, so "larger key" is the total order (score descending, index
// ascending) and a padding key of 0 ranks after every real one.  With bf16
// keys the score is rounded to bf16 before it is ranked, as the reference's
// bf16 matmul returns it.
//
// count <= kTile (16,384): one CTA of 1024 threads scores every key (a warp
// per key, 16-byte loads) into shared memory and bitonic-sorts the tile; the
// first k keys are the answer.  Larger banks: each CTA sorts one tile of
// scores and keeps its best min(k, kTile) keys in a workspace buffer; merge
// passes sort tiles of those candidates until one tile remains (k <= kTile/2,
// so every pass shrinks the candidate count by at least half).
#include <mutex>

#include "gfst_common.cuh"

// Scratch of gfst_exact_topk_noalloc: the tournament's two candidate buffers
// for banks of more than one tile, 1 MiB, shared by every call on a device.
constexpr long long kNoAllocScratchKeys = 131072;
static __device__ __align__(256) unsigned long long g_exact_topk_scratch[kNoAllocScratchKeys];

namespace gfst {
namespace {

constexpr int kTile = 16384;        // keys sorted per CTA (128 KB of shared memory)
constexpr int kTopkThreads = 1024;

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return bf16_to_f32(v); }

__device__ __forceinline__ uint32_t order_bits(float s) {
  if (s != s) return 0u;  // NaN ranks last
  if (s == 0.f) s = 0.f;  // -0 and +0 tie (then the lower index first)
  const uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float unorder_bits(uint32_t o) {
  if (o == 0u) return __int_as_float(0x7fc00000);
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

__device__ __forceinline__ uint64_t make_key(float s, uint32_t idx) {
  return ((uint64_t)order_bits(s) << 32) | (uint64_t)(~idx);
}

// bitonic sort of n (a power of two, <= kTile) keys in shared memory, largest first
__device__ void bitonic_desc(uint64_t* a, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
    }
  }
  __syncthreads();
}

// score keys [i0, i0 + n) of the bank into sk[0, n) as sort keys
template <typename T>
__device__ void score_tile(uint64_t* sk, const T* __restrict__ keys, const float* sq, int64_t i0, int n, int d,
                           bool round_bf16) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  constexpr int V = 16 / sizeof(T);
  for (int r = warp; r < n; r += nwarps) {
    const T* row = keys + (i0 + r) * (int64_t)d;
    float acc = 0.f;
    for (int c0 = lane * V; c0 < d; c0 += 32 * V) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + c0));
      if constexpr (sizeof(T) == 4) {
        acc = fmaf(__uint_as_float(v.x), sq[c0 + 0], acc);
        acc = fmaf(__uint_as_float(v.y), sq[c0 + 1], acc);
        acc = fmaf(__uint_as_float(v.z), sq[c0 + 2], acc);
        acc = fmaf(__uint_as_float(v.w), sq[c0 + 3], acc);
      } else {
        acc = fmaf(bf16_lo(v.x), sq[c0 + 0], acc);
        acc = fmaf(bf16_hi(v.x), sq[c0 + 1], acc);
        acc = fmaf(bf16_lo(v.y), sq[c0 + 2], acc);
        acc = fmaf(bf16_hi(v.y), sq[c0 + 3], acc);
        acc = fmaf(bf16_lo(v.z), sq[c0 + 4], acc);
        acc = fmaf(bf16_hi(v.z), sq[c0 + 5], acc);
        acc = fmaf(bf16_lo(v.w), sq[c0 + 6], acc);
        acc = fmaf(bf16_hi(v.w), sq[c0 + 7], acc);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      const float s = round_bf16 ? bf16_to_f32(f32_to_bf16(acc)) : acc;
      sk[r] = make_key(s, (uint32_t)(i0 + r));
    }
  }
}

// Score a tile of the bank and sort it.  final == true: write the first k as
// (score, index) outputs; otherwise write the first kk keys to cand[blockIdx.x * kk].
template <typename T>
__global__ void __launch_bounds__(kTopkThreads, 1) exact_topk_tile_kernel(const T* __restrict__ keys,
                                                                        const T* __restrict__ query, int64_t count,
                                                                        int d, int kk, bool round_bf16, bool final,
                                                                        float* out_scores, int64_t* out_idx,
                                                                        uint64_t* cand) {
  extern __shared__ uint64_t sk[];
  float* sq = reinterpret_cast<float*>(sk + kTile);
  for (int c = threadIdx.x; c < d; c += blockDim.x) sq[c] = to_float(query[c]);
  const int64_t i0 = (int64_t)blockIdx.x * kTile;
  const int n = (int)(count - i0 < (int64_t)kTile ? count - i0 : (int64_t)kTile);
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  // padding keys rank last; a short last tile still hands on kk keys
  for (int i = n + threadIdx.x; i < max(np2, kk); i += blockDim.x) sk[i] = 0ull;
  __syncthreads();
  score_tile<T>(sk, keys, sq, i0, n, d, round_bf16);
  bitonic_desc(sk, np2);
  if (final) {
    for (int i = threadIdx.x; i < kk; i += blockDim.x) {
      const uint64_t key = sk[i];
      out_scores[i] = unorder_bits((uint32_t)(key >> 32));
      out_idx[i] = (int64_t)(~(uint32_t)key);
    }
  } else {
    for (int i = threadIdx.x; i < kk; i += blockDim.x) cand[(int64_t)blockIdx.x * kk + i] = sk[i];
  }
}

// Sort tiles of n candidate keys; final == true writes the first k outputs.
__global__ void __launch_bounds__(kTopkThreads) exact_topk_merge_kernel(const uint64_t* __restrict__ in, int64_t n,
                                                                         int kk, bool final, float* out_scores,
                                                                         int64_t* out_idx, uint64_t* out) {
  extern __shared__ uint64_t sk[];
  const int64_t i0 = (int64_t)blockIdx.x * kTile;
  const int m = (int)(n - i0 < (int64_t)kTile ? n - i0 : (int64_t)kTile);
  int np2 = 1;
  while (np2 < m) np2 <<= 1;
  for (int i = threadIdx.x; i < max(np2, kk); i += blockDim.x) sk[i] = i < m ? in[i0 + i] : 0ull;
  bitonic_desc(sk, np2);
  if (final) {
    for (int i = threadIdx.x; i < kk; i += blockDim.x) {
      const uint64_t key = sk[i];
      out_scores[i] = unorder_bits((uint32_t)(key >> 32));
      out_idx[i] = (int64_t)(~(uint32_t)key);
    }
  } else {
    for (int i = threadIdx.x; i < kk; i += blockDim.x) out[(int64_t)blockIdx.x * kk + i] = sk[i];
  }
}

// per-pass candidate counts for a bank of `count` keys and top-k (k <= kTile / 2
// when count > kTile): pass 0 leaves ceil(count / kTile) * k keys, each merge
// pass ceil(n / kTile) * k, until n <= kTile
int64_t workspace_keys(int64_t count, int k) {
  if (count <= kTile) return 0;
  return ((count + kTile - 1) / kTile) * (int64_t)k;
}

template <typename T>
int launch_exact_topk(const void* keys, const void* query, int64_t count, int d, int k, bool round_bf16,
                      float* out_scores, int64_t* out_idx, uint64_t* ws, cudaStream_t stream) {
  const size_t smem_tile = (size_t)kTile * sizeof(uint64_t) + (size_t)d * sizeof(float);
  const size_t smem_merge = (size_t)kTile * sizeof(uint64_t);
  cudaError_t e = cudaFuncSetAttribute(exact_topk_tile_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_tile);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const T* kp = static_cast<const T*>(keys);
  const T* qp = static_cast<const T*>(query);
  if (count <= kTile) {
    exact_topk_tile_kernel<T><<<1, kTopkThreads, smem_tile, stream>>>(kp, qp, count, d, k, round_bf16, true,
                                                                      out_scores, out_idx, nullptr);
    return check_launch("exact_topk_tile_kernel");
  }
  e = cudaFuncSetAttribute(exact_topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_merge);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int64_t tiles = (count + kTile - 1) / kTile;
  GFST_REQUIRE(tiles <= 0x7fffffffLL, GFST_ERR_SHAPE, "bank too large");
  uint64_t* a = ws;
  uint64_t* b = ws + workspace_keys(count, k);
  exact_topk_tile_kernel<T><<<(unsigned)tiles, kTopkThreads, smem_tile, stream>>>(kp, qp, count, d, k, round_bf16,
                                                                                  false, nullptr, nullptr, a);
  int st = check_launch("exact_topk_tile_kernel");
  if (st != GFST_OK) return st;
  int64_t n = tiles * k;
  while (n > kTile) {
    const int64_t g = (n + kTile - 1) / kTile;
    exact_topk_merge_kernel<<<(unsigned)g, kTopkThreads, smem_merge, stream>>>(a, n, k, false, nullptr, nullptr,
                                                                               b);
    st = check_launch("exact_topk_merge_kernel");
    if (st != GFST_OK) return st;
    n = g * k;
    uint64_t* t = a;
    a = b;
    b = t;
  }
  exact_topk_merge_kernel<<<1, kTopkThreads, smem_merge, stream>>>(a, n, k, true, out_scores, out_idx, nullptr);
  return check_launch("exact_topk_merge_kernel");
}

}  // namespace
}  // namespace gfst

extern "C" size_t gfst_exact_topk_workspace_bytes(int64_t count, int k) {
  if (count <= 0 || k <= 0) return 0;
  return (size_t)(2 * gfst::workspace_keys(count, k)) * sizeof(uint64_t);
}

extern "C" int gfst_exact_topk(const void* keys, const void* query, int64_t count, int d, int k, int dtype,
                               int round_scores, float* out_scores, int64_t* out_idx, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(count >= 1 && count <= 0xffffffffLL, GFST_ERR_ARG, "count=%lld outside [1, 2^32 - 1]",
               (long long)count);
  GFST_REQUIRE(k >= 1 && k <= count, GFST_ERR_ARG, "k=%d outside [1, count]", k);
  GFST_REQUIRE(count <= kTile || k <= kTile / 2, GFST_ERR_SHAPE,
               "k=%d above %d for a bank of more than %d keys", k, kTile / 2, kTile);
  GFST_REQUIRE(d >= 1 && d <= 1024, GFST_ERR_SHAPE, "d=%d outside [1, 1024]", d);
  GFST_REQUIRE(keys && query && out_scores && out_idx, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(aligned16(keys), GFST_ERR_ALIGN, "keys must be 16-byte aligned");
  const size_t need = gfst_exact_topk_workspace_bytes(count, k);
  GFST_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr), GFST_ERR_ARG,
               "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  GFST_REQUIRE(need == 0 || (reinterpret_cast<uintptr_t>(workspace) & 7u) == 0, GFST_ERR_ALIGN,
               "workspace must be 8-byte aligned");
  if (dtype == GFST_F32) {
    GFST_REQUIRE(d % 4 == 0, GFST_ERR_ALIGN, "d=%d must be a multiple of 4 for float32 keys", d);
    return launch_exact_topk<float>(keys, query, count, d, k, false, out_scores, out_idx,
                                    static_cast<uint64_t*>(workspace), stream);
  }
  if (dtype == GFST_BF16) {
    GFST_REQUIRE(d % 8 == 0, GFST_ERR_ALIGN, "d=%d must be a multiple of 8 for bfloat16 keys", d);
    return launch_exact_topk<__nv_bfloat16>(keys, query, count, d, k, round_scores != 0, out_scores, out_idx,
                                            static_cast<uint64_t*>(workspace), stream);
  }
  set_last_error("unsupported dtype %d", dtype);
  return GFST_ERR_DTYPE;
}

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once
// per device (cudaGetSymbolAddress with that device current) and cached.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  GFST_REQUIRE(dev >= 0 && dev < kMaxDevices, GFST_ERR_DEVICE, "device ordinal %d above %d", dev, kMaxDevices - 1);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_exact_topk_scratch);
    GFST_REQUIRE(e == cudaSuccess && p != nullptr, GFST_ERR_DEVICE, "cudaGetSymbolAddress of the top-k scratch: %s",
                 cudaGetErrorString(e));
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return GFST_OK;
}

}  // namespace

extern "C" int gfst_exact_topk_noalloc(const void* keys, const void* query, int64_t count, int d, int k, int dtype,
                                       int round_scores, float* out_scores, int64_t* out_idx, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(count >= 1 && k >= 1 && k <= count, GFST_ERR_ARG, "need 1 <= k <= count (count=%lld k=%d)",
               (long long)count, k);
  const size_t need = gfst_exact_topk_workspace_bytes(count, k);
  const size_t have = (size_t)kNoAllocScratchKeys * sizeof(unsigned long long);
  GFST_REQUIRE(need <= have, GFST_ERR_SHAPE,
               "count=%lld with k=%d needs %zu bytes of scratch, above the %zu-byte static scratch of "
               "gfst_exact_topk_noalloc (2 * ceil(count / 16384) * k must be <= %lld); use gfst_exact_topk with a "
               "caller-provided workspace", (long long)count, k, need, have, kNoAllocScratchKeys);
  void* scratch = nullptr;
  if (need > 0) {
    const int st = scratch_address(&scratch);
    if (st != GFST_OK) return st;
  }
  return gfst_exact_topk(keys, query, count, d, k, dtype, round_scores, out_scores, out_idx, scratch, need, stream);
}
