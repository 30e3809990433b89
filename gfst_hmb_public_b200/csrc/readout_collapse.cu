// Exact readout with the log-sum-exp collapse of duplicate token ids.
//
// Reference (pkhairkh/gfst-hmb-public): the candidates of a query are the
// tokens of its retrieved blocks in retrieval order (modeling.py:599-657,
// _score_block_tokens); collapse_logsumexp_scores_and_occurrence
// (src/gfst_hmb_mpuc/perf.py:164-229) groups them by token id:
//   group max m, group score = m + log(max(sum exp(s - m), 1e-8)),
//   occurrence = (block, position) of the first candidate whose score is m;
// the selection (modeling.py:1151-1169) takes the best group score.  Here ties
// between group scores go to the lowest token id, a block listed twice for a
// query counts once, NaN scores and negative token ids take no part.
//
// One CTA per query: candidate scores into shared memory (fp32 accumulate),
// a bitonic sort of (token id, candidate index) keys, one pass over the sorted
// runs (each run's sum in candidate order, as scatter_add accumulates), and a
// block-wide arg-max over the runs.
#include <type_traits>

#include "gfst_common.cuh"

namespace gfst {
namespace {

constexpr int kCThreads = 256;
constexpr int kMaxCand = 2048;  // K * L per query

template <typename T>
__device__ __forceinline__ float load_f32(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else return __bfloat162float(*p);
}

template <typename T>
__global__ void __launch_bounds__(kCThreads) readout_collapse_kernel(
    const T* __restrict__ Q, const T* __restrict__ pool_K, const int32_t* __restrict__ token_ids,
    const int32_t* __restrict__ top_idx, int n_queries, int n_slots, int L, int d, int k, int32_t* __restrict__ best_id,
    float* __restrict__ best_score, int32_t* __restrict__ best_block, int32_t* __restrict__ best_pos) {
  __shared__ float sc[kMaxCand];
  __shared__ unsigned long long key[kMaxCand];  // (token id << 32) | candidate index; ~0 = none
  __shared__ int blocks[32];
  __shared__ float qv[256];
  __shared__ float red_s[kCThreads / 32];
  __shared__ int red_i[kCThreads / 32], red_c[kCThreads / 32];
  const int64_t sq = blockIdx.x;
  const int64_t s = sq / n_queries;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = k * L;
  for (int c = tid; c < d; c += kCThreads) qv[c] = load_f32(Q + sq * d + c);
  if (tid < k) {
    int b = top_idx[sq * k + tid];
    if (b < 0 || b >= n_slots) b = -1;
    for (int j = 0; j < tid; ++j)  // a block listed twice counts once
      if (top_idx[sq * k + j] == b) b = -1;
    blocks[tid] = b;
  }
  __syncthreads();
  int n_pow2 = 1;
  while (n_pow2 < n) n_pow2 <<= 1;
  for (int e = tid; e < n_pow2; e += kCThreads) {
    unsigned long long kv = ~0ull;
    if (e < n) {
      const int j = e / L, p = e % L, b = blocks[j];
      if (b >= 0) {
        const T* row = pool_K + (((size_t)s * n_slots + b) * L + p) * d;
        float acc = 0.f;
        for (int c = 0; c < d; ++c) acc = fmaf(load_f32(row + c), qv[c], acc);
        const int id = token_ids[((size_t)s * n_slots + b) * L + p];
        sc[e] = acc;
        if (id >= 0 && acc == acc) kv = ((unsigned long long)(uint32_t)id << 32) | (uint32_t)e;
      }
    }
    key[e] = kv;
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int e = tid; e < n_pow2; e += kCThreads) {
        const int partner = e ^ stride;
        if (partner > e) {
          const bool up = (e & size) == 0;
          const unsigned long long a = key[e], b = key[partner];
          if ((a > b) == up) {
            key[e] = b;
            key[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // runs of equal token id: thread per run head
  float bs = -INFINITY;
  int bid = 0x7fffffff, bcand = -1;
  for (int e = tid; e < n; e += kCThreads) {
    const unsigned long long kv = key[e];
    if (kv == ~0ull) continue;
    const uint32_t id = (uint32_t)(kv >> 32);
    if (e > 0 && key[e - 1] != ~0ull && (uint32_t)(key[e - 1] >> 32) == id) continue;  // not a head
    float m = -INFINITY;
    int first = -1;
    int end = e;
    for (; end < n && key[end] != ~0ull && (uint32_t)(key[end] >> 32) == id; ++end) {
      const int ci = (int)(uint32_t)key[end];
      if (sc[ci] > m) {
        m = sc[ci];
        first = ci;
      }
    }
    float sum = 0.f;
    for (int j = e; j < end; ++j) sum += expf(sc[(int)(uint32_t)key[j]] - m);
    const float g = m + logf(fmaxf(sum, 1e-8f));
    if (g > bs || (g == bs && (int)id < bid)) {
      bs = g;
      bid = (int)id;
      bcand = first;
    }
  }
  // block-wide best group (score desc, token id asc)
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bid, o);
    const int c2 = __shfl_xor_sync(0xffffffffu, bcand, o);
    if (s2 > bs || (s2 == bs && i2 < bid)) {
      bs = s2;
      bid = i2;
      bcand = c2;
    }
  }
  if (lane == 0) {
    red_s[warp] = bs;
    red_i[warp] = bid;
    red_c[warp] = bcand;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kCThreads / 32; ++w) {
      if (red_s[w] > bs || (red_s[w] == bs && red_i[w] < bid)) {
        bs = red_s[w];
        bid = red_i[w];
        bcand = red_c[w];
      }
    }
    const bool found = bcand >= 0;
    best_id[sq] = found ? bid : -1;
    best_score[sq] = found ? bs : -INFINITY;
    best_block[sq] = found ? blocks[bcand / L] : -1;
    best_pos[sq] = found ? bcand % L : -1;
  }
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_exact_readout_collapse(const void* Q, const void* pool_K, const int32_t* token_ids,
                                           const int32_t* top_idx, int64_t n_streams, int n_queries, int n_slots,
                                           int L, int d, int k, int dtype, int32_t* best_id, float* best_score,
                                           int32_t* best_block, int32_t* best_pos, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_slots >= 1 && L >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(k >= 1 && k <= 32 && (int64_t)k * L <= kMaxCand, GFST_ERR_SHAPE, "k * L = %lld outside [1, %d]",
               (long long)k * L, kMaxCand);
  GFST_REQUIRE(d >= 1 && d <= 256, GFST_ERR_SHAPE, "d=%d outside [1, 256]", d);
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(Q && pool_K && token_ids && top_idx && best_id && best_score && best_block && best_pos, GFST_ERR_ARG,
               "null buffer");
  GFST_REQUIRE(n_streams * (int64_t)n_queries <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many queries");
  const unsigned grid = (unsigned)(n_streams * n_queries);
  if (dtype == GFST_F32) {
    readout_collapse_kernel<float><<<grid, kCThreads, 0, stream>>>(
        static_cast<const float*>(Q), static_cast<const float*>(pool_K), token_ids, top_idx, n_queries, n_slots, L, d,
        k, best_id, best_score, best_block, best_pos);
  } else if (dtype == GFST_BF16) {
    readout_collapse_kernel<__nv_bfloat16><<<grid, kCThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(Q), static_cast<const __nv_bfloat16*>(pool_K), token_ids, top_idx,
        n_queries, n_slots, L, d, k, best_id, best_score, best_block, best_pos);
  } else {
    set_last_error("unsupported dtype %d", dtype);
    return GFST_ERR_DTYPE;
  }
  return check_launch("readout_collapse_kernel");
}
