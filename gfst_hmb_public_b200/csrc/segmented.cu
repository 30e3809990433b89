// Segmented reductions of the readout's candidate lists and the block token
// score -- the runtime-backend operators the reference's readout calls.
//
// Reference (pkhairkh/gfst-hmb-public):
//   segmented_max_by_group / segmented_logsumexp_occurrence
//     src/gfst_hmb_mpuc/csrc/sm120_stub.cu:16-111, called from
//     perf.collapse_max_scores_by_group / collapse_logsumexp_scores_and_occurrence
//     (src/gfst_hmb_mpuc/perf.py:136-229) with group ids from torch.unique:
//     per group g the max m of its scores; with m finite, the score
//     m + log(max(sum exp(s - m), 1e-8)) and the (block, position) of the
//     group's first element (lowest index) scoring m; with m not finite the
//     score m + log(1e-8) and no occurrence (-1, -1).
//   exact_block_score
//     exact_block_project_forward (src/gfst_hmb_mpuc/csrc/sm120_cutlass_exact_block_score.cu:42-129,
//     a bf16 GEMM features x W^T with fp32 accumulation and bf16 output) and
//     the score of each token against the query, as _score_block_tokens uses
//     it (src/gfst_hmb_mpuc/modeling.py:640-651).
//
// The segmented kernels run one CTA over the whole list: the elements are
// ordered by (group, index) with a bitonic sort in shared memory, and one
// thread walks each group's run in element order (max, first maximal index,
// sum of exponentials), so the result does not depend on scheduling.
#include <math.h>

#include "gfst_common.cuh"

namespace gfst {
namespace {

constexpr int kSegThreads = 1024;
constexpr int kMaxSegElems = 16384;

__global__ void __launch_bounds__(kSegThreads) segmented_kernel(
    const float* __restrict__ scores, const int64_t* __restrict__ inverse, const int64_t* __restrict__ blocks,
    const int64_t* __restrict__ positions, int64_t n, int64_t groups, float* __restrict__ out_score,
    int64_t* __restrict__ out_block, int64_t* __restrict__ out_pos, bool lse) {
  extern __shared__ __align__(16) unsigned char seg_smem[];
  const int tid = threadIdx.x;
  int n_pow2 = 1;
  while (n_pow2 < n) n_pow2 <<= 1;
  unsigned long long* key = reinterpret_cast<unsigned long long*>(seg_smem);  // (group << 32) | index; ~0 = none
  float* sv = reinterpret_cast<float*>(key + n_pow2);                          // scores in sorted order
  // every group starts empty: max -inf, no occurrence
  for (int64_t g = tid; g < groups; g += kSegThreads) {
    out_score[g] = -INFINITY;
    if (lse) {
      out_block[g] = -1;
      out_pos[g] = -1;
    }
  }
  for (int e = tid; e < n_pow2; e += kSegThreads) {
    unsigned long long kv = ~0ull;
    if (e < n) {
      const int64_t g = inverse[e];
      if (g >= 0 && g < groups) kv = ((unsigned long long)g << 32) | (uint32_t)e;
    }
    key[e] = kv;
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int e = tid; e < n_pow2; e += kSegThreads) {
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
  for (int e = tid; e < n; e += kSegThreads) {
    const unsigned long long kv = key[e];
    sv[e] = kv == ~0ull ? 0.f : scores[(uint32_t)kv];
  }
  __syncthreads();
  // the head of each run (first sorted slot of its group) reduces the run
  for (int e = tid; e < n; e += kSegThreads) {
    const unsigned long long kv = key[e];
    if (kv == ~0ull) continue;
    const uint32_t g = (uint32_t)(kv >> 32);
    if (e > 0 && (uint32_t)(key[e - 1] >> 32) == g) continue;  // key[e - 1] is valid: invalid keys sort last
    int end = e;
    float m = -INFINITY;
    for (; end < n && key[end] != ~0ull && (uint32_t)(key[end] >> 32) == g; ++end)
      m = fmaxf(m, sv[end]);  // fmaxf: a NaN score does not set the max
    if (!lse) {
      out_score[g] = m;
      continue;
    }
    float sum = 0.f;
    int best = -1;
    if (isfinite(m)) {
      for (int j = e; j < end; ++j) {  // element order within the run
        const float v = sv[j];
        sum += expf(v - m);
        if (best < 0 && v == m) best = (int)(uint32_t)key[j];
      }
    }
    out_score[g] = m + logf(fmaxf(sum, 1e-8f));
    out_block[g] = best >= 0 ? blocks[best] : -1;
    out_pos[g] = best >= 0 ? positions[best] : -1;
  }
}

// ---------------------------------------------------------------------------
// block token score: score[t] = sum_j bf16(sum_c F[t][c] W[j][c]) * q[j]
// ---------------------------------------------------------------------------
constexpr int kBsRows = 16;    // token rows per CTA
constexpr int kBsThreads = 256;
constexpr int kBsK = 64;       // feature columns per shared-memory tile

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(v);
  else return v;
}

template <typename T>
__global__ void __launch_bounds__(kBsThreads) block_score_kernel(const T* __restrict__ q, const T* __restrict__ F,
                                                                 const T* __restrict__ Wt, int64_t m, int n, int k,
                                                                 float* __restrict__ scores) {
  __shared__ float fs[kBsRows][kBsK + 1];
  __shared__ float red[kBsThreads / 32][kBsRows];
  const int64_t r0 = (int64_t)blockIdx.x * kBsRows;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float part[kBsRows];
#pragma unroll
  for (int i = 0; i < kBsRows; ++i) part[i] = 0.f;
  // thread j < n owns key column j of every row; key columns beyond the
  // block size loop
  for (int j0 = 0; j0 < n; j0 += kBsThreads) {
    const int j = j0 + tid;
    float acc[kBsRows];
#pragma unroll
    for (int i = 0; i < kBsRows; ++i) acc[i] = 0.f;
    for (int c0 = 0; c0 < k; c0 += kBsK) {
      __syncthreads();
      for (int x = tid; x < kBsRows * kBsK; x += kBsThreads) {
        const int i = x / kBsK, c = c0 + x % kBsK;
        fs[i][x % kBsK] = (r0 + i < m && c < k) ? to_f(F[(r0 + i) * k + c]) : 0.f;
      }
      __syncthreads();
      if (j < n) {
        const T* wr = Wt + (int64_t)j * k + c0;
        const int cn = min(kBsK, k - c0);
        for (int c = 0; c < cn; ++c) {
          const float w = to_f(wr[c]);
#pragma unroll
          for (int i = 0; i < kBsRows; ++i) acc[i] = fmaf(fs[i][c], w, acc[i]);
        }
      }
    }
    if (j < n) {
      const float qj = to_f(q[j]);
#pragma unroll
      for (int i = 0; i < kBsRows; ++i) {
        // bf16: the projected key is rounded to bf16, as the projection's output is
        const float key = sizeof(T) == 2 ? __bfloat162float(__float2bfloat16_rn(acc[i])) : acc[i];
        part[i] = fmaf(key, qj, part[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kBsRows; ++i) {
    float v = part[i];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp][i] = v;
  }
  __syncthreads();
  if (tid < kBsRows && r0 + tid < m) {
    float s = 0.f;
    for (int w = 0; w < kBsThreads / 32; ++w) s += red[w][tid];
    // bf16: the score is a bf16 product widened to fp32, as (proj(F) @ q).float() is
    scores[r0 + tid] = sizeof(T) == 2 ? __bfloat162float(__float2bfloat16_rn(s)) : s;
  }
}

int launch_segmented(const float* scores, const int64_t* inverse, const int64_t* blocks, const int64_t* positions,
                     int64_t n, int64_t groups, float* out_score, int64_t* out_block, int64_t* out_pos, bool lse,
                     cudaStream_t stream) {
  GFST_REQUIRE(n >= 0 && groups >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(n <= kMaxSegElems, GFST_ERR_SHAPE, "%lld elements exceed %d", (long long)n, kMaxSegElems);
  GFST_REQUIRE(groups <= kMaxSegElems, GFST_ERR_SHAPE, "%lld groups exceed %d", (long long)groups, kMaxSegElems);
  if (groups == 0) return GFST_OK;
  GFST_REQUIRE(out_score && (!lse || (out_block && out_pos)), GFST_ERR_ARG, "null output");
  GFST_REQUIRE(n == 0 || (scores && inverse && (!lse || (blocks && positions))), GFST_ERR_ARG, "null input");
  int n_pow2 = 1;
  while (n_pow2 < n) n_pow2 <<= 1;
  const size_t smem = (size_t)n_pow2 * (sizeof(unsigned long long) + sizeof(float));
  cudaError_t e = cudaFuncSetAttribute(segmented_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  segmented_kernel<<<1, kSegThreads, smem, stream>>>(scores, inverse, blocks, positions, n, groups, out_score,
                                                     out_block, out_pos, lse);
  return check_launch("segmented_kernel");
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_segmented_max(const float* scores, const int64_t* inverse, int64_t n, int64_t group_count,
                                  float* grouped, cudaStream_t stream) {
  return gfst::launch_segmented(scores, inverse, nullptr, nullptr, n, group_count, grouped, nullptr, nullptr, false,
                                stream);
}

extern "C" int gfst_segmented_logsumexp_occurrence(const float* scores, const int64_t* inverse,
                                                   const int64_t* occurrence_blocks,
                                                   const int64_t* occurrence_positions, int64_t n,
                                                   int64_t group_count, float* grouped_scores,
                                                   int64_t* grouped_blocks, int64_t* grouped_positions,
                                                   cudaStream_t stream) {
  return gfst::launch_segmented(scores, inverse, occurrence_blocks, occurrence_positions, n, group_count,
                                grouped_scores, grouped_blocks, grouped_positions, true, stream);
}

extern "C" int gfst_exact_block_score(const void* query, const void* token_features, const void* weight, int64_t m,
                                      int n, int k, int dtype, float* scores, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(m >= 0 && n >= 1 && k >= 1, GFST_ERR_ARG, "bad sizes (m=%lld n=%d k=%d)", (long long)m, n, k);
  if (m == 0) return GFST_OK;
  GFST_REQUIRE(query && token_features && weight && scores, GFST_ERR_ARG, "null buffer");
  const int64_t grid = (m + kBsRows - 1) / kBsRows;
  GFST_REQUIRE(grid <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many rows");
  if (dtype == GFST_BF16) {
    block_score_kernel<__nv_bfloat16><<<(unsigned)grid, kBsThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(query), static_cast<const __nv_bfloat16*>(token_features),
        static_cast<const __nv_bfloat16*>(weight), m, n, k, scores);
  } else if (dtype == GFST_F32) {
    block_score_kernel<float><<<(unsigned)grid, kBsThreads, 0, stream>>>(
        static_cast<const float*>(query), static_cast<const float*>(token_features),
        static_cast<const float*>(weight), m, n, k, scores);
  } else {
    set_last_error("unsupported dtype %d", dtype);
    return GFST_ERR_DTYPE;
  }
  return check_launch("block_score_kernel");
}
