// Segmented reductions of the readout's candidate lists -- the runtime-backend
// operators the reference's token-id collapse calls.
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
