// Merge candidate lists into a top-k in the total order (score descending,
// index ascending).  Used after the all-gather of per-GPU candidates when a long
// memory is sharded by block range: every rank merges the same gathered lists
// with the same deterministic order, so all ranks agree on the global top-k.
// One thread per row; candidates with a negative index, a NaN or a -inf score
// are skipped.
#include "block_topk.cuh"

namespace gfst {
namespace {

constexpr int kThreads = 128;

// Candidates arrive in arbitrary index order, so insertion compares with the
// full (score, index) order.
template <int KCAP>
__global__ void __launch_bounds__(kThreads) topk_merge_kernel(const float* __restrict__ scores,
                                                              const int32_t* __restrict__ idx, int64_t rows,
                                                              int n_cand, int k, float* __restrict__ out_s,
                                                              int32_t* __restrict__ out_i) {
  const int64_t row = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (row >= rows) return;
  float ts[KCAP];
  int ti[KCAP];
#pragma unroll
  for (int j = 0; j < KCAP; ++j) {
    ts[j] = -INFINITY;
    ti[j] = 0x7fffffff;
  }
  const float* sr = scores + row * n_cand;
  const int32_t* ir = idx + row * n_cand;
  for (int c = 0; c < n_cand; ++c) {
    const float s = sr[c];
    const int i = ir[c];
    if (i < 0 || !(s > -INFINITY)) continue;
    if (!better(s, i, ts[KCAP - 1], ti[KCAP - 1])) continue;
    ts[KCAP - 1] = s;
    ti[KCAP - 1] = i;
#pragma unroll
    for (int j = KCAP - 1; j > 0; --j) {
      if (better(ts[j], ti[j], ts[j - 1], ti[j - 1])) {
        const float a = ts[j];
        ts[j] = ts[j - 1];
        ts[j - 1] = a;
        const int b = ti[j];
        ti[j] = ti[j - 1];
        ti[j - 1] = b;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < KCAP; ++j) {
    if (j < k) {
      const bool filled = ti[j] != 0x7fffffff;
      out_s[row * k + j] = filled ? ts[j] : -INFINITY;
      out_i[row * k + j] = filled ? ti[j] : -1;
    }
  }
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_topk_merge(const float* scores, const int32_t* idx, int64_t rows, int n_cand, int k,
                               float* out_scores, int32_t* out_idx, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(rows >= 0 && n_cand >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(k >= 1 && k <= 32, GFST_ERR_SHAPE, "k=%d outside [1, 32]", k);
  if (rows == 0) return GFST_OK;
  GFST_REQUIRE(out_scores && out_idx && (n_cand == 0 || (scores && idx)), GFST_ERR_ARG, "null buffer");
  const int64_t blocks = (rows + kThreads - 1) / kThreads;
  GFST_REQUIRE(blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many rows");
  if (k <= 2) {
    topk_merge_kernel<2><<<(unsigned)blocks, kThreads, 0, stream>>>(scores, idx, rows, n_cand, k, out_scores, out_idx);
  } else if (k <= 8) {
    topk_merge_kernel<8><<<(unsigned)blocks, kThreads, 0, stream>>>(scores, idx, rows, n_cand, k, out_scores, out_idx);
  } else {
    topk_merge_kernel<32><<<(unsigned)blocks, kThreads, 0, stream>>>(scores, idx, rows, n_cand, k, out_scores,
                                                                      out_idx);
  }
  return check_launch("topk_merge_kernel");
}
