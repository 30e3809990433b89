// Shared pieces of the block top-k kernels: the register top-k list and the
// launcher declarations.
#pragma once
#include "gfst_common.cuh"

namespace gfst {

// Register top-k list of KCAP (score, index) entries, best first, filled with
// (-inf, INT_MAX) sentinels.  Candidates are offered in increasing index order,
// so a new entry moves ahead of an existing one only on a strictly higher
// score: ties keep the lower index first, and NaN / -inf never enter.
// One list per lane (one query row per lane).
template <int KCAP>
struct TopK {
  float s[KCAP];
  int i[KCAP];

  __device__ __forceinline__ void init() {
#pragma unroll
    for (int j = 0; j < KCAP; ++j) {
      s[j] = -INFINITY;
      i[j] = 0x7fffffff;
    }
  }
  __device__ __forceinline__ float kth() const { return s[KCAP - 1]; }
  // Branch-free insertion: when `take` is false the list is left unchanged
  // (it is sorted, so the bubble swaps nothing).  Every lane of a warp runs the
  // same instructions, whether or not it inserts.
  __device__ __forceinline__ void insert_if(bool take, float v, int idx) {
    s[KCAP - 1] = take ? v : s[KCAP - 1];
    i[KCAP - 1] = take ? idx : i[KCAP - 1];
#pragma unroll
    for (int j = KCAP - 1; j > 0; --j) {
      const bool sw = s[j] > s[j - 1];
      const float a = s[j], b = s[j - 1];
      s[j - 1] = sw ? a : b;
      s[j] = sw ? b : a;
      const int ia = i[j], ib = i[j - 1];
      i[j - 1] = sw ? ia : ib;
      i[j] = sw ? ib : ia;
    }
  }

  __device__ __forceinline__ static float pick16(const float (&v)[16], int c) {
    // binary select tree: v[c] without dynamic register indexing
    float l1[8], l2[4], l3[2];
#pragma unroll
    for (int q = 0; q < 8; ++q) l1[q] = (c & 1) ? v[2 * q + 1] : v[2 * q];
#pragma unroll
    for (int q = 0; q < 4; ++q) l2[q] = (c & 2) ? l1[2 * q + 1] : l1[2 * q];
#pragma unroll
    for (int q = 0; q < 2; ++q) l3[q] = (c & 4) ? l2[2 * q + 1] : l2[2 * q];
    return (c & 8) ? l3[1] : l3[0];
  }

  // Offer 16 consecutive candidates idx0 .. idx0+15 (only those < limit).  Must
  // be called by all 32 lanes of a warp together.  The common case -- no lane
  // has a candidate above its k-th score -- costs one max over the batch; else
  // each warp iteration inserts the next passing candidate of every lane at
  // once, so the work follows the busiest lane, not the union of all lanes.
  __device__ __forceinline__ void offer16(const float (&v)[16], int idx0, int limit) {
    float m = v[0];
#pragma unroll
    for (int c = 1; c < 16; ++c) m = fmaxf(m, v[c]);
    const bool maybe = m > kth();
    if (!__any_sync(0xffffffffu, maybe)) return;
    uint32_t mask = 0u;
    if (maybe) {
      const float t = kth();
#pragma unroll
      for (int c = 0; c < 16; ++c) mask |= ((v[c] > t && idx0 + c < limit) ? 1u : 0u) << c;
    }
    while (__any_sync(0xffffffffu, mask != 0u)) {
      const bool has = mask != 0u;
      const int c = has ? __ffs(mask) - 1 : 0;
      const float val = pick16(v, c);
      insert_if(has && val > kth(), val, idx0 + c);
      mask &= mask - 1u;
    }
  }
  __device__ __forceinline__ void write(float* os, int32_t* oi, int k) const {
#pragma unroll
    for (int j = 0; j < KCAP; ++j) {
      if (j < k) {
        const bool filled = i[j] != 0x7fffffff;
        os[j] = filled ? s[j] : -INFINITY;
        oi[j] = filled ? i[j] : -1;
      }
    }
  }
};

int block_topk_tc(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, float* ts,
                  int32_t* ti, cudaStream_t stream);
int read_device_error(int clear, unsigned int* value);
int read_readout_error(int clear, unsigned int* value);  // exact_readout.cu
int read_commit_error(int clear, unsigned int* value);   // block_commit_eig.cu
int read_score_error(int clear, unsigned int* value);    // block_score.cu
int read_scan_error(int clear, unsigned int* value);     // mpuc_scan.cu
int launch_bounded_wait_probe(long long budget, cudaStream_t stream);  // block_topk_tc.cu

int block_topk_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, int dtype,
                    float* ts, int32_t* ti, cudaStream_t stream);

}  // namespace gfst
