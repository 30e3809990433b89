// Shared pieces of the block top-k kernels: the register top-k list and the
// launcher declarations.
#pragma once
#include "gfst_common.cuh"

namespace gfst {

// Register top-k list of KCAP (score, index) entries, best first, filled with
// (-inf, INT_MAX) sentinels.  Candidates are offered in increasing index order,
// so a new entry moves ahead of an existing one only on a strictly higher
// score: ties keep the lower index first, and NaN / -inf never enter.
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
  __device__ __forceinline__ void insert(float v, int idx) {
    s[KCAP - 1] = v;
    i[KCAP - 1] = idx;
#pragma unroll
    for (int j = KCAP - 1; j > 0; --j) {
      if (s[j] > s[j - 1]) {
        const float ts = s[j];
        s[j] = s[j - 1];
        s[j - 1] = ts;
        const int ti = i[j];
        i[j] = i[j - 1];
        i[j - 1] = ti;
      }
    }
  }
  // Offer 16 consecutive candidates idx0 .. idx0+15 (only those < limit).  The
  // common case -- none beats the k-th score -- costs one max over the batch;
  // otherwise a rolled loop walks the batch with a single inlined insertion.
  __device__ __forceinline__ void offer16(const float (&v)[16], int idx0, int limit) {
    float m = v[0];
#pragma unroll
    for (int c = 1; c < 16; ++c) m = fmaxf(m, v[c]);
    if (!(m > kth())) return;
    float vl[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) vl[c] = v[c];
#pragma unroll 1
    for (int c = 0; c < 16; ++c) {
      const float val = vl[c];
      if (idx0 + c < limit && val > kth()) insert(val, idx0 + c);
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

int block_topk_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, int dtype,
                    float* ts, int32_t* ti, cudaStream_t stream);

}  // namespace gfst
