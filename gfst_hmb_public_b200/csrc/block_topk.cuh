// Shared pieces of the block top-k kernels: the register top-k list and the
// launcher declarations.
#pragma once
#include "gfst_common.cuh"

namespace gfst {

// Insert (s, i) into the sorted list ts/ti (best first, `better` order) that
// keeps the KCAP best candidates seen so far.  Callers scan candidates in
// increasing index order and only insert when s > ts[KCAP-1]; a tie therefore
// never displaces an earlier (lower) index, and NaN or -inf scores are never
// selected.  The list starts filled with (-inf, INT_MAX) sentinels.
template <int KCAP>
__device__ __forceinline__ void topk_insert(float (&ts)[KCAP], int (&ti)[KCAP], float s, int i) {
  if (!better(s, i, ts[KCAP - 1], ti[KCAP - 1])) return;
  ts[KCAP - 1] = s;
  ti[KCAP - 1] = i;
#pragma unroll
  for (int j = KCAP - 1; j > 0; --j) {
    if (better(ts[j], ti[j], ts[j - 1], ti[j - 1])) {
      const float tf = ts[j];
      ts[j] = ts[j - 1];
      ts[j - 1] = tf;
      const int tt = ti[j];
      ti[j] = ti[j - 1];
      ti[j - 1] = tt;
    }
  }
}

int block_topk_tc(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, float* ts,
                  int32_t* ti, cudaStream_t stream);
int read_device_error(int clear, unsigned int* value);

int block_topk_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, int dtype,
                    float* ts, int32_t* ti, cudaStream_t stream);

}  // namespace gfst
