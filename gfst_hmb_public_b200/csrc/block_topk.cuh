// Shared pieces of the block top-k kernels: the register top-k list and the
// launcher declarations.
#pragma once
#include "gfst_common.cuh"

namespace gfst {

// Out-of-line insertion into a sorted (better-first) list of `kcap` entries in
// local memory; returns the new k-th score.  Callers keep the k-th score in a
// register and call this only when a candidate beats it -- rare once the list
// has filled -- so the scan loop stays small (an inlined insertion per
// candidate multiplies the code size and thrashes the instruction cache).
__device__ __noinline__ inline float topk_insert_local(float* ts, int* ti, int kcap, float s, int i) {
  int j = kcap - 1;
  while (j > 0 && better(s, i, ts[j - 1], ti[j - 1])) {
    ts[j] = ts[j - 1];
    ti[j] = ti[j - 1];
    --j;
  }
  ts[j] = s;
  ti[j] = i;
  return ts[kcap - 1];
}

int block_topk_tc(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, float* ts,
                  int32_t* ti, cudaStream_t stream);
int read_device_error(int clear, unsigned int* value);

int block_topk_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, int dtype,
                    float* ts, int32_t* ti, cudaStream_t stream);

}  // namespace gfst
