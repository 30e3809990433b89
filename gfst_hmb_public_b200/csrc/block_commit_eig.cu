// Reference-faithful block commit: the eigen summary of a closed block.
//
// Reference (pkhairkh/gfst-hmb-public): GfstHmbSublayer._update_block_memory
// (src/gfst_hmb_mpuc/modeling.py:3482-3507) and its replay
// (src/gfst_hmb_mpuc/diagnostics/block_commit_replay.py:97-139):
//   average_projector = projector_sum / n          (float32)
//   reduced_mean      = reduced_sum / n            (float32)
//   top_eig_summary(average_projector, rank=max_flag_dim, rank_boundaries=flag_dims)
//     (src/gfst_hmb_mpuc/gfst.py:389-430): symmetrise in float32, eigh in
//     float64, walk eigenvalue clusters (|a - b| <= 1e-9 + 1e-7 |b|) down from
//     the top, replace each cluster by its canonical basis (gfst.py:172-214:
//     Gram-Schmidt over the cluster projector's columns in descending-diagonal
//     order, first-significant-entry signs), cast to float32 and fix signs again.
//   summary_basis = the first max_flag_dim columns, top_vector = column 0.
//
// One CTA per stream.  The float64 symmetric eigenproblem (d <= 64) is solved
// by cyclic Jacobi in shared memory with the round-robin (tournament) pair
// order: d/2 disjoint rotations per round, rows then columns updated by all
// threads, eigenvectors accumulated alongside.  A pair is rotated while its
// off-diagonal entry exceeds 1e-16 of the Frobenius norm; the iteration ends
// with the first sweep that rotates nothing, or after 40 sweeps, which raises
// GFST_ERR_NUMERIC in a sticky device word.  The
// cluster bases are built by one warp per cluster.  Eigenvectors of a cluster
// are only defined up to rotation inside it, which the canonical basis removes,
// so the result does not depend on the eigensolver's own choices.
#include "gfst_common.cuh"

namespace gfst {

// sticky GFST_ERR_NUMERIC report of the eigen commit
GFST_DEFINE_ERROR_WORD(g_commit_error, read_commit_error, "commit")

namespace {

constexpr int kEigThreads = 256;
constexpr int kEigWarps = kEigThreads / 32;
constexpr int kEigMaxD = 64;
constexpr int kMaxSweeps = 40;
constexpr double kClusterAtol = 1e-9;  // gfst.py:6
constexpr double kClusterRtol = 1e-7;  // gfst.py:7
constexpr double kMgsEps = 1e-9;       // gfst.py:176 (eps of the cluster basis)

struct EigSmem {
  double a[kEigMaxD][kEigMaxD + 1];  // working matrix (padded rows)
  double v[kEigMaxD][kEigMaxD + 1];  // eigenvectors, column j for eigenvalue a[j][j]
  double fb[kEigMaxD][kEigMaxD];     // full canonical basis, [row][column]
  double rc[kEigMaxD / 2], rs[kEigMaxD / 2];
  int rp[kEigMaxD / 2], rq[kEigMaxD / 2];
  int order[kEigMaxD];               // eigen indices by ascending eigenvalue
  int cl_start[kEigMaxD], cl_end[kEigMaxD], cl_take[kEigMaxD], cl_off[kEigMaxD];
  double red[kEigThreads / 32][2];
  double wdiag[kEigWarps][kEigMaxD];  // per-warp scratch: cluster projector diagonal
  double wvec[kEigWarps][kEigMaxD];   // per-warp scratch: the vector being orthogonalised
  int waxis[kEigWarps][kEigMaxD];     // per-warp scratch: axes by descending diagonal
  int n_clusters, fail, rotated;
};

__device__ __forceinline__ double warp_sum(double x) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// tournament pairing: round r of n - 1 (n even), pair k of n / 2
__device__ __forceinline__ void round_pair(int n, int r, int k, int& p, int& q) {
  const int m = n - 1;
  const int a = k == 0 ? 0 : (k - 1 + r) % m + 1;
  const int b = (m - 1 - k + r) % m + 1;
  p = a < b ? a : b;
  q = a < b ? b : a;
}

struct GlobalDims {
  int n;
  int v[8];
};

// first-significant-entry sign of one column (gfst.py:35-46): +1 or -1
template <typename T>
__device__ __forceinline__ T first_significant_sign(const T* col, int stride, int d, T eps_sign) {
  for (int i = 0; i < d; ++i) {
    const T x = col[i * stride];
    if (fabs((double)x) > (double)eps_sign) return x < T(0) ? T(-1) : T(1);
  }
  return T(1);
}

// Eigenpairs of the symmetric float64 matrix in sm.a (order d, padded to an
// even n with an isolated zero index): cyclic Jacobi in tournament order, V in
// sm.v (column j for the eigenvalue left in sm.a[j][j]), and sm.order = the
// indices < d by ascending eigenvalue (ties by index).  Every thread of the
// CTA calls; 40 sweeps without convergence set sm.fail.
__device__ void jacobi_eigen(EigSmem& sm, int d) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = d + (d & 1);
  for (int e = tid; e < n * n; e += kEigThreads) {
    const int i = e / n, j = e % n;
    sm.v[i][j] = i == j ? 1.0 : 0.0;
  }
  __syncthreads();

  // ---- cyclic Jacobi, tournament order ----
  // A pair is rotated while |a_pq| > 1e-16 ||A||_F (float64 round-off of the
  // whole matrix); the sweep that rotates nothing ends the iteration.
  double tot = 0.0;
  {
    double part = 0.0;
    for (int e = tid; e < n * n; e += kEigThreads) {
      const double x = sm.a[e / n][e % n];
      part += x * x;
    }
    part = warp_sum(part);
    if (lane == 0) sm.red[warp][0] = part;
    __syncthreads();
    for (int w = 0; w < kEigWarps; ++w) tot += sm.red[w][0];
  }
  const double skip = 1e-32 * tot;  // (1e-16 ||A||_F)^2; Frobenius norm is invariant under rotations
  int sweep = 0;
  for (; sweep < kMaxSweeps; ++sweep) {
    if (tid == 0) sm.rotated = 0;
    __syncthreads();
    for (int r = 0; r < n - 1; ++r) {
      if (tid < n / 2) {
        int p, q;
        round_pair(n, r, tid, p, q);
        const double apq = sm.a[p][q];
        double c = 1.0, sn = 0.0;
        if (apq * apq > skip) {
          // t = the smaller root of t^2 + 2 theta t - 1 = 0, theta = delta / (2 a_pq),
          // written as 2 a_pq sgn(delta) / (|delta| + sqrt(delta^2 + 4 a_pq^2)):
          // one square root, one division and one reciprocal square root on the
          // round's critical path
          const double delta = sm.a[q][q] - sm.a[p][p];
          const double two_a = 2.0 * apq;
          const double rr = sqrt(fma(delta, delta, two_a * two_a));
          const double t = (delta >= 0.0 ? two_a : -two_a) / (fabs(delta) + rr);
          c = rsqrt(fma(t, t, 1.0));
          sn = t * c;
          sm.rotated = 1;
        }
        sm.rc[tid] = c;
        sm.rs[tid] = sn;
        sm.rp[tid] = p;
        sm.rq[tid] = q;
      }
      __syncthreads();
      // a warp per rotation, its lanes along the row / column (no index
      // division; the rotation's parameters are read once per warp)
      for (int k = warp; k < n / 2; k += kEigWarps) {  // rows: A <- J^T A
        const int p = sm.rp[k], q = sm.rq[k];
        const double c = sm.rc[k], sn = sm.rs[k];
        for (int j = lane; j < n; j += 32) {
          const double x = sm.a[p][j], y = sm.a[q][j];
          sm.a[p][j] = c * x - sn * y;
          sm.a[q][j] = sn * x + c * y;
        }
      }
      __syncthreads();
      for (int k = warp; k < n / 2; k += kEigWarps) {  // columns: A <- A J, V <- V J
        const int p = sm.rp[k], q = sm.rq[k];
        const double c = sm.rc[k], sn = sm.rs[k];
        for (int i = lane; i < n; i += 32) {
          const double x = sm.a[i][p], y = sm.a[i][q];
          sm.a[i][p] = c * x - sn * y;
          sm.a[i][q] = sn * x + c * y;
          const double u = sm.v[i][p], w = sm.v[i][q];
          sm.v[i][p] = c * u - sn * w;
          sm.v[i][q] = sn * u + c * w;
        }
      }
      __syncthreads();
    }
    if (sm.rotated == 0) break;  // read after the last barrier of the sweep: uniform
    __syncthreads();             // everyone has read the flag before it is reset
  }
  if (sweep == kMaxSweeps && tid == 0) sm.fail = 1;

  // ---- eigenvalues ascending (the padded index, if any, is left out) ----
  for (int i = tid; i < d; i += kEigThreads) {
    const double ei = sm.a[i][i];
    int pos = 0;
    for (int j = 0; j < d; ++j) {
      const double ej = sm.a[j][j];
      pos += (ej < ei || (ej == ei && j < i)) ? 1 : 0;
    }
    sm.order[pos] = i;
  }
  __syncthreads();
}

// The canonical top basis of the symmetric float64 matrix in sm.a (order d,
// padded to even n): eigenpairs by Jacobi, clusters from the top, canonical
// cluster bases (float64, in sm.fb), then the float32 basis with its signs
// fixed again, written to fb32 [d][target] (which may alias sm.a once the
// eigenpairs are known).  Every thread of the CTA calls; failures set sm.fail.
__device__ void canonical_top_basis(EigSmem& sm, int d, int target, double eps_sign) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  jacobi_eigen(sm, d);

  // ---- clusters from the top (gfst.py:248-297) ----
  if (tid == 0) {
    int remaining = target, end = d - 1, nc = 0, off = 0;
    while (end >= 0 && remaining > 0) {
      int start = end;
      while (start > 0) {
        const double lo = sm.a[sm.order[start - 1]][sm.order[start - 1]];
        const double hi = sm.a[sm.order[start]][sm.order[start]];
        if (!(fabs(lo - hi) <= kClusterAtol + kClusterRtol * fabs(hi))) break;
        --start;
      }
      const int take = min(end - start + 1, remaining);
      sm.cl_start[nc] = start;
      sm.cl_end[nc] = end;
      sm.cl_take[nc] = take;
      sm.cl_off[nc] = off;
      ++nc;
      off += take;
      remaining -= take;
      end = start - 1;
    }
    sm.n_clusters = nc;
    if (remaining > 0) sm.fail = 1;
  }
  __syncthreads();

  // ---- canonical basis of each cluster (gfst.py:172-214), one warp per cluster ----
  for (int c = warp; c < sm.n_clusters; c += kEigWarps) {
    const int start = sm.cl_start[c], m = sm.cl_end[c] - start + 1, t = sm.cl_take[c], off = sm.cl_off[c];
    double* diag = sm.wdiag[warp];
    double* vec = sm.wvec[warp];
    int* axis_at = sm.waxis[warp];
    // diagonal of the cluster projector C C^T, then axes by (-diagonal, index)
    for (int i = lane; i < d; i += 32) {
      double acc = 0.0;
      for (int k = 0; k < m; ++k) {
        const double x = sm.v[i][sm.order[start + k]];
        acc = fma(x, x, acc);
      }
      diag[i] = acc;
    }
    __syncwarp();
    for (int i = lane; i < d; i += 32) {
      int pos = 0;
      for (int j = 0; j < d; ++j) pos += (diag[j] > diag[i] || (diag[j] == diag[i] && j < i)) ? 1 : 0;
      axis_at[pos] = i;
    }
    __syncwarp();
    int have = 0;
    // candidates: projector columns in axis order, then the cluster's own columns
    for (int cand = 0; cand < d + m && have < t; ++cand) {
      for (int i = lane; i < d; i += 32) {
        double x = 0.0;
        if (cand < d) {
          const int ax = axis_at[cand];
          for (int k = 0; k < m; ++k) {
            const int ev = sm.order[start + k];
            x = fma(sm.v[i][ev], sm.v[ax][ev], x);
          }
        } else {
          x = sm.v[i][sm.order[start + cand - d]];
        }
        vec[i] = x;
      }
      __syncwarp();
      // modified Gram-Schmidt against the columns found so far
      for (int j = 0; j < have; ++j) {
        double part = 0.0;
        for (int i = lane; i < d; i += 32) part = fma(sm.fb[i][off + j], vec[i], part);
        const double dot = warp_sum(part);
        for (int i = lane; i < d; i += 32) vec[i] = fma(-dot, sm.fb[i][off + j], vec[i]);
        __syncwarp();
      }
      double part = 0.0;
      for (int i = lane; i < d; i += 32) part = fma(vec[i], vec[i], part);
      const double norm = sqrt(warp_sum(part));
      if (norm > kMgsEps) {
        for (int i = lane; i < d; i += 32) sm.fb[i][off + have] = vec[i] / norm;
        ++have;
      }
      __syncwarp();
    }
    if (have < t) {
      if (lane == 0) sm.fail = 1;
    } else {  // signs of the cluster's columns (float64)
      for (int j = lane; j < t; j += 32) {
        const double sg = first_significant_sign<double>(&sm.fb[0][off + j], kEigMaxD, d, eps_sign);
        for (int i = 0; i < d; ++i) sm.fb[i][off + j] *= sg;
      }
    }
    __syncwarp();
  }
  __syncthreads();

  // ---- float32 basis, signs again (float32) ----
  float* fb32 = reinterpret_cast<float*>(&sm.a[0][0]);  // [d][target], the matrix is no longer needed
  for (int e = tid; e < d * target; e += kEigThreads) {
    const int i = e / target, j = e % target;
    fb32[e] = (float)sm.fb[i][j];
  }
  __syncthreads();
  for (int j = tid; j < target; j += kEigThreads) {
    const float sg = first_significant_sign<float>(fb32 + j, target, d, (float)eps_sign);
    for (int i = 0; i < d; ++i) fb32[i * target + j] *= sg;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kEigThreads) block_commit_eig_kernel(
    const float* __restrict__ projector_sum, const float* __restrict__ reduced_sum, int d, float count, int rank,
    int target, double eps_sign, float* __restrict__ summary_basis, float* __restrict__ reduced_mean,
    float* __restrict__ top_vector, float* __restrict__ average_projector) {
  extern __shared__ __align__(16) unsigned char dyn_raw[];
  EigSmem& sm = *reinterpret_cast<EigSmem*>(dyn_raw);
  const int64_t s = blockIdx.x;
  const int tid = threadIdx.x;
  const int n = d + (d & 1);  // even order for the tournament; a padded index is isolated
  const float* ps = projector_sum + s * (int64_t)d * d;

  // ---- average projector (float32), symmetrised in float32, widened ----
  float* avg = reinterpret_cast<float*>(&sm.v[0][0]);  // scratch until V is set up
  for (int e = tid; e < d * d; e += kEigThreads) {
    const float x = __fdiv_rn(ps[e], count);
    avg[e] = x;
    average_projector[s * (int64_t)d * d + e] = x;
  }
  for (int i = tid; i < d; i += kEigThreads)
    reduced_mean[s * d + i] = __fdiv_rn(reduced_sum[s * d + i], count);
  if (tid == 0) sm.fail = 0;
  __syncthreads();
  for (int e = tid; e < n * n; e += kEigThreads) {
    const int i = e / n, j = e % n;
    sm.a[i][j] = (i < d && j < d) ? (double)(0.5f * __fadd_rn(avg[i * d + j], avg[j * d + i])) : 0.0;
  }
  __syncthreads();
  canonical_top_basis(sm, d, target, eps_sign);
  const float* fb32 = reinterpret_cast<const float*>(&sm.a[0][0]);
  for (int e = tid; e < d * rank; e += kEigThreads) {
    const int i = e / rank, j = e % rank;
    summary_basis[s * (int64_t)d * rank + e] = fb32[i * target + j];
  }
  for (int i = tid; i < d; i += kEigThreads) top_vector[s * d + i] = fb32[i * target];
  if (tid == 0 && sm.fail) atomicExch(&g_commit_error, (unsigned)GFST_ERR_NUMERIC);
}


// ---------------------------------------------------------------------------
// global sketch features (one CTA per (stream, query))
// ---------------------------------------------------------------------------
// weights = softmax(scores * temperature) over the valid selections; sketch =
// sum_k w_k P[idx_k] (float32, k in order); the canonical top basis B of the
// sketch as above; for each flag dim m: P_m = B[:, :m] B[:, :m]^T and
// c_m = x^T P_m x / (x . x + eps); features = (c_m, c_m - c_{m-1}) pairs.
__global__ void __launch_bounds__(kEigThreads) global_features_kernel(
    const float* __restrict__ bank, const int32_t* __restrict__ sel_idx, const float* __restrict__ sel_scores,
    const float* __restrict__ X, int n_queries, int n_blocks, int d, int k, float temperature, int rank, int target,
    GlobalDims dims, float eps, double eps_sign, float* __restrict__ features, float* __restrict__ sketch_out,
    float* __restrict__ basis_out) {
  extern __shared__ __align__(16) unsigned char dyn_raw[];
  EigSmem& sm = *reinterpret_cast<EigSmem*>(dyn_raw);
  __shared__ float w[32];
  __shared__ int bidx[32];
  __shared__ float xs[kEigMaxD], ys[kEigMaxD];
  __shared__ int n_sel;
  const int64_t sq = blockIdx.x;  // (stream, query)
  const int64_t s = sq / n_queries;
  const int tid = threadIdx.x;
  const int n = d + (d & 1);
  // softmax over the valid selections (float32, max-subtracted)
  if (tid == 0) {
    int m = 0;
    float mx = -INFINITY;
    for (int j = 0; j < k; ++j) {
      const int b = sel_idx[sq * k + j];
      if (b >= 0 && b < n_blocks) {
        const float z = sel_scores[sq * k + j] * temperature;
        bidx[m] = b;
        w[m] = z;
        mx = fmaxf(mx, z);
        ++m;
      }
    }
    float sum = 0.f;
    for (int j = 0; j < m; ++j) {
      w[j] = expf(w[j] - mx);
      sum += w[j];
    }
    for (int j = 0; j < m; ++j) w[j] = w[j] / sum;
    n_sel = m;
    sm.fail = 0;
  }
  for (int i = tid; i < d; i += kEigThreads) xs[i] = X[sq * d + i];
  __syncthreads();
  const int m = n_sel;
  float* sketch = reinterpret_cast<float*>(&sm.v[0][0]);  // scratch until V is set up
  for (int e = tid; e < d * d; e += kEigThreads) {
    float acc = 0.f;
    for (int j = 0; j < m; ++j) acc = __fadd_rn(acc, __fmul_rn(w[j], bank[((int64_t)s * n_blocks + bidx[j]) * d * d + e]));
    sketch[e] = acc;
    if (sketch_out != nullptr) sketch_out[sq * d * d + e] = acc;
  }
  __syncthreads();
  for (int e = tid; e < n * n; e += kEigThreads) {
    const int i = e / n, j = e % n;
    sm.a[i][j] = (i < d && j < d) ? (double)(0.5f * __fadd_rn(sketch[i * d + j], sketch[j * d + i])) : 0.0;
  }
  __syncthreads();
  canonical_top_basis(sm, d, target, eps_sign);
  const float* fb32 = reinterpret_cast<const float*>(&sm.a[0][0]);
  if (basis_out != nullptr)
    for (int e = tid; e < d * rank; e += kEigThreads) basis_out[sq * d * rank + e] = fb32[(e / rank) * target + e % rank];
  // x^T P_m x for every flag dim m (P_m formed entry by entry, column order)
  float prev = 0.f;
  float xx = 0.f;
  for (int i = 0; i < d; ++i) xx = fmaf(xs[i], xs[i], xx);  // same order on every thread
  const float denom = __fadd_rn(xx, eps);
  for (int f = 0; f < dims.n; ++f) {
    const int mdim = dims.v[f];
    for (int i = tid; i < d; i += kEigThreads) {
      float y = 0.f;
      for (int j = 0; j < d; ++j) {
        float pij = 0.f;
        for (int c = 0; c < mdim; ++c) pij = fmaf(fb32[i * target + c], fb32[j * target + c], pij);
        y = fmaf(pij, xs[j], y);
      }
      ys[i] = y;
    }
    __syncthreads();
    if (tid == 0) {
      float num = 0.f;
      for (int i = 0; i < d; ++i) num = fmaf(xs[i], ys[i], num);
      const float cum = m > 0 ? __fdiv_rn(num, denom) : 0.f;
      features[sq * 2 * dims.n + 2 * f] = cum;
      features[sq * 2 * dims.n + 2 * f + 1] = __fsub_rn(cum, prev);
      prev = cum;
    }
    __syncthreads();
  }
  if (tid == 0 && sm.fail) atomicExch(&g_commit_error, (unsigned)GFST_ERR_NUMERIC);
}

// ---------------------------------------------------------------------------
// batched symmetric eigendecomposition (one CTA per matrix)
// ---------------------------------------------------------------------------
// The lower triangle of each d x d matrix (LAPACK's uplo = 'L'), widened to
// float64; eigenvalues ascending; column j of the eigenvector matrix belongs
// to eigenvalue j, its sign fixed so that its largest-magnitude entry (the
// lowest index among equal magnitudes) is positive.
template <typename T>
__global__ void __launch_bounds__(kEigThreads) heev_kernel(const T* __restrict__ A, int d, T* __restrict__ eigvals,
                                                           T* __restrict__ eigvecs, int32_t* __restrict__ info) {
  extern __shared__ __align__(16) unsigned char dyn_raw[];
  EigSmem& sm = *reinterpret_cast<EigSmem*>(dyn_raw);
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  const int n = d + (d & 1);
  const T* a = A + b * (int64_t)d * d;
  if (tid == 0) sm.fail = 0;
  for (int e = tid; e < n * n; e += kEigThreads) {
    const int i = e / n, j = e % n;
    sm.a[i][j] = (i < d && j < d) ? (double)(i >= j ? a[i * d + j] : a[j * d + i]) : 0.0;
  }
  __syncthreads();
  jacobi_eigen(sm, d);
  for (int j = tid; j < d; j += kEigThreads) {
    const int src = sm.order[j];
    eigvals[b * d + j] = (T)sm.a[src][src];
    int imax = 0;
    double vmax = -1.0;
    for (int i = 0; i < d; ++i) {
      const double x = fabs(sm.v[i][src]);
      if (x > vmax) {
        vmax = x;
        imax = i;
      }
    }
    const double sg = sm.v[imax][src] < 0.0 ? -1.0 : 1.0;
    for (int i = 0; i < d; ++i) eigvecs[b * (int64_t)d * d + i * d + j] = (T)(sg * sm.v[i][src]);
  }
  if (tid == 0) {
    if (info != nullptr) info[b] = sm.fail ? 1 : 0;
    if (sm.fail) atomicExch(&g_commit_error, (unsigned)GFST_ERR_NUMERIC);
  }
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_block_commit_eig(const float* projector_sum, const float* reduced_sum, int64_t n_streams, int d,
                                     int token_count, int max_flag_dim, const int32_t* flag_dims, int n_flags,
                                     double eps_sign, float* summary_basis, float* reduced_mean, float* top_vector,
                                     float* average_projector, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(d >= 1 && d <= kEigMaxD, GFST_ERR_SHAPE, "d=%d outside [1, %d]", d, kEigMaxD);
  GFST_REQUIRE(token_count >= 1, GFST_ERR_ARG, "token_count must be >= 1");
  GFST_REQUIRE(max_flag_dim >= 1 && max_flag_dim <= d, GFST_ERR_SHAPE, "max_flag_dim=%d outside [1, d]",
               max_flag_dim);
  GFST_REQUIRE(n_flags >= 0 && (n_flags == 0 || flag_dims != nullptr), GFST_ERR_ARG, "flag_dims missing");
  int target = max_flag_dim;
  for (int i = 0; i < n_flags; ++i) {
    GFST_REQUIRE(flag_dims[i] >= 0 && flag_dims[i] <= d, GFST_ERR_SHAPE, "flag dim %d outside [0, d]", flag_dims[i]);
    target = flag_dims[i] > target ? flag_dims[i] : target;
  }
  if (n_streams == 0) return GFST_OK;
  GFST_REQUIRE(projector_sum && reduced_sum && summary_basis && reduced_mean && top_vector && average_projector,
               GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(n_streams <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many streams");
  const size_t smem = sizeof(EigSmem);
  cudaError_t e = cudaFuncSetAttribute(block_commit_eig_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  block_commit_eig_kernel<<<(unsigned)n_streams, kEigThreads, smem, stream>>>(
      projector_sum, reduced_sum, d, (float)token_count, max_flag_dim, target, eps_sign, summary_basis, reduced_mean,
      top_vector, average_projector);
  return check_launch("block_commit_eig_kernel");
}

extern "C" int gfst_global_features(const float* projector_bank, const int32_t* sel_idx, const float* sel_scores,
                                    const float* x, int64_t n_streams, int n_queries, int n_blocks, int d, int k,
                                    float temperature, int max_flag_dim, const int32_t* flag_dims, int n_flags,
                                    float eps, double eps_sign, float* features, float* sketch_out,
                                    float* basis_out, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_blocks >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(d >= 1 && d <= kEigMaxD, GFST_ERR_SHAPE, "d=%d outside [1, %d]", d, kEigMaxD);
  GFST_REQUIRE(k >= 1 && k <= 32, GFST_ERR_SHAPE, "k=%d outside [1, 32]", k);
  GFST_REQUIRE(max_flag_dim >= 1 && max_flag_dim <= d, GFST_ERR_SHAPE, "max_flag_dim=%d outside [1, d]",
               max_flag_dim);
  GFST_REQUIRE(n_flags >= 1 && n_flags <= 8 && flag_dims != nullptr, GFST_ERR_SHAPE, "need 1..8 flag dims");
  GlobalDims dims{};
  dims.n = n_flags;
  int target = max_flag_dim;
  for (int i = 0; i < n_flags; ++i) {
    GFST_REQUIRE(flag_dims[i] >= 1 && flag_dims[i] <= d, GFST_ERR_SHAPE, "flag dim %d outside [1, d]", flag_dims[i]);
    dims.v[i] = flag_dims[i];
    target = flag_dims[i] > target ? flag_dims[i] : target;
  }
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(sel_idx && sel_scores && x && features && (projector_bank || n_blocks == 0), GFST_ERR_ARG,
               "null buffer");
  GFST_REQUIRE(n_streams * (int64_t)n_queries <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many requests");
  const size_t smem = sizeof(EigSmem);
  cudaError_t e = cudaFuncSetAttribute(global_features_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  global_features_kernel<<<(unsigned)(n_streams * n_queries), kEigThreads, smem, stream>>>(
      projector_bank, sel_idx, sel_scores, x, n_queries, n_blocks, d, k, temperature, max_flag_dim, target, dims,
      eps, eps_sign, features, sketch_out, basis_out);
  return check_launch("global_features_kernel");
}

extern "C" int gfst_heev(const void* matrices, int64_t batch, int d, int dtype, void* eigenvalues,
                         void* eigenvectors, int32_t* info, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(batch >= 0, GFST_ERR_ARG, "negative batch");
  GFST_REQUIRE(d >= 1 && d <= kEigMaxD, GFST_ERR_SHAPE, "d=%d outside [1, %d]", d, kEigMaxD);
  GFST_REQUIRE(dtype == GFST_F32 || dtype == GFST_F64, GFST_ERR_DTYPE, "unsupported dtype %d (f32 or f64)", dtype);
  if (batch == 0) return GFST_OK;
  GFST_REQUIRE(matrices && eigenvalues && eigenvectors, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(batch <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many matrices");
  const size_t smem = sizeof(EigSmem);
  if (dtype == GFST_F32) {
    cudaError_t e = cudaFuncSetAttribute(heev_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    heev_kernel<float><<<(unsigned)batch, kEigThreads, smem, stream>>>(
        static_cast<const float*>(matrices), d, static_cast<float*>(eigenvalues), static_cast<float*>(eigenvectors),
        info);
  } else {
    cudaError_t e = cudaFuncSetAttribute(heev_kernel<double>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    heev_kernel<double><<<(unsigned)batch, kEigThreads, smem, stream>>>(
        static_cast<const double*>(matrices), d, static_cast<double*>(eigenvalues),
        static_cast<double*>(eigenvectors), info);
  }
  return check_launch("heev_kernel");
}
