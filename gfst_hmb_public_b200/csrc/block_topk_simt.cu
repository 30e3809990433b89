// Coarse block retrieval on CUDA cores (fp32 FMA): score every committed block
// summary against each query and keep the k best in the total order
// (score descending, block index ascending).
//
// Reference: FaissGpuRetriever.exact_topk / search
// (src/gfst_hmb_mpuc/retrieval.py:136-172 of pkhairkh/gfst-hmb-public), which
// scores keys @ q in float32 and takes torch.topk.  This kernel serves fp32
// memories: their products must stay exact fp32, which the bf16 tensor-core
// path (block_topk_tc.cu) cannot give.
//
// One thread per query: the CTA stages its 128 queries transposed in shared
// memory (conflict-free per-thread reads) and streams the stream's summaries
// through a shared tile (broadcast reads).  Each (query, block) score is a
// sequential fp32 FMA chain over d; each thread keeps a sorted top-k list and
// inserts blocks in increasing index order.
#include "block_topk.cuh"

namespace gfst {
namespace {

constexpr int kQ = 128;     // queries (threads) per CTA
constexpr int kTile = 16;   // summaries per shared tile

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p);
template <>
__device__ __forceinline__ float ld_f32<float>(const float* p) { return __ldg(p); }

template <typename T, int KCAP>
__global__ void __launch_bounds__(kQ) block_topk_simt_kernel(const T* __restrict__ Q, const T* __restrict__ Ksum,
                                                             int n_queries, int n_blocks, int n_blocks_stride,
                                                             int d, int k, float* __restrict__ top_scores,
                                                             int32_t* __restrict__ top_idx) {
  extern __shared__ __align__(16) float smem[];
  float* qT = smem;                    // [d][kQ]
  float* kb = smem + (size_t)d * kQ;   // [kTile][d]
  const int64_t s = blockIdx.y;
  const int q0 = blockIdx.x * kQ;
  const int tid = threadIdx.x;
  const T* Qs = Q + ((size_t)s * n_queries) * d;
  const T* Ks = Ksum + ((size_t)s * n_blocks_stride) * d;

  for (int e = tid; e < kQ * d; e += kQ) {
    const int qq = e / d, c = e % d;
    qT[(size_t)c * kQ + qq] = (q0 + qq < n_queries) ? ld_f32(Qs + (size_t)(q0 + qq) * d + c) : 0.f;
  }

  TopK<KCAP> top;
  top.init();

  for (int b0 = 0; b0 < n_blocks; b0 += kTile) {
    __syncthreads();
    for (int e = tid; e < kTile * d; e += kQ) {
      const int bb = e / d, c = e % d;
      kb[e] = (b0 + bb < n_blocks) ? ld_f32(Ks + (size_t)(b0 + bb) * d + c) : 0.f;
    }
    __syncthreads();
    float acc[kTile];
#pragma unroll
    for (int j = 0; j < kTile; ++j) acc[j] = 0.f;
    for (int c = 0; c < d; c += 4) {
      const float q_0 = qT[(size_t)(c + 0) * kQ + tid];
      const float q_1 = qT[(size_t)(c + 1) * kQ + tid];
      const float q_2 = qT[(size_t)(c + 2) * kQ + tid];
      const float q_3 = qT[(size_t)(c + 3) * kQ + tid];
#pragma unroll
      for (int j = 0; j < kTile; ++j) {
        const float4 kv = *reinterpret_cast<const float4*>(kb + j * d + c);
        acc[j] = fmaf(q_0, kv.x, acc[j]);
        acc[j] = fmaf(q_1, kv.y, acc[j]);
        acc[j] = fmaf(q_2, kv.z, acc[j]);
        acc[j] = fmaf(q_3, kv.w, acc[j]);
      }
    }
    top.offer16(acc, b0, n_blocks);
  }

  const int q = q0 + tid;
  if (q < n_queries) {
    top.write(top_scores + ((size_t)s * n_queries + q) * k, top_idx + ((size_t)s * n_queries + q) * k, k);
  }
}

template <typename T, int KCAP>
int launch_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, float* ts,
                int32_t* ti, cudaStream_t stream) {
  const size_t smem = ((size_t)d * kQ + (size_t)kTile * d) * sizeof(float);
  auto kern = block_topk_simt_kernel<T, KCAP>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  GFST_REQUIRE(S <= 65535, GFST_ERR_SHAPE, "n_streams %lld exceeds 65535", (long long)S);
  dim3 grid((unsigned)((Nq + kQ - 1) / kQ), (unsigned)S);
  kern<<<grid, kQ, smem, stream>>>(static_cast<const T*>(Q), static_cast<const T*>(Ksum), Nq, NB, NBs, d, k, ts,
                                   ti);
  return check_launch("block_topk_simt_kernel");
}

}  // namespace

int block_topk_simt(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, int dtype,
                    float* ts, int32_t* ti, cudaStream_t stream) {
  GFST_REQUIRE(d % 4 == 0, GFST_ERR_SHAPE, "d=%d must be a multiple of 4", d);
  (void)dtype;
  if (k <= 2) return launch_simt<float, 2>(Q, Ksum, S, Nq, NB, NBs, d, k, ts, ti, stream);
  if (k <= 4) return launch_simt<float, 4>(Q, Ksum, S, Nq, NB, NBs, d, k, ts, ti, stream);
  if (k <= 8) return launch_simt<float, 8>(Q, Ksum, S, Nq, NB, NBs, d, k, ts, ti, stream);
  if (k <= 16) return launch_simt<float, 16>(Q, Ksum, S, Nq, NB, NBs, d, k, ts, ti, stream);
  return launch_simt<float, 32>(Q, Ksum, S, Nq, NB, NBs, d, k, ts, ti, stream);
}

}  // namespace gfst
