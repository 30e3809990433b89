// Open-block readout: the exact readout over the prefix of the block that is
// still being written, merged into the result over the committed blocks.
//
// Reference (pkhairkh/gfst-hmb-public): each token is appended to the exact
// store (src/gfst_hmb_mpuc/modeling.py:3807, state.py:651-815) before the
// retrieval of the same token (modeling.py:3853), and the readout appends the
// current block with its prefix length to the retrieved blocks
// (modeling.py:2948-2963), so a query scores positions [0, t] of its own block.
// When t is the block's last position, append_exact_token has already closed
// the block (state.py:749-815) while its summary is appended only after the
// retrieval (modeling.py:3632), so that query sees neither.
//
// One CTA per (stream, chunk of 64 queries): the queries and 64-position
// chunks of the open block are staged in shared memory as fp32 (rows padded by
// 4 floats, so a quarter-warp's float4 reads of 8 consecutive rows hit all 32
// banks once), each warp scores 8 queries against the chunk's 64 positions
// (two positions per lane, fp32 FMAs), then a warp butterfly picks each
// query's best open position in the total order (score descending, position
// ascending; NaN scores never win) and the winner replaces the committed
// result when it ranks first in (score descending, token index ascending).
#include "gfst_common.cuh"

namespace gfst {
namespace {

constexpr int kOQ = 64;               // queries per CTA
constexpr int kOWarps = 8;            // warps per CTA
constexpr int kOQW = kOQ / kOWarps;   // queries per warp
constexpr int kOKC = 64;              // open positions per shared-memory chunk (two per lane)
constexpr int kOThreads = kOWarps * 32;

template <typename T>
__device__ __forceinline__ float load_f32(const T* p);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) { return bf16_to_f32(*p); }

// (score, position) pair with position -1 = nothing yet; NaN never enters
__device__ __forceinline__ void offer(float s, int p, float& bs, int& bp) {
  if (s != s) return;
  if (bp < 0 || better(s, p, bs, bp)) {
    bs = s;
    bp = p;
  }
}

__device__ __forceinline__ void warp_best_pair(float& bs, int& bp) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, bs, o);
    const int op = __shfl_xor_sync(0xffffffffu, bp, o);
    if (op >= 0 && (bp < 0 || better(os, op, bs, bp))) {
      bs = os;
      bp = op;
    }
  }
}

// rows [0, n) of a [*, d] matrix into shared memory as fp32 rows of pitch dp
// (rows n..nrows-1 zero).  16-byte vectors when d and the source line up, with
// every vector load of a thread issued before its stores so the loads overlap.
template <typename T>
__device__ __forceinline__ void stage_rows(float* dst, const T* src, int n, int nrows, int d, int dp, bool vec) {
  const int tid = threadIdx.x;
  if (vec) {
    constexpr int V = 16 / sizeof(T);
    const int vpr = d / V;  // vectors per row
    const int total = nrows * vpr;
    for (int base = 0; base < total; base += 4 * kOThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kOThreads + tid;
        const int r = i / vpr;
        v[u] = (i < total && r < n) ? __ldg(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = base + u * kOThreads + tid;
        if (i >= total) continue;
        const int r = i / vpr, c = (i - r * vpr) * V;
        float* o = dst + r * dp + c;
        if constexpr (sizeof(T) == 4) {
          *reinterpret_cast<float4*>(o) = make_float4(__uint_as_float(v[u].x), __uint_as_float(v[u].y),
                                                      __uint_as_float(v[u].z), __uint_as_float(v[u].w));
        } else {
          *reinterpret_cast<float4*>(o) = make_float4(bf16_lo(v[u].x), bf16_hi(v[u].x), bf16_lo(v[u].y),
                                                      bf16_hi(v[u].y));
          *reinterpret_cast<float4*>(o + 4) = make_float4(bf16_lo(v[u].z), bf16_hi(v[u].z), bf16_lo(v[u].w),
                                                          bf16_hi(v[u].w));
        }
      }
    }
    return;
  }
  for (int i = tid; i < nrows * d; i += kOThreads) {
    const int r = i / d, c = i - r * d;
    dst[r * dp + c] = r < n ? load_f32<T>(src + (int64_t)r * d + c) : 0.f;
  }
}

__device__ __forceinline__ int open_len_of(const int32_t* open_len, int64_t row, int q, int Lo) {
  if (open_len == nullptr) return q < Lo - 1 ? q + 1 : 0;
  const int n = open_len[row];
  return n < 0 ? 0 : (n > Lo ? Lo : n);
}

template <typename T>
__global__ void __launch_bounds__(kOThreads) open_block_readout_kernel(
    const T* __restrict__ Q, const T* __restrict__ Ko, const T* __restrict__ Vo,
    const int32_t* __restrict__ open_len, int Nq, int n_chunks, int Lo, int d, int dv, int64_t open_base,
    bool vec, int32_t* __restrict__ best_tok, float* __restrict__ best_score, T* __restrict__ out_V) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  __shared__ int s_nmax;
  const int dp = d + 4;
  float* sq = sm;               // [kOQ][dp]
  float* sk = sm + kOQ * dp;    // [kOKC][dp]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t s = blockIdx.x / n_chunks;
  const int q0 = (int)(blockIdx.x % n_chunks) * kOQ;
  const int nq = min(kOQ, Nq - q0);
  const int64_t row0 = s * (int64_t)Nq + q0;

  if (tid == 0) s_nmax = 0;
  __syncthreads();
  if (tid < nq) atomicMax(&s_nmax, open_len_of(open_len, row0 + tid, q0 + tid, Lo));
  // queries of the chunk as fp32 (rows past nq are zero)
  stage_rows<T>(sq, Q + row0 * d, nq, kOQ, d, dp, vec);
  __syncthreads();
  const int n_max = s_nmax;
  if (n_max == 0) return;

  int len[kOQW];
  float bs[kOQW];
  int bp[kOQW];
#pragma unroll
  for (int j = 0; j < kOQW; ++j) {
    const int ql = warp * kOQW + j;
    len[j] = ql < nq ? open_len_of(open_len, row0 + ql, q0 + ql, Lo) : 0;
    bs[j] = -INFINITY;
    bp[j] = -1;
  }
  const T* ksrc = Ko + s * (int64_t)Lo * d;
  for (int c0 = 0; c0 < n_max; c0 += kOKC) {
    const int nk = min(kOKC, n_max - c0);
    __syncthreads();  // the previous chunk has been read
    stage_rows<T>(sk, ksrc + (int64_t)c0 * d, nk, kOKC, d, dp, vec);
    __syncthreads();
    float a0[kOQW], a1[kOQW];
#pragma unroll
    for (int j = 0; j < kOQW; ++j) a0[j] = a1[j] = 0.f;
    const float* k0 = sk + lane * dp;
    const float* k1 = sk + (lane + 32) * dp;
    const float* qw = sq + warp * kOQW * dp;
    for (int c = 0; c < d; c += 4) {
      const float4 x0 = *reinterpret_cast<const float4*>(k0 + c);
      const float4 x1 = *reinterpret_cast<const float4*>(k1 + c);
#pragma unroll
      for (int j = 0; j < kOQW; ++j) {
        const float4 qv = *reinterpret_cast<const float4*>(qw + j * dp + c);
        a0[j] = fmaf(x0.x, qv.x, a0[j]);
        a0[j] = fmaf(x0.y, qv.y, a0[j]);
        a0[j] = fmaf(x0.z, qv.z, a0[j]);
        a0[j] = fmaf(x0.w, qv.w, a0[j]);
        a1[j] = fmaf(x1.x, qv.x, a1[j]);
        a1[j] = fmaf(x1.y, qv.y, a1[j]);
        a1[j] = fmaf(x1.z, qv.z, a1[j]);
        a1[j] = fmaf(x1.w, qv.w, a1[j]);
      }
    }
    const int p0 = c0 + lane, p1 = c0 + lane + 32;
#pragma unroll
    for (int j = 0; j < kOQW; ++j) {
      if (p0 < len[j]) offer(a0[j], p0, bs[j], bp[j]);
      if (p1 < len[j]) offer(a1[j], p1, bs[j], bp[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < kOQW; ++j) {
    warp_best_pair(bs[j], bp[j]);
    const int ql = warp * kOQW + j;
    if (ql >= nq || bp[j] < 0) continue;  // warp-uniform
    const int64_t row = row0 + ql;
    const int ot = (int)(open_base + bp[j]);
    const int ct = best_tok[row];
    const float cs = best_score[row];
    const bool wins = ct < 0 || better(bs[j], ot, cs, ct);
    if (!wins) continue;
    __syncwarp();
    if (lane == 0) {
      best_tok[row] = ot;
      best_score[row] = bs[j];
    }
    if (out_V != nullptr) {
      const T* src = Vo + (s * (int64_t)Lo + bp[j]) * dv;
      T* dst = out_V + row * dv;
      for (int c = lane; c < dv; c += 32) dst[c] = src[c];
    }
  }
}

template <typename T>
int launch_open(const void* Q, const void* Ko, const void* Vo, const int32_t* open_len, int64_t S, int Nq, int Lo,
                int d, int dv, int64_t open_base, int32_t* best_tok, float* best_score, void* out_V,
                cudaStream_t stream) {
  const int64_t n_chunks = (Nq + kOQ - 1) / kOQ;
  GFST_REQUIRE(S * n_chunks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many query chunks");
  const size_t dyn = (size_t)(kOQ + kOKC) * (d + 4) * sizeof(float);
  // 16-byte vector staging: rows of whole vectors and 16-byte aligned bases
  const bool vec = (d * sizeof(T)) % 16 == 0 && aligned16(Q) && aligned16(Ko);
  auto kern = open_block_readout_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)(S * n_chunks), kOThreads, dyn, stream>>>(
      static_cast<const T*>(Q), static_cast<const T*>(Ko), static_cast<const T*>(Vo), open_len, Nq, (int)n_chunks,
      Lo, d, dv, open_base, vec, best_tok, best_score, static_cast<T*>(out_V));
  return check_launch("open_block_readout_kernel");
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_open_block_readout(const void* Q, const void* K_open, const void* V_open,
                                       const int32_t* open_len, int64_t n_streams, int n_queries, int L_open, int d,
                                       int dv, int64_t open_base, int dtype, int32_t* best_tok, float* best_score,
                                       void* out_V, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && L_open >= 0 && dv >= 0, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(d >= 4 && d <= 256 && d % 4 == 0, GFST_ERR_SHAPE, "d=%d must be a multiple of 4 in [4, 256]", d);
  GFST_REQUIRE(open_base >= 0 && open_base + (int64_t)L_open <= 0x7fffffffLL, GFST_ERR_SHAPE,
               "open token index overflows int32");
  GFST_REQUIRE((V_open == nullptr) == (out_V == nullptr), GFST_ERR_ARG, "V_open and out_V go together");
  if (n_streams == 0 || n_queries == 0 || L_open == 0) return GFST_OK;
  GFST_REQUIRE(Q && K_open && best_tok && best_score, GFST_ERR_ARG, "null buffer");
  if (dtype == GFST_F32)
    return launch_open<float>(Q, K_open, V_open, open_len, n_streams, n_queries, L_open, d, dv, open_base, best_tok,
                              best_score, out_V, stream);
  if (dtype == GFST_BF16)
    return launch_open<__nv_bfloat16>(Q, K_open, V_open, open_len, n_streams, n_queries, L_open, d, dv, open_base,
                                      best_tok, best_score, out_V, stream);
  set_last_error("unsupported dtype %d", dtype);
  return GFST_ERR_DTYPE;
}
