// Block token scores through the within-block projection:
//   score[t] = sum_j key[t, j] q[j],  key[t, j] = sum_c F[t, c] W[j, c]
// with, for bf16 inputs, the key rounded to bf16 (the projection's output type)
// and the score rounded to bf16 before widening -- (proj(F) @ q).float().
//
// Reference (pkhairkh/gfst-hmb-public): exact_block_project_forward
// (src/gfst_hmb_mpuc/csrc/sm120_cutlass_exact_block_score.cu:42-129, a bf16
// GEMM F W^T with fp32 accumulation and bf16 output) and the dot with the query
// in ExactRecallReadout._score_block_tokens (src/gfst_hmb_mpuc/modeling.py:640-651).
//
// bf16 with k a multiple of 64 (<= 256) and n a multiple of 16 (<= 256) runs
// on the tensor cores: a persistent CTA per SM loads W once by TMA, streams
// 128-token tiles of F through a ring (TMA, 128-byte swizzle), one thread
// issues tcgen05.mma (M = 128 tokens, N = n, K = 16) into one of two TMEM
// accumulators, and two groups of four epilogue warps (one per accumulator)
// read their token row's n keys with tcgen05.ld, round them and fold in the
// query.  Other shapes and fp32 run a
// SIMT kernel (fp32 FMAs, 16 tokens per CTA).
#include "block_topk.cuh"
#include "umma.cuh"

namespace gfst {

// sticky GFST_ERR_TIMEOUT report of the tensor-core block-score kernel
GFST_DEFINE_ERROR_WORD(g_score_error, read_score_error, "block score")

namespace {

// ---------------------------------------------------------------------------
// SIMT kernel (fp32, and bf16 shapes the tensor-core kernel does not take)
// ---------------------------------------------------------------------------
constexpr int kBsRows = 16;  // token rows per CTA
constexpr int kBsThreads = 256;
constexpr int kBsK = 64;  // feature columns per shared-memory tile

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(v);
  else return v;
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

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
  // thread j owns key column j (and j + 256, ...) of every row
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
        const float key = sizeof(T) == 2 ? round_bf16(acc[i]) : acc[i];
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
    scores[r0 + tid] = sizeof(T) == 2 ? round_bf16(s) : s;
  }
}

// ---------------------------------------------------------------------------
// tensor-core kernel (bf16)
// ---------------------------------------------------------------------------
constexpr int kTileRows = 128;  // tokens per tile = TMEM lanes
constexpr int kBoxBytes = kTileRows * 128;  // one 64-column box of a tile
// two epilogue groups of four warps (group g reads accumulator g, so the two
// accumulators' tiles are rounded and reduced concurrently), then the TMA
// producer warp and the MMA warp
constexpr int kGroupWarps = 4, kEpiWarps = 8, kProducerWarp = 8, kMmaWarp = 9, kTcThreads = 320;
constexpr int kMaxStages = 4;
constexpr int kSmemBudget = 220 * 1024;

struct ScoreLayout {
  int w_bytes, tile_bytes, bar_off, q_off, total;
};

// W boxes, the F ring, barriers (full[S], empty[S], tfull[2], tempty[2], wfull,
// done), the TMEM slot and three flags, then the query as fp32.
__host__ __device__ inline ScoreLayout score_layout(int nkb, int n, int stages) {
  ScoreLayout L;
  L.w_bytes = nkb * n * 128;
  L.tile_bytes = nkb * kBoxBytes;
  L.bar_off = L.w_bytes + stages * L.tile_bytes;
  L.q_off = L.bar_off + (2 * stages + 6) * 8 + 16;
  L.total = 1024 + L.q_off + n * 4;
  return L;
}

template <int NKB>
__global__ void __launch_bounds__(kTcThreads, 1)
    block_score_tc_kernel(const __grid_constant__ CUtensorMap tmF, const __grid_constant__ CUtensorMap tmW,
                          const __nv_bfloat16* __restrict__ q, int64_t m, int n, int stages, uint32_t acc_stride,
                          uint32_t tmem_cols, float* __restrict__ scores) {
  const ScoreLayout LY = score_layout(NKB, n, stages);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sF = smem + LY.w_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY.bar_off);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* wfull = tempty + 2;
  uint64_t* done = wfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_issued = const_cast<int*>(abort_flag + 1);
  int* n_consumed = n_issued + 1;
  float* qs = reinterpret_cast<float*>(smem + LY.q_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_tiles = (m + kTileRows - 1) / kTileRows;
  const int my_tiles = (int64_t)blockIdx.x < n_tiles ? (int)((n_tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

  for (int j = threadIdx.x; j < n; j += kTcThreads) qs[j] = __bfloat162float(q[j]);
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kGroupWarps);
    }
    mbar_init(wfull, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    mbar_init_fence();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      mbar_arrive_expect_tx(wfull, (uint32_t)LY.w_bytes);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) tma_load_2d(sW + kb * n * 128, &tmW, wfull, kb * 64, 0);
      int i = 0;
      for (; i < my_tiles; ++i) {
        const int st = i % stages;
        if (!mbar_wait(&empty[st], ((i / stages) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int row0 = (int)(((int64_t)blockIdx.x + (int64_t)i * gridDim.x) * kTileRows);
        mbar_arrive_expect_tx(&full[st], (uint32_t)LY.tile_bytes);
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb)
          tma_load_2d(sF + (st * NKB + kb) * kBoxBytes, &tmF, &full[st], kb * 64, row0);
      }
      *n_issued = i;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTileRows, n);
      int i = 0;
      if (!mbar_wait(wfull, 0)) {
        *abort_flag = 1;
      } else {
        for (; i < my_tiles; ++i) {
          const int st = i % stages, acc = i & 1;
          if (!mbar_wait(&tempty[acc], ((i >> 1) & 1) ^ 1) || !mbar_wait(&full[st], (i / stages) & 1)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)acc * acc_stride;
#pragma unroll
          for (int kk = 0; kk < NKB * 4; ++kk) {
            const int kb = kk >> 2, koff = (kk & 3) * 32;
            const uint64_t ad = sw128_desc(smem_u32(sF + (st * NKB + kb) * kBoxBytes) + koff);
            const uint64_t bd = sw128_desc(smem_u32(sW + kb * n * 128) + koff);
            umma_bf16(d_tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty[st]);
          umma_commit(&tfull[acc]);
        }
      }
      *n_consumed = i;
      umma_commit(done);  // arrives once every MMA issued above has completed
    }
  } else {
    // epilogue: warp w owns TMEM lane quadrant w % 4 (thread = token row) of
    // accumulator w / 4, i.e. of tiles i = w / 4, w / 4 + 2, ...
    const int quad = warp & 3, acc = warp >> 2;
    for (int i = acc; i < my_tiles; i += 2) {
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(&tfull[acc], (i >> 1) & 1) ? 1 : 0;
        if (!ok) *abort_flag = 1;
        if (*abort_flag) ok = 0;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)acc * acc_stride;
      // 64 columns per TMEM wait; four partial sums break the FMA chain
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c0 = 0; c0 < n; c0 += 64) {
        float v[64];
#pragma unroll
        for (int h = 0; h < 4; ++h)
          if (c0 + 16 * h < n) tmem_ld16(taddr + c0 + 16 * h, v + 16 * h);  // n % 16 == 0: uniform
        tmem_wait_ld();
        const float4* q4 = reinterpret_cast<const float4*>(qs + c0);
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          if (c0 + c < n) {
            const float4 qv = q4[c >> 2];
            // keys rounded to bf16 two at a time (cvt.rn.bf16x2.f32)
            const __nv_bfloat162 k01 = __floats2bfloat162_rn(v[c], v[c + 1]);
            const __nv_bfloat162 k23 = __floats2bfloat162_rn(v[c + 2], v[c + 3]);
            s4[0] = fmaf(__low2float(k01), qv.x, s4[0]);
            s4[1] = fmaf(__high2float(k01), qv.y, s4[1]);
            s4[2] = fmaf(__low2float(k23), qv.z, s4[2]);
            s4[3] = fmaf(__high2float(k23), qv.w, s4[3]);
          }
        }
      }
      const float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);  // accumulator free for tile i + 2
      const int64_t row = ((int64_t)blockIdx.x + (int64_t)i * gridDim.x) * kTileRows + quad * 32 + lane;
      if (row < m) scores[row] = round_bf16(s);
    }
  }
  __syncthreads();
  if (threadIdx.x == 32 * kProducerWarp) {
    // drain copies that were issued but never consumed (only after a timeout)
    for (int i = *n_consumed; i < *n_issued; ++i) mbar_wait(&full[i % stages], (i / stages) & 1);
    if (*abort_flag) mbar_wait(wfull, 0);
  }
  if (warp == kMmaWarp) {
    if (!mbar_wait(done, 0)) *abort_flag = 1;
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_score_error, (unsigned)GFST_ERR_TIMEOUT);
}

template <int NKB>
int launch_tc(const void* q, const void* F, const void* W, int64_t m, int n, int k, float* scores,
              cudaStream_t stream) {
  int stages = 0;
  for (int s = kMaxStages; s >= 2 && stages == 0; --s)
    if (score_layout(NKB, n, s).total <= kSmemBudget) stages = s;
  if (stages == 0) return -1;  // does not fit: the caller takes the SIMT kernel
  CUtensorMap mf, mw;
  int st = make_bf16_map(&mf, F, (uint64_t)m, k, kTileRows);
  if (st != GFST_OK) return st;
  st = make_bf16_map(&mw, W, (uint64_t)n, k, n);
  if (st != GFST_OK) return st;
  uint32_t acc_stride = 16;
  while ((int)acc_stride < n) acc_stride <<= 1;
  const uint32_t tmem_cols = acc_stride * 2 < 32 ? 32 : acc_stride * 2;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "device query: %s", cudaGetErrorString(e));
  const ScoreLayout LY = score_layout(NKB, n, stages);
  auto kern = block_score_tc_kernel<NKB>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, LY.total);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int64_t n_tiles = (m + kTileRows - 1) / kTileRows;
  const unsigned grid = (unsigned)(n_tiles < sms ? n_tiles : sms);
  kern<<<grid, kTcThreads, LY.total, stream>>>(mf, mw, static_cast<const __nv_bfloat16*>(q), m, n, stages,
                                               acc_stride, tmem_cols, scores);
  return check_launch("block_score_tc_kernel");
}

int launch_tc_any(const void* q, const void* F, const void* W, int64_t m, int n, int k, float* scores,
                  cudaStream_t stream) {
  switch (k / 64) {
    case 1: return launch_tc<1>(q, F, W, m, n, k, scores, stream);
    case 2: return launch_tc<2>(q, F, W, m, n, k, scores, stream);
    case 3: return launch_tc<3>(q, F, W, m, n, k, scores, stream);
    default: return launch_tc<4>(q, F, W, m, n, k, scores, stream);
  }
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_exact_block_score(const void* query, const void* token_features, const void* weight, int64_t m,
                                      int n, int k, int dtype, float* scores, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(m >= 0 && n >= 1 && k >= 1, GFST_ERR_ARG, "bad sizes (m=%lld n=%d k=%d)", (long long)m, n, k);
  if (m == 0) return GFST_OK;
  GFST_REQUIRE(query && token_features && weight && scores, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(dtype == GFST_F32 || dtype == GFST_BF16, GFST_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (dtype == GFST_BF16 && k % 64 == 0 && k <= 256 && n % 16 == 0 && n <= 256 && m < (1LL << 31) &&
      aligned16(token_features) && aligned16(weight)) {
    const int st = launch_tc_any(query, token_features, weight, m, n, k, scores, stream);
    if (st >= 0) return st;
  }
  const int64_t grid = (m + kBsRows - 1) / kBsRows;
  GFST_REQUIRE(grid <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many rows");
  if (dtype == GFST_BF16) {
    block_score_kernel<__nv_bfloat16><<<(unsigned)grid, kBsThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(query), static_cast<const __nv_bfloat16*>(token_features),
        static_cast<const __nv_bfloat16*>(weight), m, n, k, scores);
  } else {
    block_score_kernel<float><<<(unsigned)grid, kBsThreads, 0, stream>>>(
        static_cast<const float*>(query), static_cast<const float*>(token_features),
        static_cast<const float*>(weight), m, n, k, scores);
  }
  return check_launch("block_score_kernel");
}
