// Coarse block retrieval on the 5th-generation tensor cores (bf16 operands,
// fp32 accumulation in TMEM): scores = Q K_sum^T per stream, fused with a
// per-query top-k in the total order (score descending, block index ascending).
//
// Reference: FaissGpuRetriever.exact_topk / search
// (src/gfst_hmb_mpuc/retrieval.py:136-172 of pkhairkh/gfst-hmb-public) scores
// keys @ q and takes torch.topk; this is the same selection batched over all
// queries of a stream, with the score matrix never leaving the SM.
//
// One CTA per (stream, 128-query tile), 10 warps:
//   warp 8  TMA producer: the query tile once, then 128-summary tiles into a
//           STAGES-deep ring of 128B-swizzled shared-memory buffers
//   warp 9  MMA issuer: tcgen05.mma.cta_group::1.kind::f16 (M=128, N=128, K=16)
//           into one of two TMEM accumulators (2 x 128 fp32 columns), then
//           tcgen05.commit to free the smem stage and publish the accumulator
//   warps 0-7  epilogue: warp w reads TMEM lane quadrant w % 4 (thread = query
//           row) and column half w / 4 of each accumulator with tcgen05.ld,
//           releases the accumulator and inserts the 64 scores into a register
//           top-k list; the two halves of a row are merged at the end
// Every mbarrier wait is bounded (about a second of clock cycles); a wait that
// gives up sets a sticky device error word (read with gfst_check_device_errors)
// and the CTA drains its in-flight copies and MMAs, frees TMEM and returns.
#include "block_topk.cuh"
#include "umma.cuh"

namespace gfst {

// sticky GFST_ERR_TIMEOUT report of the tensor-core retrieval and the wait probe
GFST_DEFINE_ERROR_WORD(g_device_error, read_device_error, "retrieval")

namespace {

constexpr int BM = 128;            // query rows per CTA (TMEM lanes)
constexpr int BN = 128;            // summaries per tile (TMEM columns per accumulator)
constexpr int KBOX = 64;           // bf16 elements per 128-byte swizzle row
// EPW epilogue warps (4 or 8: the TMEM lane quadrants x 1 or 2 column parts),
// then one TMA producer warp and one MMA warp
template <int EPW>
struct TcWarps {
  static_assert(EPW == 4 || EPW == 8, "4 or 8 epilogue warps");
  static constexpr int kEpiWarps = EPW;
  static constexpr int kProducerWarp = EPW;
  static constexpr int kMmaWarp = EPW + 1;
  static constexpr int kThreads = (EPW + 2) * 32;
  static constexpr int kPartN = BN / (EPW / 4);  // accumulator columns per epilogue warp
};

// kind::f16 instruction descriptor of the score tile.
constexpr uint32_t kIdesc = idesc_bf16(BM, BN);

template <int NKB, int STAGES>
struct TcLayout {
  static constexpr int A_BYTES = NKB * BM * 128;
  static constexpr int B_STAGE_BYTES = NKB * BN * 128;
  static constexpr int BAR_OFF = A_BYTES + STAGES * B_STAGE_BYTES;
  // full[S], empty[S], tfull[2], tempty[2], afull, done; then tmem slot, flags
  static constexpr int N_BARS = 2 * STAGES + 6;
  static constexpr int SMEM_BYTES = 1024 + BAR_OFF + N_BARS * 8 + 64;
};

template <int NKB, int STAGES, int KCAP, int EPW>
__global__ void __launch_bounds__(TcWarps<EPW>::kThreads, 2)
    block_topk_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         int n_queries, int n_blocks, int n_blocks_stride, int k, float* __restrict__ top_scores,
                         int32_t* __restrict__ top_idx) {
  using LY = TcLayout<NKB, STAGES>;
  using W = TcWarps<EPW>;
  constexpr int kEpiWarps = W::kEpiWarps, kProducerWarp = W::kProducerWarp, kMmaWarp = W::kMmaWarp;
  constexpr int kHalfN = W::kPartN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + LY::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* afull = tempty + 2;
  uint64_t* done = afull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_issued = const_cast<int*>(abort_flag + 1);
  int* n_consumed = n_issued + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t s = blockIdx.y;
  const int q0 = blockIdx.x * BM;
  const int n_tiles = (n_blocks + BN - 1) / BN;
  // epilogue warps whose 32 rows hold queries (a stream with fewer than 128
  // queries leaves the upper lane quadrants empty: they take no part)
  const int active_quads = min(4, max(1, (n_queries - q0 + 31) / 32));
  const int active_epi = active_quads * (kEpiWarps / 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], active_epi);
    }
    mbar_init(afull, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 2 * BN);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // query tile (rows of other streams or past the end only feed unused rows)
      mbar_arrive_expect_tx(afull, LY::A_BYTES);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb)
        tma_load_2d(sA + kb * BM * 128, &tmQ, afull, kb * KBOX, (int)(s * n_queries + q0));
      int i = 0;
      for (; i < n_tiles; ++i) {
        const int st = i % STAGES;
        if (!mbar_wait(&empty[st], ((i / STAGES) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(&full[st], LY::B_STAGE_BYTES);
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb)
          tma_load_2d(sB + (st * NKB + kb) * BN * 128, &tmK, &full[st], kb * KBOX,
                      (int)(s * n_blocks_stride + i * BN));
      }
      *n_issued = i;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      int i = 0;
      if (!mbar_wait(afull, 0)) {
        *abort_flag = 1;
      } else {
        for (; i < n_tiles; ++i) {
          const int st = i % STAGES, acc = i & 1;
          if (!mbar_wait(&tempty[acc], ((i >> 1) & 1) ^ 1) || !mbar_wait(&full[st], (i / STAGES) & 1)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
#pragma unroll
          for (int kk = 0; kk < NKB * 4; ++kk) {
            const int kb = kk >> 2, koff = (kk & 3) * 32;
            const uint64_t ad = sw128_desc(smem_u32(sA + kb * BM * 128) + koff);
            const uint64_t bd = sw128_desc(smem_u32(sB + (st * NKB + kb) * BN * 128) + koff);
            umma_bf16(d_tmem, ad, bd, kIdesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty[st]);
          umma_commit(&tfull[acc]);
        }
      }
      *n_consumed = i;
      umma_commit(done);  // arrives once every MMA issued above has completed
    }
  } else {
    // epilogue: warp w reads TMEM lane quadrant w % 4 (row = 32 (w % 4) + lane)
    // and column part w / 4 of every accumulator; with two parts each keeps its
    // own top-k list and the two are merged per row at the end
    const int quad = warp & 3, half = warp >> 2;
    TopK<KCAP> top;
    top.init();
    const int my_tiles = quad < active_quads ? n_tiles : 0;  // empty quadrants skip the tiles
    for (int i = 0; i < my_tiles; ++i) {
      const int acc = i & 1;
      // one lane waits and the warp follows its verdict, so the .sync.aligned
      // TMEM loads below always run with the whole warp
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(&tfull[acc], (i >> 1) & 1) ? 1 : 0;
        if (!ok) *abort_flag = 1;
        if (*abort_flag) ok = 0;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN) + (uint32_t)(half * kHalfN);
      const int b0 = i * BN + half * kHalfN;
      // 32 columns per TMEM load round keep the register footprint small
      // enough for two CTAs per SM; the accumulator is released after the last
#pragma unroll 1
      for (int c0 = 0; c0 < kHalfN; c0 += 32) {
        float v[16], w[16];
        tmem_ld16(taddr + c0, v);
        tmem_ld16(taddr + c0 + 16, w);
        tmem_wait_ld();
        top.offer16(v, b0 + c0, n_blocks);
        top.offer16(w, b0 + c0 + 16, n_blocks);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);  // accumulator free for tile i + 2
    }
    if constexpr (EPW == 4) {
      const int q = q0 + quad * 32 + lane;
      if (q < n_queries)
        top.write(top_scores + ((size_t)s * n_queries + q) * k, top_idx + ((size_t)s * n_queries + q) * k, k);
    } else {
      // merge the two halves of each row through shared memory (the B ring is
      // idle once a warp has consumed every tile; the warps of empty quadrants
      // consumed none and write nothing; after a timeout nothing is merged)
      const int row = quad * 32 + lane;
      const int q = q0 + row;
      float* ms = reinterpret_cast<float*>(sB);                 // [2][BM][KCAP]
      int* mi = reinterpret_cast<int*>(sB + 2 * BM * KCAP * 4);  // [2][BM][KCAP]
      const bool merge = *abort_flag == 0;
      if (merge && quad < active_quads) {
  #pragma unroll
        for (int j = 0; j < KCAP; ++j) {
          ms[(half * BM + row) * KCAP + j] = top.s[j];
          mi[(half * BM + row) * KCAP + j] = top.i[j];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
      if (half == 0 && q < n_queries) {
        float* os = top_scores + ((size_t)s * n_queries + q) * k;
        int32_t* oi = top_idx + ((size_t)s * n_queries + q) * k;
        if (merge) {
          const float* as = ms + row * KCAP;
          const int* ai = mi + row * KCAP;
          const float* bs = ms + (BM + row) * KCAP;
          const int* bi = mi + (BM + row) * KCAP;
          int pa = 0, pb = 0;
          for (int j = 0; j < k; ++j) {
            const float sa = pa < KCAP ? as[pa] : -INFINITY;
            const int ia = pa < KCAP ? ai[pa] : 0x7fffffff;
            const float sb2 = pb < KCAP ? bs[pb] : -INFINITY;
            const int ib = pb < KCAP ? bi[pb] : 0x7fffffff;
            const bool take_a = better(sa, ia, sb2, ib);
            const float sv = take_a ? sa : sb2;
            const int iv = take_a ? ia : ib;
            pa += take_a ? 1 : 0;
            pb += take_a ? 0 : 1;
            const bool filled = iv != 0x7fffffff;
            os[j] = filled ? sv : -INFINITY;
            oi[j] = filled ? iv : -1;
          }
        } else {
          top.write(os, oi, k);
        }
      }
    }
    }
  __syncthreads();
  if (threadIdx.x == 32 * kProducerWarp) {
    // drain copies that were issued but never consumed (only after a timeout)
    for (int i = *n_consumed; i < *n_issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    if (*abort_flag) mbar_wait(afull, 0);
  }
  if (warp == kMmaWarp) {
    if (!mbar_wait(done, 0)) *abort_flag = 1;
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_device_error, (unsigned)GFST_ERR_TIMEOUT);
}

// --- host: tensor maps through the driver entry point ------------------------
template <int NKB, int STAGES, int KCAP, int EPW>
int launch_tc_epw(const CUtensorMap& mq, const CUtensorMap& mk, int64_t S, int Nq, int NB, int NBs, int k,
                  float* ts, int32_t* ti, cudaStream_t stream) {
  using LY = TcLayout<NKB, STAGES>;
  auto kern = block_topk_tc_kernel<NKB, STAGES, KCAP, EPW>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, LY::SMEM_BYTES);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  dim3 grid((unsigned)((Nq + BM - 1) / BM), (unsigned)S);
  kern<<<grid, TcWarps<EPW>::kThreads, LY::SMEM_BYTES, stream>>>(mq, mk, Nq, NB, NBs, k, ts, ti);
  return check_launch("block_topk_tc_kernel");
}

// Long score rows (many summary tiles per query tile) keep the top-k epilogue
// busy: split each row's columns over two warps.  Short rows use one.
template <int NKB, int STAGES, int KCAP>
int launch_tc(const CUtensorMap& mq, const CUtensorMap& mk, int64_t S, int Nq, int NB, int NBs, int k, float* ts,
              int32_t* ti, cudaStream_t stream) {
  if (NB > 16 * BN) return launch_tc_epw<NKB, STAGES, KCAP, 8>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  return launch_tc_epw<NKB, STAGES, KCAP, 4>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
}

template <int NKB, int STAGES>
int dispatch_kcap(const CUtensorMap& mq, const CUtensorMap& mk, int64_t S, int Nq, int NB, int NBs, int k, float* ts,
                  int32_t* ti, cudaStream_t stream) {
  if (k <= 2) return launch_tc<NKB, STAGES, 2>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  if (k <= 4) return launch_tc<NKB, STAGES, 4>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  if (k <= 8) return launch_tc<NKB, STAGES, 8>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  if (k <= 16) return launch_tc<NKB, STAGES, 16>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  return launch_tc<NKB, STAGES, 32>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
}

}  // namespace

int block_topk_tc(const void* Q, const void* Ksum, int64_t S, int Nq, int NB, int NBs, int d, int k, float* ts,
                  int32_t* ti, cudaStream_t stream) {
  GFST_REQUIRE(d % 8 == 0, GFST_ERR_SHAPE, "bf16 retrieval needs d a multiple of 8 (d=%d)", d);
  GFST_REQUIRE(aligned16(Q) && aligned16(Ksum), GFST_ERR_ALIGN, "Q and Ksum must be 16-byte aligned");
  GFST_REQUIRE(S <= 65535, GFST_ERR_SHAPE, "n_streams %lld exceeds 65535", (long long)S);
  GFST_REQUIRE(S * (int64_t)Nq < (1LL << 31) && S * (int64_t)NBs < (1LL << 31), GFST_ERR_SHAPE,
               "row count exceeds the TMA coordinate range");
  CUtensorMap mq, mk;
  int st = make_bf16_map(&mq, Q, (uint64_t)S * Nq, d, BM);
  if (st != GFST_OK) return st;
  st = make_bf16_map(&mk, Ksum, (uint64_t)S * NBs, d, BN);
  if (st != GFST_OK) return st;
  const int nkb = (d + KBOX - 1) / KBOX;
  if (nkb == 1) return dispatch_kcap<1, 4>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  if (nkb == 2) return dispatch_kcap<2, 2>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
  return dispatch_kcap<4, 2>(mq, mk, S, Nq, NB, NBs, k, ts, ti, stream);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int make_bf16_map(CUtensorMap* map, const void* base, uint64_t rows, int d, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  GFST_REQUIRE(enc != nullptr, GFST_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  GFST_REQUIRE(r == CUDA_SUCCESS, GFST_ERR_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GFST_OK;
}

int make_u8_map(CUtensorMap* map, const void* base, uint64_t rows, int row_bytes, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  GFST_REQUIRE(enc != nullptr, GFST_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  GFST_REQUIRE(r == CUDA_SUCCESS, GFST_ERR_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GFST_OK;
}

// One thread waits on an mbarrier that nothing arrives at, for at most
// `budget` clock cycles, and gives up the way the pipelines' waits do: the
// sticky word records GFST_ERR_TIMEOUT and the kernel returns.
__global__ void bounded_wait_probe_kernel(long long budget) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_init_fence();
  if (!mbar_wait_for(&bar, 0, budget)) atomicExch(&g_device_error, (unsigned)GFST_ERR_TIMEOUT);
}

int launch_bounded_wait_probe(long long budget, cudaStream_t stream) {
  bounded_wait_probe_kernel<<<1, 32, 0, stream>>>(budget);
  return check_launch("bounded_wait_probe_kernel");
}


}  // namespace gfst
