// Exact-token readout: inside the k blocks selected for a query, score every
// token key against the query, take the best token in the total order
// (score descending, token index ascending; token index = block * L + position)
// and copy that token's value row out.
//
// Reference (pkhairkh/gfst-hmb-public): ExactRecallReadout._score_block_tokens
// scores each retrieved block's tokens against the query
// (src/gfst_hmb_mpuc/modeling.py:599-657); the collapsed scores are sorted
// descending and the first token is the copy target (modeling.py:1151-1169).
//
// HBM-bound gather.  Where a key row is a power-of-two number of 16-byte
// chunks that divides a warp (d = 64/128/256 bf16, 32/64/128 fp32), one CTA
// serves a chunk of 64 queries of a stream: their (block, query) selections are
// sorted by block, each distinct selected block is streamed from HBM once per
// chunk into a shared-memory ring by 1-D TMA bulk copies, and the consumer
// warps score the block's rows from shared memory (the query's chunk in
// registers, one butterfly per 16 row groups).  Other widths use a lane-per-row
// kernel (one CTA per query).  bf16 products are exact in fp32; sums are fp32.
// NaN scores never win.
#include "gfst_common.cuh"

namespace gfst {

// sticky GFST_ERR_TIMEOUT report of the pipelined readout's bounded waits
__device__ unsigned int g_readout_error = 0;

int read_readout_error(int clear, unsigned int* value) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_readout_error, sizeof(v));
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "reading the readout error word: %s", cudaGetErrorString(e));
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_readout_error, &zero, sizeof(zero));
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "clearing the readout error word: %s", cudaGetErrorString(e));
  }
  *value = v;
  return GFST_OK;
}

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <typename T>
struct Elems16 {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ float dot16(const uint4& v, const float* q, float acc, float) {
  acc = fmaf(__uint_as_float(v.x), q[0], acc);
  acc = fmaf(__uint_as_float(v.y), q[1], acc);
  acc = fmaf(__uint_as_float(v.z), q[2], acc);
  acc = fmaf(__uint_as_float(v.w), q[3], acc);
  return acc;
}
__device__ __forceinline__ float dot16(const uint4& v, const float* q, float acc, __nv_bfloat16) {
  acc = fmaf(bf16_lo(v.x), q[0], acc);
  acc = fmaf(bf16_hi(v.x), q[1], acc);
  acc = fmaf(bf16_lo(v.y), q[2], acc);
  acc = fmaf(bf16_hi(v.y), q[3], acc);
  acc = fmaf(bf16_lo(v.z), q[4], acc);
  acc = fmaf(bf16_hi(v.z), q[5], acc);
  acc = fmaf(bf16_lo(v.w), q[6], acc);
  acc = fmaf(bf16_hi(v.w), q[7], acc);
  return acc;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return bf16_to_f32(v); }

__device__ __forceinline__ void warp_best(float& s, int& i) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float so = __shfl_xor_sync(0xffffffffu, s, o);
    const int io = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(so, io, s, i)) {
      s = so;
      i = io;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) exact_readout_kernel(
    const T* __restrict__ Q, const T* __restrict__ pool_K, const T* __restrict__ pool_V,
    const int32_t* __restrict__ top_idx, int n_queries, int n_slots, int L, int d, int dv, int k,
    int32_t* __restrict__ best_tok, float* __restrict__ best_score, T* __restrict__ out_V) {
  constexpr int N = Elems16<T>::N;
  extern __shared__ __align__(16) float qs[];  // [d] query in fp32
  __shared__ float red_s[kWarps];
  __shared__ int red_i[kWarps];
  const int64_t sq = blockIdx.x;  // stream * n_queries + query
  const int64_t s = sq / n_queries;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int c = tid; c < d; c += kThreads) qs[c] = to_f32(Q[sq * d + c]);
  __syncthreads();

  const int32_t* sel = top_idx + sq * k;
  const int vecs = d / N;
  float bs = __int_as_float(0x7fc00000);  // NaN sentinel ranks last
  int bi = 0x7fffffff;
  for (int j = warp; j < k; j += kWarps) {
    const int b = __ldg(sel + j);
    if (b < 0 || b >= n_slots) continue;
    const uint4* blk = reinterpret_cast<const uint4*>(pool_K + ((size_t)s * n_slots + b) * L * d);
    for (int p = lane; p < L; p += 32) {
      const uint4* row = blk + (size_t)p * vecs;
      float acc = 0.f;
      for (int c = 0; c < vecs; c += 4) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = (c + u < vecs) ? __ldg(row + c + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c + u < vecs) acc = dot16(v[u], qs + (c + u) * N, acc, T());
      }
      const int tok = b * L + p;
      if (better(acc, tok, bs, bi)) {
        bs = acc;
        bi = tok;
      }
    }
  }
  warp_best(bs, bi);
  if (lane == 0) {
    red_s[warp] = bs;
    red_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bs = lane < kWarps ? red_s[lane] : __int_as_float(0x7fc00000);
    bi = lane < kWarps ? red_i[lane] : 0x7fffffff;
    warp_best(bs, bi);
    if (lane == 0) {
      red_s[0] = bs;
      red_i[0] = bi;
    }
  }
  __syncthreads();
  bs = red_s[0];
  bi = red_i[0];
  const bool found = bi != 0x7fffffff;
  if (tid == 0) {
    best_tok[sq] = found ? bi : -1;
    best_score[sq] = found ? bs : -INFINITY;
  }
  if (out_V != nullptr) {
    const int vv = dv / N;
    uint4* dst = reinterpret_cast<uint4*>(out_V + sq * dv);
    if (found) {
      const int b = bi / L, p = bi % L;
      const uint4* src = reinterpret_cast<const uint4*>(pool_V + (((size_t)s * n_slots + b) * L + p) * dv);
      for (int c = tid; c < vv; c += kThreads) dst[c] = __ldg(src + c);
    } else {
      for (int c = tid; c < vv; c += kThreads) dst[c] = make_uint4(0, 0, 0, 0);
    }
  }
}

// 16-byte chunk . query chunk (fp32 accumulate, packed FMAs)
__device__ __forceinline__ float chunk_dot(const uint4& v, const float* q, float) {
  float2 acc = make_float2(0.f, 0.f);
  acc = ffma2(make_float2(__uint_as_float(v.x), __uint_as_float(v.y)), make_float2(q[0], q[1]), acc);
  acc = ffma2(make_float2(__uint_as_float(v.z), __uint_as_float(v.w)), make_float2(q[2], q[3]), acc);
  return acc.x + acc.y;
}
__device__ __forceinline__ float chunk_dot(const uint4& v, const float* q, __nv_bfloat16) {
  float2 acc = make_float2(0.f, 0.f);
  acc = ffma2(make_float2(bf16_lo(v.x), bf16_hi(v.x)), make_float2(q[0], q[1]), acc);
  acc = ffma2(make_float2(bf16_lo(v.y), bf16_hi(v.y)), make_float2(q[2], q[3]), acc);
  acc = ffma2(make_float2(bf16_lo(v.z), bf16_hi(v.z)), make_float2(q[4], q[5]), acc);
  acc = ffma2(make_float2(bf16_lo(v.w), bf16_hi(v.w)), make_float2(q[6], q[7]), acc);
  return acc.x + acc.y;
}

// LPR lanes per key row (16-byte chunks per row), RPL = 32 / LPR rows per warp
// load: consecutive lanes read consecutive 16-byte chunks of whole rows.
// ---------------------------------------------------------------------------
// pipelined readout: one CTA per (stream, chunk of kQC queries).
//  1. the chunk's (block, query) selections are sorted by block (bitonic, smem)
//     and grouped into runs, one run per distinct block;
//  2. a producer thread streams each distinct block, once, into a ring of
//     shared-memory stages with 1-D TMA bulk copies (cp.async.bulk, completion
//     on an mbarrier with the byte count);
//  3. consumer warps take the sorted pairs round robin, wait for their block's
//     stage, score the block's rows against the pair's query from shared
//     memory and fold the best token into the query's 64-bit key with a shared
//     atomicMax (order independent); the last pair of a run frees its stage.
// Each selected block crosses HBM once per query chunk, fully overlapped with
// the scoring.  All waits are bounded; a wait that gives up raises the sticky
// device error word and the CTA drains its copies and returns.
// ---------------------------------------------------------------------------
constexpr int kCWarps = 8;                    // consumer warps
constexpr int kPThreads = (kCWarps + 1) * 32;  // + one producer warp
constexpr int kQC = 64;                        // queries per CTA
constexpr int kMaxPairs = 2048;                // kQC * k, k <= 32
constexpr int kMaxStages = 8;
constexpr long long kWaitCycles = 2000000000LL;

// larger key = better: higher score, then lower token index; NaN never wins
__device__ __forceinline__ unsigned long long pack_best(float s, int tok) {
  uint32_t u = __float_as_uint(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (s != s) u = 0u;
  return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)tok);
}
__device__ __forceinline__ float unpack_score(unsigned long long key) {
  uint32_t u = (uint32_t)(key >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

template <typename T, int LPR>
__global__ void __launch_bounds__(kPThreads) exact_readout_pipelined_kernel(
    const T* __restrict__ Q, const T* __restrict__ pool_K, const T* __restrict__ pool_V,
    const int32_t* __restrict__ top_idx, int n_queries, int n_chunks, int n_slots, int L, int d, int dv, int k,
    int n_stages, int32_t* __restrict__ best_tok, float* __restrict__ best_score, T* __restrict__ out_V) {
  constexpr int N = Elems16<T>::N;
  constexpr int RPL = 32 / LPR;
  constexpr int G = 16;
  extern __shared__ __align__(128) uint8_t dyn[];
  __shared__ uint32_t keys[kMaxPairs];
  __shared__ uint16_t run_of[kMaxPairs];
  __shared__ uint16_t run_start[kMaxPairs + 1];
  __shared__ unsigned long long best[kQC];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ int pending[kMaxStages];
  __shared__ int stage_run[kMaxStages];  // run whose block the stage holds (or is receiving)
  __shared__ int warp_heads[kCWarps];
  __shared__ int n_runs_s, n_valid_s, abort_s, issued_s;
  volatile int* abort_v = &abort_s;
  volatile int* stage_run_v = stage_run;

  const uint32_t block_bytes = (uint32_t)L * d * sizeof(T);
  T* stage = reinterpret_cast<T*>(dyn);                                   // [n_stages][L][d]
  T* qs = reinterpret_cast<T*>(dyn + (size_t)n_stages * block_bytes);     // [kQC][d]
  const int64_t s = blockIdx.x / n_chunks;
  const int q0 = (int)(blockIdx.x % n_chunks) * kQC;
  const int nq = min(kQC, n_queries - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- selections -> sorted (block << 11 | local query) keys ----
  const int n_pairs = nq * k;
  int n_pow2 = 1;
  while (n_pow2 < n_pairs) n_pow2 <<= 1;
  const int32_t* sel = top_idx + ((size_t)s * n_queries + q0) * k;
  for (int e = tid; e < n_pow2; e += kPThreads) {
    uint32_t key = 0xffffffffu;
    if (e < n_pairs) {
      const int b = __ldg(sel + e);
      if (b >= 0 && b < n_slots) key = ((uint32_t)b << 11) | (uint32_t)(e / k);
    }
    keys[e] = key;
  }
  for (int q = tid; q < kQC; q += kPThreads) best[q] = 0ull;
  {
    const uint4* src = reinterpret_cast<const uint4*>(Q + ((size_t)s * n_queries + q0) * d);
    uint4* dst = reinterpret_cast<uint4*>(qs);
    for (int e = tid; e < nq * d / N; e += kPThreads) dst[e] = __ldg(src + e);
  }
  if (tid == 0) {
    for (int i = 0; i < n_stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      stage_run[i] = -1;
    }
    abort_s = 0;
    issued_s = 0;
    n_valid_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int e = tid; e < n_pow2; e += kPThreads) {
        const int partner = e ^ stride;
        if (partner > e) {
          const bool up = (e & size) == 0;
          const uint32_t a = keys[e], b = keys[partner];
          if ((a > b) == up) {
            keys[e] = b;
            keys[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // runs: one per distinct block.  Consumer thread t scans keys [8t, 8t+8):
  // it flags run heads, the heads are prefix-summed over the CTA and each key
  // gets its run index.
  {
    constexpr int PER = kMaxPairs / (kCWarps * 32);
    int cnt = 0, incl = 0;
    uint32_t heads = 0;
    const int e0 = tid * PER;
    if (warp < kCWarps) {
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = e0 + i;
        if (e < n_pairs) {
          const uint32_t key = keys[e];
          if (key != 0xffffffffu) {
            if (e == 0 || (keys[e - 1] >> 11) != (key >> 11)) {
              heads |= 1u << i;
              ++cnt;
            }
            if (e + 1 == n_pairs || keys[e + 1] == 0xffffffffu) n_valid_s = e + 1;
          }
        }
      }
      incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) warp_heads[warp] = incl;
    }
    __syncthreads();
    if (warp < kCWarps) {
      int base = 0;
      for (int w = 0; w < warp; ++w) base += warp_heads[w];
      int r = base + incl - cnt - 1;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = e0 + i;
        if (e < n_pairs && keys[e] != 0xffffffffu) {
          if ((heads >> i) & 1u) {
            ++r;
            run_start[r] = (uint16_t)e;
          }
          run_of[e] = (uint16_t)r;
        }
      }
      if (tid == kCWarps * 32 - 1) n_runs_s = base + incl;
    }
    __syncthreads();
    if (tid == 0) run_start[n_runs_s] = (uint16_t)n_valid_s;
    __syncthreads();
  }
  const int n_runs = n_runs_s;
  const int n_valid = n_valid_s;

  if (warp == kCWarps) {
    // ---- producer: one bulk copy per distinct block ----
    if (lane == 0) {
      int r = 0;
      for (; r < n_runs; ++r) {
        const int st = r % n_stages;
        if (!mbar_wait(&empty[st], ((r / n_stages) & 1) ^ 1)) {
          *abort_v = 1;
          break;
        }
        if (*abort_v) break;
        const int b = (int)(keys[run_start[r]] >> 11);
        pending[st] = run_start[r + 1] - run_start[r];
        stage_run_v[st] = r;
        mbar_arrive_expect_tx(&full[st], block_bytes);
        bulk_load(reinterpret_cast<uint8_t*>(stage) + (size_t)st * block_bytes,
                  pool_K + ((size_t)s * n_slots + b) * L * d, block_bytes, &full[st]);
      }
      issued_s = r;
    }
  } else {
    // ---- consumers ----
    // A pair of run r waits until its stage is tagged with r (the producer
    // tags a stage only after the stage's previous run is fully consumed), then
    // on the stage's full barrier for that phase: a warp that runs ahead of
    // the ring can never mistake an older phase of the same parity for its own.
    const int c = lane % LPR, h = lane / LPR;
    for (int pi = warp; pi < n_valid; pi += kCWarps) {
      const int r = run_of[pi];
      const int st = r % n_stages;
      int ok = 1;
      if (lane == 0) {
        if (stage_run_v[st] != r) {
          const long long t0 = clock64();
          while (stage_run_v[st] != r) {
            if (*abort_v || clock64() - t0 > kWaitCycles) {
              ok = 0;
              break;
            }
          }
        }
        if (ok && !mbar_wait(&full[st], (r / n_stages) & 1)) ok = 0;
        if (!ok) *abort_v = 1;
        if (*abort_v) ok = 0;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const uint32_t key = keys[pi];
      const int b = (int)(key >> 11), ql = (int)(key & 2047u);
      const bool dup = pi > 0 && keys[pi - 1] == key;  // a block listed twice for one query
      if (!dup) {
        float qc[N];
        {
          const uint4 qv = reinterpret_cast<const uint4*>(qs + (size_t)ql * d)[c];
          const T* qe = reinterpret_cast<const T*>(&qv);
#pragma unroll
          for (int i = 0; i < N; ++i) qc[i] = to_f32(qe[i]);
        }
        const uint4* blk = reinterpret_cast<const uint4*>(reinterpret_cast<uint8_t*>(stage) + (size_t)st * block_bytes);
        float bs = __int_as_float(0x7fc00000);
        int bi = 0x7fffffff;
        for (int r0 = 0; r0 < L; r0 += G * RPL) {
          float v[G];
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int p = r0 + g * RPL + h;
            v[g] = p < L ? chunk_dot(blk[(size_t)p * LPR + c], qc, T()) : 0.f;
          }
          subgroup_reduce_scatter<G, LPR>(v, c);
          if constexpr (G >= LPR) {
            constexpr int C = G / LPR;
#pragma unroll
            for (int i = 0; i < C; ++i) {
              const int p = r0 + (c * C + i) * RPL + h;
              if (p < L && better(v[i], b * L + p, bs, bi)) {
                bs = v[i];
                bi = b * L + p;
              }
            }
          } else {
            const int p = r0 + (c / (LPR / G)) * RPL + h;
            if (p < L && better(v[0], b * L + p, bs, bi)) {
              bs = v[0];
              bi = b * L + p;
            }
          }
        }
        warp_best(bs, bi);
        if (lane == 0 && bi != 0x7fffffff) atomicMax(&best[ql], pack_best(bs, bi));
      }
      __syncwarp();
      if (lane == 0 && atomicSub(&pending[st], 1) == 1) mbar_arrive(&empty[st]);
    }
  }
  __syncthreads();
  if (tid == kCWarps * 32) {
    // after a timeout: wait (bounded) for the copies still in flight
    if (*abort_v) {
      const int issued = issued_s;
      for (int r = max(0, issued - n_stages); r < issued; ++r) mbar_wait(&full[r % n_stages], (r / n_stages) & 1);
      atomicExch(&g_readout_error, (unsigned)GFST_ERR_TIMEOUT);
    }
  }

  // ---- outputs: one warp per query ----
  for (int ql = warp; ql < nq; ql += kCWarps + 1) {
    const unsigned long long key = best[ql];
    const bool found = key != 0ull;
    const int tok = found ? (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : -1;
    const int64_t sq = (int64_t)s * n_queries + q0 + ql;
    if (lane == 0) {
      best_tok[sq] = tok;
      best_score[sq] = found ? unpack_score(key) : -INFINITY;
    }
    if (out_V != nullptr) {
      const int vv = dv / N;
      uint4* dst = reinterpret_cast<uint4*>(out_V + sq * dv);
      if (found) {
        const int bb = tok / L, p = tok % L;
        const uint4* src = reinterpret_cast<const uint4*>(pool_V + (((size_t)s * n_slots + bb) * L + p) * dv);
        for (int cc = lane; cc < vv; cc += 32) dst[cc] = __ldg(src + cc);
      } else {
        for (int cc = lane; cc < vv; cc += 32) dst[cc] = make_uint4(0, 0, 0, 0);
      }
    }
  }
}

template <typename T>
int launch(const void* Q, const void* pool_K, const void* pool_V, const int32_t* top_idx, int64_t S, int Nq,
           int NS, int L, int d, int dv, int k, int32_t* best_tok, float* best_score, void* out_V,
           cudaStream_t stream) {
  constexpr int N = Elems16<T>::N;
  GFST_REQUIRE(d % N == 0, GFST_ERR_ALIGN, "d=%d must be a multiple of %d", d, N);
  GFST_REQUIRE(out_V == nullptr || dv % N == 0, GFST_ERR_ALIGN, "dv=%d must be a multiple of %d", dv, N);
  const int64_t grid = S * (int64_t)Nq;
  GFST_REQUIRE(grid <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many queries");
  const T* q = static_cast<const T*>(Q);
  const T* pk = static_cast<const T*>(pool_K);
  const T* pv = static_cast<const T*>(pool_V);
  T* ov = static_cast<T*>(out_V);
  const int64_t n_chunks = (Nq + kQC - 1) / kQC;
  const size_t block_bytes = (size_t)L * d * sizeof(T);
  // stages: about 80 KB of ring per CTA (two CTAs per SM), 2 to 8 blocks
  int n_stages = (int)((80u * 1024u) / block_bytes);
  n_stages = n_stages < 2 ? 2 : (n_stages > kMaxStages ? kMaxStages : n_stages);
  const size_t dyn = (size_t)n_stages * block_bytes + (size_t)kQC * d * sizeof(T);
  const bool pipelined_ok = (int64_t)NS < (1LL << 21) && S * n_chunks <= 0x7fffffffLL && dyn <= 200u * 1024u &&
                            (L * (int64_t)d * (int64_t)sizeof(T)) % 16 == 0 && aligned16(Q) && k <= 32;
  if (pipelined_ok) {
    const unsigned pgrid = (unsigned)(S * n_chunks);
    cudaError_t e = cudaSuccess;
    switch (d / N) {
#define GFST_READOUT_CASE(LPRV)                                                                                   \
  case LPRV: {                                                                                                    \
    auto kern = exact_readout_pipelined_kernel<T, LPRV>;                                                           \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);                         \
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));           \
    kern<<<pgrid, kPThreads, dyn, stream>>>(q, pk, pv, top_idx, Nq, (int)n_chunks, NS, L, d, dv, k, n_stages,       \
                                            best_tok, best_score, ov);                                             \
    return check_launch("exact_readout_pipelined_kernel");                                                         \
  }
      GFST_READOUT_CASE(8)
      GFST_READOUT_CASE(16)
      GFST_READOUT_CASE(32)
#undef GFST_READOUT_CASE
      default:
        break;
    }
  }
  exact_readout_kernel<T><<<(unsigned)grid, kThreads, (size_t)d * sizeof(float), stream>>>(
      q, pk, pv, top_idx, Nq, NS, L, d, dv, k, best_tok, best_score, ov);
  return check_launch("exact_readout_kernel");
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_exact_readout(const void* Q, const void* pool_K, const void* pool_V, const int32_t* top_idx,
                                  int64_t n_streams, int n_queries, int n_slots, int L, int d, int dv, int k,
                                  int dtype, int32_t* best_tok, float* best_score, void* out_V,
                                  cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_slots >= 1 && L >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(k >= 1 && k <= 32, GFST_ERR_SHAPE, "k=%d outside [1, 32]", k);
  GFST_REQUIRE(d >= 1 && d <= 256, GFST_ERR_SHAPE, "d=%d outside [1, 256]", d);
  GFST_REQUIRE((pool_V == nullptr) == (out_V == nullptr), GFST_ERR_ARG, "pool_V and out_V go together");
  GFST_REQUIRE((int64_t)n_slots * L <= 0x7fffffffLL, GFST_ERR_SHAPE, "token index overflows int32");
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(Q && pool_K && top_idx && best_tok && best_score, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(aligned16(pool_K) && aligned16(pool_V) && aligned16(out_V), GFST_ERR_ALIGN,
               "pool and output buffers must be 16-byte aligned");
  if (dtype == GFST_F32)
    return launch<float>(Q, pool_K, pool_V, top_idx, n_streams, n_queries, n_slots, L, d, dv, k, best_tok,
                         best_score, out_V, stream);
  if (dtype == GFST_BF16)
    return launch<__nv_bfloat16>(Q, pool_K, pool_V, top_idx, n_streams, n_queries, n_slots, L, d, dv, k, best_tok,
                                 best_score, out_V, stream);
  set_last_error("unsupported dtype %d", dtype);
  return GFST_ERR_DTYPE;
}
