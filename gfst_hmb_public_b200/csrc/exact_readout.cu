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
#include <type_traits>

#include "async_copy.cuh"

namespace gfst {

// sticky GFST_ERR_TIMEOUT report of the pipelined readout's bounded waits
GFST_DEFINE_ERROR_WORD(g_readout_error, read_readout_error, "readout")

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
  const bool found = bi != 0x7fffffff && bs == bs;  // NaN scores never win
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

// ---------------------------------------------------------------------------
// pipelined readout: one CTA per (stream, chunk of kQC queries).
//  1. the chunk's (block, query) selections are sorted by block (bitonic, smem)
//     and grouped into runs, one run per distinct block;
//  2. a producer thread streams each distinct block, once, into a ring of
//     shared-memory stages (TMA, completion on an mbarrier with the byte count);
//  3. consumer warps wait for their block's stage, score its token rows against
//     the queries that selected it, fold each query's best token into a 64-bit
//     key with a shared atomicMax (order independent) and free the stage.
// Each selected block crosses HBM once per query chunk, overlapped with the
// scoring.  All waits are bounded; a wait that gives up raises the sticky
// readout error word and the CTA drains its copies and returns.
//
// Ring protocol: the producer tags a stage with the run it is loading only
// after the stage's previous run is fully consumed; a consumer of run r waits
// for the tag r, then for the stage's full barrier in r's phase.  A consumer
// that runs ahead of the ring therefore never takes an older phase of the same
// parity for its own.
// ---------------------------------------------------------------------------
constexpr int kQC = 64;          // queries per CTA
constexpr int kMaxPairs = 2048;  // kQC * k, k <= 32
constexpr int kMaxStages = 8;
constexpr uint32_t kNoKey = 0xffffffffu;

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

struct RunTable {
  uint32_t keys[kMaxPairs];           // sorted (block << 11 | local query); kNoKey = no entry
  uint16_t run_start[kMaxPairs + 1];  // first key of each run; run_start[n_runs] = n_valid
  int warp_heads[32];
  int n_runs, n_valid;
};

// Fill, sort and split the chunk's selections into runs.  Every thread of the
// CTA (NT) calls; the first NSCAN threads scan kMaxPairs / NSCAN keys each.
// run_of (optional) receives each key's run index.
template <int NT, int NSCAN>
__device__ __forceinline__ void build_runs(RunTable& rt, uint16_t* run_of, const int32_t* __restrict__ sel,
                                           int n_pairs, int k, int n_slots) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int n_pow2 = 1;
  while (n_pow2 < n_pairs) n_pow2 <<= 1;
  for (int e = tid; e < n_pow2; e += NT) {
    uint32_t key = kNoKey;
    if (e < n_pairs) {
      const int b = __ldg(sel + e);
      if (b >= 0 && b < n_slots) key = ((uint32_t)b << 11) | (uint32_t)(e / k);
    }
    rt.keys[e] = key;
  }
  if (tid == 0) rt.n_valid = 0;
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int e = tid; e < n_pow2; e += NT) {
        const int partner = e ^ stride;
        if (partner > e) {
          const bool up = (e & size) == 0;
          const uint32_t a = rt.keys[e], b = rt.keys[partner];
          if ((a > b) == up) {
            rt.keys[e] = b;
            rt.keys[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  // run heads, prefix-summed over the scanning threads
  constexpr int PER = kMaxPairs / NSCAN;
  static_assert(NSCAN % 32 == 0 && NSCAN <= NT && kMaxPairs % NSCAN == 0 && PER <= 32, "scan split");
  int cnt = 0, incl = 0;
  uint32_t heads = 0;
  const int e0 = tid * PER;
  if (tid < NSCAN) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = e0 + i;
      if (e < n_pairs) {
        const uint32_t key = rt.keys[e];
        if (key != kNoKey) {
          if (e == 0 || (rt.keys[e - 1] >> 11) != (key >> 11)) {
            heads |= 1u << i;
            ++cnt;
          }
          if (e + 1 == n_pairs || rt.keys[e + 1] == kNoKey) rt.n_valid = e + 1;
        }
      }
    }
    incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) rt.warp_heads[warp] = incl;
  }
  __syncthreads();
  if (tid < NSCAN) {
    int base = 0;
    for (int w = 0; w < warp; ++w) base += rt.warp_heads[w];
    int r = base + incl - cnt - 1;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = e0 + i;
      if (e < n_pairs && rt.keys[e] != kNoKey) {
        if ((heads >> i) & 1u) {
          ++r;
          rt.run_start[r] = (uint16_t)e;
        }
        if (run_of != nullptr) run_of[e] = (uint16_t)r;
      }
    }
    if (tid == NSCAN - 1) rt.n_runs = base + incl;
  }
  __syncthreads();
  if (tid == 0) rt.run_start[rt.n_runs] = (uint16_t)rt.n_valid;
  __syncthreads();
}

// build_runs by a counting sort over the block indices (n_slots <= the
// histogram's size, hist: n_slots ints of scratch shared memory): the keys
// come out grouped by block in ascending block order; inside a block their
// order is the order the scatter's atomics happen to take, which nothing
// downstream depends on (every query's result is order-free).  Three CTA
// barriers instead of the bitonic sort's log^2.
template <int NT>
__device__ __forceinline__ void build_runs_counting(RunTable& rt, int* hist, const int32_t* __restrict__ sel,
                                                    int n_pairs, int k, int n_slots) {
  const int tid = threadIdx.x;
  for (int i = tid; i < n_slots; i += NT) hist[i] = 0;
  __syncthreads();
  for (int e = tid; e < n_pairs; e += NT) {
    const int b = __ldg(sel + e);
    if (b >= 0 && b < n_slots) atomicAdd(&hist[b], 1);
  }
  __syncthreads();
  if (tid < 32) {
    // exclusive scans of the counts (key offsets) and of the non-empty bins (run indices)
    int base_e = 0, base_r = 0;
    for (int c0 = 0; c0 < n_slots; c0 += 32) {
      const int i = c0 + tid;
      const int cnt = i < n_slots ? hist[i] : 0;
      int ie = cnt, ir = cnt > 0 ? 1 : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ye = __shfl_up_sync(0xffffffffu, ie, o), yr = __shfl_up_sync(0xffffffffu, ir, o);
        if (tid >= o) {
          ie += ye;
          ir += yr;
        }
      }
      const int ex = base_e + ie - cnt, rx = base_r + ir - (cnt > 0 ? 1 : 0);
      if (i < n_slots) {
        hist[i] = ex;
        if (cnt > 0) rt.run_start[rx] = (uint16_t)ex;
      }
      base_e += __shfl_sync(0xffffffffu, ie, 31);
      base_r += __shfl_sync(0xffffffffu, ir, 31);
    }
    if (tid == 0) {
      rt.n_runs = base_r;
      rt.n_valid = base_e;
      rt.run_start[base_r] = (uint16_t)base_e;
    }
  }
  __syncthreads();
  for (int e = tid; e < n_pairs; e += NT) {
    const int b = __ldg(sel + e);
    if (b >= 0 && b < n_slots) rt.keys[atomicAdd(&hist[b], 1)] = ((uint32_t)b << 11) | (uint32_t)(e / k);
  }
  __syncthreads();
}

// Consumer side of the ring: wait until stage st holds run r.  Lane 0 waits;
// the verdict is broadcast.  false: give up (timeout or another warp aborted).
__device__ __forceinline__ bool wait_stage(volatile int* stage_run, uint64_t* full, volatile int* abort_flag,
                                           int st, int r, int n_stages) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (stage_run[st] != r) {
      const long long t0 = clock64();
      while (stage_run[st] != r) {
        if (*abort_flag || clock64() - t0 > kMbarWaitCycles) {
          ok = 0;
          break;
        }
        __nanosleep(64);  // leave the issue slots to warps with work
      }
    }
    if (ok && !mbar_wait(&full[st], (r / n_stages) & 1)) ok = 0;
    if (!ok) *abort_flag = 1;
    if (*abort_flag) ok = 0;
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// After a give-up: wait (bounded) for the copies still in flight, then report.
__device__ __forceinline__ void drain_after_abort(uint64_t* full, int issued, int n_stages) {
  for (int r = max(0, issued - n_stages); r < issued; ++r) mbar_wait(&full[r % n_stages], (r / n_stages) & 1);
  atomicExch(&g_readout_error, (unsigned)GFST_ERR_TIMEOUT);
}

// Outputs of the chunk: one warp per query.
template <typename T>
__device__ __forceinline__ void write_outputs(const unsigned long long* best, int nq, int nwarps, int64_t sq0, int L,
                                              int n_slots, int dv, int64_t s, const T* __restrict__ pool_V,
                                              int32_t* __restrict__ best_tok, float* __restrict__ best_score,
                                              T* __restrict__ out_V) {
  constexpr int N = Elems16<T>::N;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int ql = warp; ql < nq; ql += nwarps) {
    const unsigned long long key = best[ql];
    const bool found = key != 0ull;
    const int tok = found ? (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : -1;
    const int64_t sq = sq0 + ql;
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

// ---- SIMT consumers (fp32 pools, and bf16 shapes the tensor-core kernel does
// not take).  1-D bulk copies of whole blocks; consumer warps take the sorted
// pairs round robin (LPR lanes per key row, RPL = 32 / LPR rows per warp load)
// and the last pair of a run frees its stage.
constexpr int kCWarps = 8;
constexpr int kPThreads = (kCWarps + 1) * 32;

template <typename T, int LPR>
__global__ void __launch_bounds__(kPThreads) exact_readout_pipelined_kernel(
    const T* __restrict__ Q, const T* __restrict__ pool_K, const T* __restrict__ pool_V,
    const int32_t* __restrict__ top_idx, int n_queries, int n_chunks, int n_slots, int L, int d, int dv, int k,
    int n_stages, int32_t* __restrict__ best_tok, float* __restrict__ best_score, T* __restrict__ out_V) {
  constexpr int N = Elems16<T>::N;
  constexpr int RPL = 32 / LPR;
  constexpr int G = 16;
  extern __shared__ __align__(128) uint8_t dyn[];
  __shared__ RunTable rt;
  __shared__ uint16_t run_of[kMaxPairs];
  __shared__ unsigned long long best[kQC];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ int pending[kMaxStages];
  __shared__ int stage_run[kMaxStages];
  __shared__ int abort_s, issued_s;
  volatile int* abort_v = &abort_s;
  volatile int* stage_run_v = stage_run;

  const uint32_t block_bytes = (uint32_t)L * d * sizeof(T);
  T* stage = reinterpret_cast<T*>(dyn);                                // [n_stages][L][d]
  T* qs = reinterpret_cast<T*>(dyn + (size_t)n_stages * block_bytes);  // [kQC][d]
  const int64_t s = blockIdx.x / n_chunks;
  const int q0 = (int)(blockIdx.x % n_chunks) * kQC;
  const int nq = min(kQC, n_queries - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

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
    mbar_init_fence();
  }
  build_runs<kPThreads, kCWarps * 32>(rt, run_of, top_idx + ((size_t)s * n_queries + q0) * k, nq * k, k, n_slots);
  const int n_runs = rt.n_runs;
  const int n_valid = rt.n_valid;

  if (warp == kCWarps) {
    if (lane == 0) {
      int r = 0;
      for (; r < n_runs; ++r) {
        const int st = r % n_stages;
        if (!mbar_wait(&empty[st], ((r / n_stages) & 1) ^ 1)) {
          *abort_v = 1;
          break;
        }
        if (*abort_v) break;
        const int b = (int)(rt.keys[rt.run_start[r]] >> 11);
        pending[st] = rt.run_start[r + 1] - rt.run_start[r];
        stage_run_v[st] = r;
        mbar_arrive_expect_tx(&full[st], block_bytes);
        bulk_load(reinterpret_cast<uint8_t*>(stage) + (size_t)st * block_bytes,
                  pool_K + ((size_t)s * n_slots + b) * L * d, block_bytes, &full[st]);
      }
      issued_s = r;
    }
  } else {
    const int c = lane % LPR, h = lane / LPR;
    for (int pi = warp; pi < n_valid; pi += kCWarps) {
      const int r = run_of[pi];
      const int st = r % n_stages;
      if (!wait_stage(stage_run_v, full, abort_v, st, r, n_stages)) break;
      const uint32_t key = rt.keys[pi];
      const int b = (int)(key >> 11), ql = (int)(key & 2047u);
      const bool dup = pi > 0 && rt.keys[pi - 1] == key;  // a block listed twice for one query
      if (!dup) {
        float qc[N];
        {
          const uint4 qv = reinterpret_cast<const uint4*>(qs + (size_t)ql * d)[c];
          const T* qe = reinterpret_cast<const T*>(&qv);
#pragma unroll
          for (int i = 0; i < N; ++i) qc[i] = to_f32(qe[i]);
        }
        const uint4* blk =
            reinterpret_cast<const uint4*>(reinterpret_cast<uint8_t*>(stage) + (size_t)st * block_bytes);
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
        if (lane == 0 && bi != 0x7fffffff && bs == bs) atomicMax(&best[ql], pack_best(bs, bi));
      }
      __syncwarp();
      if (lane == 0 && atomicSub(&pending[st], 1) == 1) mbar_arrive(&empty[st]);
    }
  }
  __syncthreads();
  if (tid == kCWarps * 32 && *abort_v) drain_after_abort(full, issued_s, n_stages);
  write_outputs<T>(best, nq, kCWarps + 1, (int64_t)s * n_queries + q0, L, n_slots, dv, s, pool_V, best_tok,
                   best_score, out_V);
}

// ---- tensor-core consumers (bf16 pools, d = 64 * NKB, L % 16 == 0) ----
// The producer loads a block as NKB TMA boxes of [L rows x 64 columns] with the
// 128-byte swizzle, so a warp's ldmatrix of 8 rows x 16 bytes hits 8 distinct
// bank groups.  A consumer warp takes whole runs (warp w: runs w, w + 4, ...)
// and, for each group of up to 8 queries that selected the block, computes the
// [L x 8] score tile with mma.sync m16n8k16 (bf16 products are exact in fp32;
// fp32 accumulation), keeping per lane the best token of its two query columns.
// Queries sit in shared memory with their 16-byte chunks XOR-swizzled by row
// (chunk c of query q at (c & ~7) | ((c ^ q) & 7)); unused query columns read a
// zero row and are ignored.  The scores are N <= 8 columns wide per block: the
// warp-level MMA keeps them in registers with no accumulator round trip, and the
// kernel stays bound by HBM, not by the tensor pipe.
#ifndef GFST_READOUT_RING_KB
#define GFST_READOUT_RING_KB 80u
#endif
constexpr int kMWarps = 4;
constexpr int kMThreads = (kMWarps + 1) * 32;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Best (score, token) of one query column as seen by one lane.  Tokens are
// offered in increasing order, so an equal score never replaces the held one;
// NaN never replaces a number, and a lane that saw only NaN holds nothing.
struct TokenBest {
  float s = -INFINITY;
  int i = 0x7fffffff;
  __device__ __forceinline__ void offer(float v, int tok) {
    const bool take = v > s || (i == 0x7fffffff && v == v);
    s = take ? v : s;
    i = take ? tok : i;
  }
  // combine the 8 lanes that hold the same query columns (lane % 4 equal)
  __device__ __forceinline__ void reduce_rows() {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
      if (i2 != 0x7fffffff && (i == 0x7fffffff || better(s2, i2, s, i))) {
        s = s2;
        i = i2;
      }
    }
  }
  __device__ __forceinline__ bool found() const { return i != 0x7fffffff; }
};

template <int NKB>
__global__ void __launch_bounds__(kMThreads) exact_readout_mma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __nv_bfloat16* __restrict__ Q,
    const __nv_bfloat16* __restrict__ pool_V, const int32_t* __restrict__ top_idx, int n_queries, int n_chunks,
    int n_slots, int L, int dv, int k, int n_stages, int32_t* __restrict__ best_tok, float* __restrict__ best_score,
    __nv_bfloat16* __restrict__ out_V) {
  constexpr int D = NKB * 64;
  constexpr int QROW = D * 2;   // bytes per key / query row
  constexpr int KSTEPS = D / 16;
  extern __shared__ uint8_t dyn_raw[];
  __shared__ RunTable rt;
  __shared__ unsigned long long best[kQC];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ int stage_run[kMaxStages];
  __shared__ int abort_s, issued_s;
  volatile int* abort_v = &abort_s;
  volatile int* stage_run_v = stage_run;

  const uint32_t stage_bytes = (uint32_t)L * QROW;  // NKB boxes of L x 128 bytes
  const uint32_t raw = smem_u32(dyn_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;     // the 128-byte swizzle repeats every 1024 bytes
  uint8_t* dyn = dyn_raw + (base - raw);
  uint8_t* qs = dyn + (size_t)n_stages * stage_bytes;  // [kQC][D], chunk-swizzled
  uint8_t* zrow = qs + kQC * QROW;                     // one zero row
  const uint32_t qs_u = base + n_stages * stage_bytes;
  const uint32_t zrow_u = qs_u + kQC * QROW;
  const int64_t s = blockIdx.x / n_chunks;
  const int q0 = (int)(blockIdx.x % n_chunks) * kQC;
  const int nq = min(kQC, n_queries - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int q = tid; q < kQC; q += kMThreads) best[q] = 0ull;
  {
    constexpr int CPR = QROW / 16;  // 16-byte chunks per row
    const uint4* src = reinterpret_cast<const uint4*>(Q + ((size_t)s * n_queries + q0) * D);
    for (int e = tid; e < nq * CPR; e += kMThreads) {
      const int q = e / CPR, c = e % CPR;
      const int pos = (c & ~7) | ((c ^ q) & 7);
      *reinterpret_cast<uint4*>(qs + q * QROW + pos * 16) = __ldg(src + e);
    }
    for (int e = tid; e < CPR; e += kMThreads) reinterpret_cast<uint4*>(zrow)[e] = make_uint4(0, 0, 0, 0);
  }
  if (tid == 0) {
    for (int i = 0; i < n_stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      stage_run[i] = -1;
    }
    abort_s = 0;
    issued_s = 0;
    mbar_init_fence();
  }
  // the ring is idle until the pipeline starts: it holds the counting sort's
  // histogram when the ring has room for one count per slot (three CTA
  // barriers; the bitonic sort takes log^2 of the pair capacity)
  const bool counting = (int64_t)n_slots * 4 <= (int64_t)n_stages * stage_bytes;
  if (counting)
    build_runs_counting<kMThreads>(rt, reinterpret_cast<int*>(dyn), top_idx + ((size_t)s * n_queries + q0) * k,
                                   nq * k, k, n_slots);
  else
    build_runs<kMThreads, kMWarps * 32>(rt, nullptr, top_idx + ((size_t)s * n_queries + q0) * k, nq * k, k,
                                        n_slots);
  const int n_runs = rt.n_runs;

  if (warp == kMWarps) {
    if (lane == 0) {
      // generic-proxy writes to the ring (the histogram) precede its copies
      if (counting) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      int r = 0;
      for (; r < n_runs; ++r) {
        const int st = r % n_stages;
        if (!mbar_wait(&empty[st], ((r / n_stages) & 1) ^ 1)) {
          *abort_v = 1;
          break;
        }
        if (*abort_v) break;
        const int b = (int)(rt.keys[rt.run_start[r]] >> 11);
        const int row0 = (int)(((int64_t)s * n_slots + b) * L);
        stage_run_v[st] = r;
        mbar_arrive_expect_tx(&full[st], stage_bytes);
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb)
          tma_load_2d(dyn + (size_t)st * stage_bytes + (size_t)kb * L * 128, &tmK, &full[st], kb * 64, row0);
      }
      issued_s = r;
    }
  } else {
    // ldmatrix address roles: A (token rows) lane -> row (lane & 7) + 8 * ((lane >> 3) & 1),
    // 16-byte chunk 2 kk + (lane >> 4); B (queries) lane -> query column lane & 7,
    // chunk 2 kk + (lane >> 3) (two k-steps per x4 load)
    const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int a_hi = lane >> 4;
    const int bcol = lane & 7;
    const int nt = L / 16;
    // per k-step offset of this lane's A chunk inside a 16-row tile: box (kk / 4),
    // 16-byte chunk (2 kk + a_hi) % 8 XOR (row % 8), row % 8 == lane % 8
    uint32_t aoff[KSTEPS];
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      aoff[kk] = (uint32_t)((kk >> 2) * L * 128) + (uint32_t)((((2 * kk + a_hi) & 7) ^ (lane & 7)) << 4);
    for (int r = warp; r < n_runs; r += kMWarps) {
      const int st = r % n_stages;
      if (!wait_stage(stage_run_v, full, abort_v, st, r, n_stages)) break;
      const int p0 = rt.run_start[r], p1 = rt.run_start[r + 1];
      const int b = (int)(rt.keys[p0] >> 11);
      const uint32_t abase = base + st * stage_bytes + a_row * 128;
      for (int g0 = p0; g0 < p1; g0 += 8) {
        const int pn = g0 + bcol;
        const int qn = pn < p1 ? (int)(rt.keys[pn] & 2047u) : -1;
        uint32_t bq[KSTEPS][2];
#pragma unroll
        for (int kk = 0; kk < KSTEPS; kk += 2) {
          const int c = 2 * kk + (lane >> 3);
          const uint32_t addr =
              qn >= 0 ? qs_u + qn * QROW + (uint32_t)(((c & ~7) | ((c ^ qn) & 7)) << 4) : zrow_u + (uint32_t)(c << 4);
          ldsm_x4(addr, bq[kk][0], bq[kk][1], bq[kk + 1][0], bq[kk + 1][1]);
        }
        TokenBest best0, best1;
        int t = 0;
        // four 16-row tiles at a time: independent accumulators hide the MMA latency
        for (; t + 4 <= nt; t += 4) {
          float acc[4][4] = {};
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint32_t a0, a1, a2, a3;
              ldsm_x4(abase + (uint32_t)((t + u) * 16 * 128) + aoff[kk], a0, a1, a2, a3);
              mma_16816(acc[u], a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            // acc[u][0], [1]: token row 16 (t + u) + lane / 4, query columns 2 (lane % 4), +1;
            // acc[u][2], [3]: the same columns, token row + 8
            const int tok = b * L + (t + u) * 16 + (lane >> 2);
            best0.offer(acc[u][0], tok);
            best1.offer(acc[u][1], tok);
            best0.offer(acc[u][2], tok + 8);
            best1.offer(acc[u][3], tok + 8);
          }
        }
        for (; t < nt; ++t) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(abase + (uint32_t)(t * 16 * 128) + aoff[kk], a0, a1, a2, a3);
            mma_16816(acc, a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
          }
          const int tok = b * L + t * 16 + (lane >> 2);
          best0.offer(acc[0], tok);
          best1.offer(acc[1], tok);
          best0.offer(acc[2], tok + 8);
          best1.offer(acc[3], tok + 8);
        }
        best0.reduce_rows();
        best1.reduce_rows();
        if (lane < 4) {
          const int n0 = g0 + 2 * lane, n1 = n0 + 1;
          if (n0 < p1 && best0.found()) atomicMax(&best[rt.keys[n0] & 2047u], pack_best(best0.s, best0.i));
          if (n1 < p1 && best1.found()) atomicMax(&best[rt.keys[n1] & 2047u], pack_best(best1.s, best1.i));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  __syncthreads();
  if (tid == kMWarps * 32 && *abort_v) drain_after_abort(full, issued_s, n_stages);
  write_outputs<__nv_bfloat16>(best, nq, kMWarps + 1, (int64_t)s * n_queries + q0, L, n_slots, dv, s, pool_V,
                               best_tok, best_score, out_V);
}

// ---- exact readout with an int8 first look (bf16 pools, d = 128 * NB8) ----
// The committed keys also exist as int8 copies k8 = round(k / s_k) with a
// per-token scale s_k = max|k| / 127 (gfst_block_commit_i8), and per block
// E >= max |k - s_k k8|_2 and N >= max |k|_2 over its tokens.  The kernel
// streams those copies (L d + 4 L + 16 bytes per block instead of 2 L d),
// quantises each query the same way (s_q, q8, e_q >= |q - s_q q8|_2,
// n_q >= |q|_2) and takes the integer products q8 . k8 on the tensor cores
// (mma.sync m16n8k32, exact int32 sums).  For every (query, token) pair of a
// block the fp32 score S of the exact readout then lies within A +- b with
//     A = s_q s_k (q8 . k8),
//     b = n_q E + e_q (N + E) + slack n_q N  (+ 2^-20 of the largest |A| + b)
// (q.k - q^.k^ = q.(k - k^) + (q - q^).k^ and Cauchy-Schwarz; slack covers the
// fp32 rounding of A and of any fp32 evaluation of S).  Each query keeps
// LB = max(A - b) over its tokens and a list of the tokens whose A + b reached
// the LB current when they were scored; the argmax of S (and every token tied
// with it) has A + b >= S_max >= LB, so it is on the list.  The listed tokens
// with A + b >= the final LB are re-scored exactly from the bf16 keys, and the
// best in the total order (score descending, token ascending; NaN never wins)
// is the result: the same token the exact readout picks.  A query whose list
// overflows, or whose own values are not finite or all zero, and any block
// holding a key with a non-finite value (E = inf), is scored in full from the
// bf16 keys instead.
constexpr int kCandCap = 32;
constexpr int kMaxStagesI8 = 16;  // ring stages of the int8 readout
constexpr int kI8Warps = 8;       // its consumer warps (plus one TMA warp)

__device__ __forceinline__ void mma_i8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// order-preserving float -> uint (NaN -> 0, the smallest)
__device__ __forceinline__ uint32_t ord_u32(float x) {
  uint32_t u = __float_as_uint(x);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return x != x ? 0u : u;
}
__device__ __forceinline__ float ord_f32(uint32_t u) {
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}

// fp32 dot of one bf16 key row and one bf16 query row (d / 8 16-byte chunks)
__device__ __forceinline__ float bf16_row_dot(const __nv_bfloat16* __restrict__ kr, const __nv_bfloat16* __restrict__ qr,
                                              int d) {
  const uint4* k4 = reinterpret_cast<const uint4*>(kr);
  const uint4* q4 = reinterpret_cast<const uint4*>(qr);
  float acc = 0.f;
  for (int c = 0; c < d / 8; ++c) {
    const uint4 kv = __ldg(k4 + c), qv = __ldg(q4 + c);
    acc = fmaf(bf16_lo(kv.x), bf16_lo(qv.x), acc);
    acc = fmaf(bf16_hi(kv.x), bf16_hi(qv.x), acc);
    acc = fmaf(bf16_lo(kv.y), bf16_lo(qv.y), acc);
    acc = fmaf(bf16_hi(kv.y), bf16_hi(qv.y), acc);
    acc = fmaf(bf16_lo(kv.z), bf16_lo(qv.z), acc);
    acc = fmaf(bf16_hi(kv.z), bf16_hi(qv.z), acc);
    acc = fmaf(bf16_lo(kv.w), bf16_lo(qv.w), acc);
    acc = fmaf(bf16_hi(kv.w), bf16_hi(qv.w), acc);
  }
  return acc;
}

template <int NB8, int CW>
__global__ void __launch_bounds__((CW + 1) * 32) exact_readout_i8_kernel(
    const __grid_constant__ CUtensorMap tmK8, const __nv_bfloat16* __restrict__ Q,
    const __nv_bfloat16* __restrict__ pool_K, const float* __restrict__ k8_scale,
    const __nv_bfloat16* __restrict__ pool_V, const int32_t* __restrict__ top_idx, int n_queries, int n_chunks,
    int n_slots, int L, int dv, int k, int n_stages, float slack, int32_t* __restrict__ best_tok,
    float* __restrict__ best_score, __nv_bfloat16* __restrict__ out_V) {
  constexpr int D = NB8 * 128;  // key width = int8 bytes per key row
  constexpr int NT = (CW + 1) * 32;  // CW consumer warps + the TMA warp
  constexpr int KSTEPS = D / 32;
  extern __shared__ uint8_t dyn_raw[];
  __shared__ RunTable rt;
  __shared__ unsigned long long best[kQC];
  __shared__ uint32_t lbk[kQC];
  __shared__ int ccount[kQC];
  __shared__ uint2 cand[kQC][kCandCap];
  __shared__ float4 qstat[kQC];  // s_q, e_q, n_q, 1 = score in full
  __shared__ uint64_t full[kMaxStagesI8], empty[kMaxStagesI8];
  __shared__ int stage_run[kMaxStagesI8];
  __shared__ int abort_s, issued_p[4];
  volatile int* abort_v = &abort_s;
  volatile int* stage_run_v = stage_run;

  const uint32_t key_bytes = (uint32_t)L * D;
  const uint32_t side_bytes = (uint32_t)(L + 4) * 4u;  // scales, then E, N, 0, 0 (a multiple of 16)
  // key stages 1024-byte aligned (the swizzle atom); the side data in a ring
  // of its own after them, so that no stage carries alignment padding
  const uint32_t stage_bytes = (key_bytes + 1023u) & ~1023u;
  const uint32_t raw = smem_u32(dyn_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* dyn = dyn_raw + (base - raw);
  uint8_t* side = dyn + (size_t)n_stages * stage_bytes;        // [n_stages][L + 4] fp32
  uint8_t* qs = side + (size_t)n_stages * side_bytes;           // [kQC][D] int8, chunk-swizzled
  uint8_t* zrow = qs + kQC * D;
  const uint32_t qs_u = base + n_stages * (stage_bytes + side_bytes);
  const uint32_t zrow_u = qs_u + kQC * D;
  const int64_t s = blockIdx.x / n_chunks;
  const int q0 = (int)(blockIdx.x % n_chunks) * kQC;
  const int nq = min(kQC, n_queries - q0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const __nv_bfloat16* Qc = Q + ((size_t)s * n_queries + q0) * D;

  for (int q = tid; q < kQC; q += NT) {
    best[q] = 0ull;
    lbk[q] = ord_u32(-INFINITY);
    ccount[q] = 0;
  }
  for (int e = tid; e < D / 16; e += NT) reinterpret_cast<uint4*>(zrow)[e] = make_uint4(0, 0, 0, 0);
  // the chunk's bf16 queries into the (still idle) ring, one coalesced copy
  __nv_bfloat16* qbf = reinterpret_cast<__nv_bfloat16*>(dyn);
  for (int e = tid; e < nq * D / 8; e += NT)
    reinterpret_cast<uint4*>(qbf)[e] = __ldg(reinterpret_cast<const uint4*>(Qc) + e);
  __syncthreads();
  // quantise them: one warp per query, D / 32 values per lane
  for (int q = warp; q < kQC; q += CW + 1) {
    constexpr int PL = D / 32;
    float v[PL];
    float mx = 0.f, nn = 0.f;
    bool bad = q >= nq;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      v[i] = q < nq ? bf16_to_f32(qbf[q * D + lane * PL + i]) : 0.f;
      mx = fmaxf(mx, fabsf(v[i]));
      nn = fmaf(v[i], v[i], nn);
      bad = bad || !(fabsf(v[i]) <= 3.0e38f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      nn += __shfl_xor_sync(0xffffffffu, nn, o);
    }
    bad = __any_sync(0xffffffffu, bad) || !(mx > 0.f);
    const float sq = bad ? 0.f : mx / 127.f;
    const float inv = bad ? 0.f : 127.f / mx;
    float ee = 0.f;
    uint32_t packed[PL / 4];
#pragma unroll
    for (int i = 0; i < PL / 4; ++i) packed[i] = 0u;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int q8 = bad ? 0 : max(-127, min(127, __float2int_rn(v[i] * inv)));
      const float r = v[i] - sq * (float)q8;
      ee = fmaf(r, r, ee);
      packed[i >> 2] |= ((uint32_t)(q8 & 0xff)) << (8 * (i & 3));
    }
    // bytes [lane PL, lane PL + PL) of the row, 4 at a time: chunk c, swizzled
#pragma unroll
    for (int w = 0; w < PL / 4; ++w) {
      const int byte0 = lane * PL + 4 * w;
      const int c = byte0 >> 4;
      const int pos = (c & ~7) | ((c ^ q) & 7);
      *reinterpret_cast<uint32_t*>(qs + q * D + pos * 16 + (byte0 & 15)) = packed[w];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ee += __shfl_xor_sync(0xffffffffu, ee, o);
    if (lane == 0) {
      const float n_q = sqrtf(nn) * (1.f + 1.f / 1024.f);
      const float e_q = sqrtf(ee) * (1.f + 1.f / 1024.f) + n_q * (1.f / 1048576.f);
      qstat[q] = make_float4(sq, e_q, n_q, bad ? 1.f : 0.f);
    }
  }
  if (tid == 0) {
    for (int i = 0; i < n_stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      stage_run[i] = -1;
    }
    abort_s = 0;
    issued_p[0] = issued_p[1] = issued_p[2] = issued_p[3] = 0;
    mbar_init_fence();
  }
  if (n_slots <= kCandCap * kQC * 2)  // the candidate lists (unused until the scoring) hold the histogram
    build_runs_counting<NT>(rt, reinterpret_cast<int*>(&cand[0][0]),
                                   top_idx + ((size_t)s * n_queries + q0) * k, nq * k, k, n_slots);
  else
    build_runs<NT, CW * 32>(rt, nullptr, top_idx + ((size_t)s * n_queries + q0) * k, nq * k, k,
                                        n_slots);
  const int n_runs = rt.n_runs;
  // (the builders end with a CTA barrier: the ring's bf16 query copy is dead)

  // producer lanes: lane p issues the runs r = p (mod np) into the stages
  // r % n_stages, which no other lane touches (np divides n_stages); one
  // issuing thread spends several hundred cycles per run between its barrier
  // waits and copies, which held the ring below what the consumers take
  const int np = n_stages % 4 == 0 ? 4 : (n_stages % 2 == 0 ? 2 : 1);
  if (warp == CW) {
    if (lane < np) {
      // the generic-proxy writes of the query copy precede the ring's copies
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      int r = lane;
      for (; r < n_runs; r += np) {
        const int st = r % n_stages;
        if (!mbar_wait(&empty[st], ((r / n_stages) & 1) ^ 1)) {
          *abort_v = 1;
          break;
        }
        if (*abort_v) break;
        const int b = (int)(rt.keys[rt.run_start[r]] >> 11);
        const int64_t blk = (int64_t)s * n_slots + b;
        stage_run_v[st] = r;
        mbar_arrive_expect_tx(&full[st], key_bytes + side_bytes);
        uint8_t* sb = dyn + (size_t)st * stage_bytes;
#pragma unroll
        for (int kb = 0; kb < NB8; ++kb)
          tma_load_2d(sb + (size_t)kb * L * 128, &tmK8, &full[st], kb * 128, (int)(blk * L));
        bulk_load(side + (size_t)st * side_bytes, k8_scale + blk * (L + 4), side_bytes, &full[st]);
      }
      issued_p[lane] = r;
    }
  } else {
    const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
    const int a_hi = lane >> 4;
    const int bcol = lane & 7;
    const int nt = L / 16;
    uint32_t aoff[KSTEPS];
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      aoff[kk] = (uint32_t)((kk >> 2) * L * 128) + (uint32_t)((((2 * kk + a_hi) & 7) ^ (lane & 7)) << 4);
    for (int r = warp; r < n_runs; r += CW) {
      const int st = r % n_stages;
      if (!wait_stage(stage_run_v, full, abort_v, st, r, n_stages)) break;
      const int p0 = rt.run_start[r], p1 = rt.run_start[r + 1];
      const int b = (int)(rt.keys[p0] >> 11);
      const uint32_t abase = base + st * stage_bytes + a_row * 128;
      const float* sk = reinterpret_cast<const float*>(side + (size_t)st * side_bytes);
      const float E = sk[L], N = sk[L + 1];
      // the stage is handed back as soon as its last key tile and scales are
      // in registers, so the producer refills it while this warp finishes the
      // block's selection work (with as many stages as consumer warps, a run
      // and the run CW later share a stage: a warp's next block is requested
      // only when its current one is released)
      bool released = false;
      if (!(E <= 3.0e38f)) {
        // a key of this block has a non-finite value: its queries are scored in full
        for (int pp = p0 + lane; pp < p1; pp += 32) qstat[rt.keys[pp] & 2047u].w = 1.f;
      } else {
        for (int g0 = p0; g0 < p1; g0 += 8) {
          const int pn = g0 + bcol;
          const int qn = pn < p1 ? (int)(rt.keys[pn] & 2047u) : -1;
          uint32_t bq[KSTEPS][2];
#pragma unroll
          for (int kk = 0; kk < KSTEPS; kk += 2) {
            const int c = 2 * kk + (lane >> 3);
            const uint32_t addr =
                qn >= 0 ? qs_u + qn * D + (uint32_t)(((c & ~7) | ((c ^ qn) & 7)) << 4) : zrow_u + (uint32_t)(c << 4);
            ldsm_x4(addr, bq[kk][0], bq[kk][1], bq[kk + 1][0], bq[kk + 1][1]);
          }
          // this lane's two query columns (pairs g0 + 2 (lane % 4) and + 1):
          // scale s_q and the block's bound b
          int qc[2];
          float sq[2], bq_[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int pj = g0 + 2 * (lane & 3) + j;
            qc[j] = pj < p1 ? (int)(rt.keys[pj] & 2047u) : -1;
            const float4 st4 = qc[j] >= 0 ? qstat[qc[j]] : make_float4(0.f, 0.f, 0.f, 1.f);
            sq[j] = st4.x;
            float bb = fmaf(st4.z, E, st4.y * (N + E)) + slack * st4.z * N;
            bb += (bb + (st4.z + st4.y) * (N + E)) * (1.f / 1048576.f);
            bq_[j] = bb;
          }
          float amax[2] = {-INFINITY, -INFINITY};
          float av[4][4];  // A of the 16 (token, query) pairs this lane holds
          for (int t = 0; t < nt; t += 4) {
            const int tn = min(4, nt - t);  // 16-row tiles of this group (the last may hold fewer)
            int acc[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0;
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (u < tn) {
                  uint32_t a0, a1, a2, a3;
                  ldsm_x4(abase + (uint32_t)((t + u) * 16 * 128) + aoff[kk], a0, a1, a2, a3);
                  mma_i8_16832(acc[u], a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
                }
              }
            }
            float sc0[4], sc1[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int row = (t + u) * 16 + (lane >> 2);
              sc0[u] = u < tn ? sk[row] : 0.f;
              sc1[u] = u < tn ? sk[row + 8] : 0.f;
            }
            if (g0 + 8 >= p1 && t + 4 >= nt) {  // the run's last reads of the stage are done
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[st]);
              released = true;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = e & 1;
                av[u][e] = u < tn ? (float)acc[u][e] * ((e & 2) ? sc1[u] : sc0[u]) * sq[j] : -INFINITY;
              }
            }
            // column maxima as a tree (fmaxf is exact, so the order is free)
#pragma unroll
            for (int j = 0; j < 2; ++j)
              amax[j] = fmaxf(fmaxf(fmaxf(av[0][j], av[0][j + 2]), fmaxf(av[1][j], av[1][j + 2])),
                              fmaxf(fmaxf(av[2][j], av[2][j + 2]), fmaxf(av[3][j], av[3][j + 2])));
            // LB of each column: max over the 8 lanes that hold it, then over the
            // CTA.  The atomicMax returns the CTA's LB before this warp's
            // contribution, so max(old, own) is the LB right after it -- a valid
            // lower bound without a second read (any LB at or below the final
            // one prunes correctly; the final filter uses the final LB)
            float lbc[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              float m = amax[j];
#pragma unroll
              for (int o = 4; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
              const uint32_t own = ord_u32(m - bq_[j]);
              uint32_t lb = own;
              if ((lane >> 2) == 0 && qc[j] >= 0) lb = max(atomicMax(&lbk[qc[j]], own), own);
              lb = __shfl_sync(0xffffffffu, lb, lane & 3);  // lanes t, t + 4, ... hold column 2t + j
              lbc[j] = qc[j] >= 0 ? ord_f32(lb) - bq_[j] : INFINITY;
            }
            // candidates: A >= LB - b, i.e. A + b >= LB; most pairs fail, so
            // the tests come first as one mask and the appends only run for it
            uint32_t pass = 0u;
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int e = 0; e < 4; ++e) pass |= (av[u][e] >= lbc[e & 1] ? 1u : 0u) << (4 * u + e);
            if (pass != 0u) {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = e & 1;
                  if ((pass >> (4 * u + e)) & 1u) {
                    const int row = (t + u) * 16 + (lane >> 2) + ((e & 2) ? 8 : 0);
                    const int slot = atomicAdd(&ccount[qc[j]], 1);
                    if (slot < kCandCap)
                      cand[qc[j]][slot] = make_uint2((uint32_t)(b * L + row), __float_as_uint(av[u][e] + bq_[j]));
                  }
                }
              }
            }
          }
        }
      }
      if (!released) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
    }
  }
  __syncthreads();
  if (tid == CW * 32 && *abort_v) {
    // wait (bounded) for every lane's copies still in flight, then report
    for (int p = 0; p < np; ++p)
      for (int r = max(p, issued_p[p] - n_stages); r < issued_p[p]; r += np)
        mbar_wait(&full[r % n_stages], (r / n_stages) & 1);
    atomicExch(&g_readout_error, (unsigned)GFST_ERR_TIMEOUT);
  }
  // exact re-score of the surviving candidates, flattened over the chunk: the
  // (query, token) pairs with A + b >= the query's final LB are listed in the
  // (now idle) run table, one thread per pair computes the fp32 score from
  // the bf16 rows, and one thread per query takes the best of its pairs in
  // the total order.  Queries scored in full take a warp each afterwards.
  int* pair_off = reinterpret_cast<int*>(rt.run_start);     // [kQC + 1]
  uint32_t* pair_tok = rt.keys;                             // [<= kQC * kCandCap]
  float* pair_score = reinterpret_cast<float*>(dyn);        // the idle ring
  if (!*abort_v) {
    if (warp == 0) {
      int n_keep[2], ex[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q = lane + 32 * h;
        n_keep[h] = 0;
        if (q < nq && qstat[q].w == 0.f && ccount[q] <= kCandCap) {
          const float lb = ord_f32(lbk[q]);
          for (int j = 0; j < ccount[q]; ++j) n_keep[h] += __uint_as_float(cand[q][j].y) >= lb ? 1 : 0;
        }
      }
      int base = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int incl = n_keep[h];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        ex[h] = base + incl - n_keep[h];
        base += __shfl_sync(0xffffffffu, incl, 31);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q = lane + 32 * h;
        pair_off[q] = ex[h];
        if (n_keep[h] > 0) {
          const float lb = ord_f32(lbk[q]);
          int w = ex[h];
          for (int j = 0; j < ccount[q]; ++j)
            if (__uint_as_float(cand[q][j].y) >= lb) pair_tok[w++] = ((uint32_t)q << 24) | cand[q][j].x;
        }
      }
      if (lane == 0) pair_off[kQC] = base;
    }
    __syncthreads();
    const int n_pairs = pair_off[kQC];
    for (int p = tid; p < n_pairs; p += NT) {
      const uint32_t e = pair_tok[p];
      const int q = (int)(e >> 24), tok = (int)(e & 0xffffffu);
      pair_score[p] = bf16_row_dot(pool_K + (((size_t)s * n_slots) * L + tok) * D, Qc + (size_t)q * D, D);
    }
    __syncthreads();
    if (tid < nq) {
      float bs = __int_as_float(0x7fc00000);
      int bi = 0x7fffffff;
      for (int p = pair_off[tid]; p < pair_off[tid + 1]; ++p) {
        const int tok = (int)(pair_tok[p] & 0xffffffu);
        if (better(pair_score[p], tok, bs, bi)) {
          bs = pair_score[p];
          bi = tok;
        }
      }
      best[tid] = (bi != 0x7fffffff && bs == bs) ? pack_best(bs, bi) : 0ull;
    }
    // queries scored in full: a warp each, lanes over the tokens of each selected block
    for (int ql = warp; ql < nq; ql += CW + 1) {
      if (!(qstat[ql].w != 0.f || ccount[ql] > kCandCap)) continue;
      const __nv_bfloat16* qrow = Qc + (size_t)ql * D;
      float bs = __int_as_float(0x7fc00000);
      int bi = 0x7fffffff;
      const int32_t* sel = top_idx + ((size_t)s * n_queries + q0 + ql) * k;
      for (int j = 0; j < k; ++j) {
        const int b = __ldg(sel + j);
        if (b < 0 || b >= n_slots) continue;
        for (int p = lane; p < L; p += 32) {
          const int tok = b * L + p;
          const float v = bf16_row_dot(pool_K + (((size_t)s * n_slots) * L + tok) * D, qrow, D);
          if (better(v, tok, bs, bi)) {
            bs = v;
            bi = tok;
          }
        }
      }
      warp_best(bs, bi);
      if (lane == 0) best[ql] = (bi != 0x7fffffff && bs == bs) ? pack_best(bs, bi) : 0ull;
    }
  }
  __syncthreads();
  // outputs, flattened: the value rows move as 16-byte chunks over all threads
  const int64_t sq0 = (int64_t)s * n_queries + q0;
  if (tid < nq) {
    const unsigned long long key = best[tid];
    const bool found = key != 0ull;
    best_tok[sq0 + tid] = found ? (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : -1;
    best_score[sq0 + tid] = found ? unpack_score(key) : -INFINITY;
  }
  if (out_V != nullptr) {
    const int vv = dv / 8;
    for (int e = tid; e < nq * vv; e += NT) {
      const int ql = e / vv, c = e - ql * vv;
      const unsigned long long key = best[ql];
      uint4 v = make_uint4(0, 0, 0, 0);
      if (key != 0ull) {
        const int tok = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
        const int bb = tok / L, p = tok % L;
        v = __ldg(reinterpret_cast<const uint4*>(pool_V + (((size_t)s * n_slots + bb) * L + p) * dv) + c);
      }
      reinterpret_cast<uint4*>(out_V + (sq0 + ql) * dv)[c] = v;
    }
  }
}

// int8 copy of one committed block per stream: one CTA per stream, a warp per
// token row (D / 32 values per lane).  Per token the scale s = max|k| / 127;
// per block E >= max |k - s k8|_2 and N >= max |k|_2 (fp32 norms rounded up by
// a relative 2^-10, plus 2^-20 of N on E; +inf for a non-finite key) follow
// the L scales in k8_scale [.., L + 4] as (E, N, 0, 0).
template <int PL>
__global__ void __launch_bounds__(256) block_commit_i8_kernel(const __nv_bfloat16* __restrict__ K,
                                                              int8_t* __restrict__ pool_K8,
                                                              float* __restrict__ k8_scale, int n_slots, int slot,
                                                              int L) {
  constexpr int D = PL * 32;
  __shared__ float red_e[8], red_n[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t s = blockIdx.x;
  const int64_t blk = s * n_slots + slot;
  float emax = 0.f, nmax = 0.f;
  for (int p = warp; p < L; p += 8) {
    const __nv_bfloat16* src = K + (s * L + p) * D;
    float v[PL];
    float mx = 0.f, nn = 0.f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      v[i] = bf16_to_f32(src[lane * PL + i]);
      mx = fmaxf(mx, fabsf(v[i]));
      nn = fmaf(v[i], v[i], nn);
      bad = bad || !(fabsf(v[i]) <= 3.0e38f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      nn += __shfl_xor_sync(0xffffffffu, nn, o);
    }
    bad = __any_sync(0xffffffffu, bad);
    const float sk = (bad || !(mx > 0.f)) ? 0.f : mx / 127.f;
    const float inv = sk > 0.f ? 127.f / mx : 0.f;
    int8_t* dst = pool_K8 + (blk * L + p) * D + lane * PL;
    float ee = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int q8 = sk > 0.f ? max(-127, min(127, __float2int_rn(v[i] * inv))) : 0;
      const float r = v[i] - sk * (float)q8;
      ee = fmaf(r, r, ee);
      dst[i] = (int8_t)q8;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ee += __shfl_xor_sync(0xffffffffu, ee, o);
    const float n_k = bad ? INFINITY : sqrtf(nn) * (1.f + 1.f / 1024.f);
    const float e_k = bad ? INFINITY : sqrtf(ee) * (1.f + 1.f / 1024.f) + n_k * (1.f / 1048576.f);
    emax = fmaxf(emax, e_k);
    nmax = fmaxf(nmax, n_k);
    if (lane == 0) k8_scale[blk * (L + 4) + p] = sk;
  }
  if (lane == 0) {
    red_e[warp] = emax;
    red_n[warp] = nmax;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) {
      emax = fmaxf(emax, red_e[w]);
      nmax = fmaxf(nmax, red_n[w]);
    }
    // fmaxf drops NaN: a non-finite key already gave +inf
    float* tail = k8_scale + blk * (L + 4) + L;
    tail[0] = emax;
    tail[1] = nmax;
    tail[2] = 0.f;
    tail[3] = 0.f;
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
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    // tensor-core consumers: a ring of GFST_READOUT_RING_KB (5 stages of 16 KB for
    // 64 x 128 blocks, 112 KB per CTA with the run table: two CTAs per SM, or
    // one beside a frame-update CTA; 4 stages measured 11 % slower)
    const size_t stage_bytes = (size_t)L * d * 2;
    const bool mma_ok = (d == 64 || d == 128 || d == 256) && L % 16 == 0 && L <= 256 &&
                        (int64_t)NS < (1LL << 21) && S * (int64_t)NS * L < (1LL << 31) &&
                        S * n_chunks <= 0x7fffffffLL && aligned16(Q) && k <= 32;
    // blocks of 32 KB and more: one CTA per SM with a 160 KB ring (five 32 KB
    // stages) keeps more bytes in flight than two CTAs of two stages each
    // (128-token blocks of d = 128: 0.82 against 0.95 ms on the long-memory case)
    int n_stages = (int)((GFST_READOUT_RING_KB * 1024u) / stage_bytes);
    if (stage_bytes >= 32768) n_stages = (int)((160u * 1024u) / stage_bytes);
    n_stages = n_stages < 2 ? 2 : (n_stages > kMaxStages ? kMaxStages : n_stages);
    const size_t dyn = 1024 + (size_t)n_stages * stage_bytes + (size_t)(kQC + 1) * d * 2;
    if (mma_ok && dyn <= 200u * 1024u) {
      CUtensorMap tm;
      const int st = make_bf16_map(&tm, pool_K, (uint64_t)S * NS * L, d, L);
      if (st != GFST_OK) return st;
      const unsigned mgrid = (unsigned)(S * n_chunks);
      cudaError_t e = cudaSuccess;
      switch (d / 64) {
#define GFST_READOUT_MMA(NKBV)                                                                                   \
  case NKBV: {                                                                                                   \
    auto kern = exact_readout_mma_kernel<NKBV>;                                                                  \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);                       \
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));         \
    kern<<<mgrid, kMThreads, dyn, stream>>>(tm, q, pv, top_idx, Nq, (int)n_chunks, NS, L, dv, k, n_stages,       \
                                            best_tok, best_score, ov);                                           \
    return check_launch("exact_readout_mma_kernel");                                                             \
  }
        GFST_READOUT_MMA(1)
        GFST_READOUT_MMA(2)
        GFST_READOUT_MMA(4)
#undef GFST_READOUT_MMA
        default:
          break;
      }
    }
  }
  const size_t block_bytes = (size_t)L * d * sizeof(T);
  // stages: about 80 KB of ring per CTA, 2 to 8 blocks
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

// int8 first look: bf16 pools, d = 128 or 256, L % 16 == 0, L <= 256
int launch_i8(const void* Q, const void* pool_K, const int8_t* pool_K8, const float* k8_scale, const void* pool_V,
              const int32_t* top_idx, int64_t S, int Nq, int NS, int L, int d, int dv, int k, int32_t* best_tok,
              float* best_score, void* out_V, cudaStream_t stream) {
  const int64_t n_chunks = (Nq + kQC - 1) / kQC;
  GFST_REQUIRE(S * n_chunks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many query chunks");
  const size_t stage_bytes = ((size_t)L * d + 1023) & ~(size_t)1023;
  const size_t side_bytes = (size_t)(L + 4) * 4;
  const size_t fixed = 1024 + (size_t)(kQC + 1) * d;  // alignment slack, quantised queries, zero row
  // the ring takes what shared memory leaves beside the kernel's static arrays
  // at two CTAs per SM (d = 128: 8 stages).  Measured on B200, 2048 streams x
  // 64 queries x 16 of 512 blocks: two CTAs of 8 consumer warps 1.50 ms, of 4
  // consumer warps 1.60 ms; one CTA of 8 consumer warps with a 22-stage ring
  // 2.51 ms -- the consumers' per-block chains, not the bytes in flight, set
  // the pace, so more CTAs per SM beat a deeper ring.
  int dev = 0, smem_sm = 0, reserved = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, d == 128 ? (const void*)exact_readout_i8_kernel<1, kI8Warps>
                                                      : (const void*)exact_readout_i8_kernel<2, kI8Warps>);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
  const long long budget = (long long)smem_sm / 2 - reserved - (long long)fa.sharedSizeBytes - (long long)fixed;
  int n_stages = budget > 0 ? (int)(budget / (long long)(stage_bytes + side_bytes)) : 0;
  n_stages = n_stages < 2 ? 2 : (n_stages > kMaxStagesI8 ? kMaxStagesI8 : n_stages);
  // the ring holds the chunk's bf16 queries before the pipeline starts
  while ((size_t)n_stages * stage_bytes < (size_t)kQC * d * 2) ++n_stages;
  const size_t dyn = fixed + (size_t)n_stages * (stage_bytes + side_bytes);
  CUtensorMap tm;
  const int st = make_u8_map(&tm, pool_K8, (uint64_t)S * NS * L, d, L);
  if (st != GFST_OK) return st;
  // fp32 rounding of A and of an fp32 evaluation of the exact score: 2 d + 16 units of 2^-24
  const float slack = (float)(2 * d + 16) / 16777216.f;
  const unsigned grid = (unsigned)(S * n_chunks);
#define GFST_READOUT_I8(NB, CWV)                                                                                  \
  {                                                                                                               \
    auto kern = exact_readout_i8_kernel<NB, CWV>;                                                                 \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);                        \
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));          \
    kern<<<grid, (CWV + 1) * 32, dyn, stream>>>(tm, static_cast<const __nv_bfloat16*>(Q),                               \
                                           static_cast<const __nv_bfloat16*>(pool_K),                             \
                                           k8_scale,                                                              \
                                           static_cast<const __nv_bfloat16*>(pool_V), top_idx, Nq, (int)n_chunks, \
                                           NS, L, dv, k, n_stages, slack, best_tok, best_score,                  \
                                           static_cast<__nv_bfloat16*>(out_V));                                   \
    return check_launch("exact_readout_i8_kernel");                                                                \
  }
  if (d == 128) GFST_READOUT_I8(1, kI8Warps)
  GFST_READOUT_I8(2, kI8Warps)
#undef GFST_READOUT_I8
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

extern "C" int gfst_block_commit_i8(const void* K, int8_t* pool_K8, float* k8_scale, int64_t n_streams, int n_slots,
                                    int slot, int L, int d, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_slots >= 1 && L >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(slot >= 0 && slot < n_slots, GFST_ERR_ARG, "slot %d outside [0, %d)", slot, n_slots);
  GFST_REQUIRE(d == 128 || d == 256, GFST_ERR_SHAPE, "int8 key copies cover d = 128 or 256 (d=%d)", d);
  GFST_REQUIRE(n_streams <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many streams");
  if (n_streams == 0) return GFST_OK;
  GFST_REQUIRE(K && pool_K8 && k8_scale, GFST_ERR_ARG, "null buffer");
  if (d == 128)
    block_commit_i8_kernel<4><<<(unsigned)n_streams, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(K), pool_K8,
                                                                       k8_scale, n_slots, slot, L);
  else
    block_commit_i8_kernel<8><<<(unsigned)n_streams, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(K), pool_K8,
                                                                       k8_scale, n_slots, slot, L);
  return check_launch("block_commit_i8_kernel");
}

extern "C" int gfst_exact_readout_i8(const void* Q, const void* pool_K, const int8_t* pool_K8, const float* k8_scale,
                                     const void* pool_V, const int32_t* top_idx, int64_t n_streams, int n_queries,
                                     int n_slots, int L, int d, int dv, int k, int32_t* best_tok, float* best_score,
                                     void* out_V, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_slots >= 1 && L >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(k >= 1 && k <= 32, GFST_ERR_SHAPE, "k=%d outside [1, 32]", k);
  GFST_REQUIRE(d == 128 || d == 256, GFST_ERR_SHAPE, "the int8 first look covers d = 128 or 256 (d=%d)", d);
  GFST_REQUIRE(L % 16 == 0 && L <= 256, GFST_ERR_SHAPE, "the int8 first look needs L %% 16 == 0 and L <= 256 (L=%d)",
               L);
  GFST_REQUIRE(dv % 8 == 0, GFST_ERR_ALIGN, "dv=%d must be a multiple of 8", dv);
  GFST_REQUIRE((pool_V == nullptr) == (out_V == nullptr), GFST_ERR_ARG, "pool_V and out_V go together");
  GFST_REQUIRE((int64_t)n_slots * L < (1LL << 24) && n_streams * (int64_t)n_slots * L < (1LL << 31), GFST_ERR_SHAPE,
               "the int8 first look needs n_slots * L < 2^24 (token index)");
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(Q && pool_K && pool_K8 && k8_scale && top_idx && best_tok && best_score, GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(aligned16(Q) && aligned16(pool_K) && aligned16(pool_K8) && aligned16(k8_scale) && aligned16(pool_V) &&
                   aligned16(out_V),
               GFST_ERR_ALIGN, "buffers must be 16-byte aligned");
  return launch_i8(Q, pool_K, pool_K8, k8_scale, pool_V, top_idx, n_streams, n_queries, n_slots, L, d, dv, k,
                   best_tok, best_score, out_V, stream);
}
