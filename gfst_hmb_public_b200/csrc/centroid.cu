// Centroid path of the exact-token memory.
//
// Reference (pkhairkh/gfst-hmb-public):
//   cell write  -- GfstDecodeState._append_exact_token_cuda_packed
//                  (src/gfst_hmb_mpuc/state.py:315-470) per token, and
//                  _finalise_block_cells (state.py:501-551) at block end:
//                  u8 cell ids (clamped to [0, C-1]), weights quantised
//                  round(w * 255) clamped to [0, 255]; per cell the sums of
//                  (q/255) * key, (q/255) * value and q/255 over the block's
//                  tokens (positive weights only, token then membership order);
//                  mean key in fp16, round(mean value * 32) in int8 [-127, 127],
//                  round(count * 32) in int16 [0, 32767].
//   readout     -- ExactRecallReadout._build_centroid_candidates
//                  (src/gfst_hmb_mpuc/modeling.py:659-982) on the selected
//                  blocks, then the log-sum-exp collapse by token id and the
//                  best group (perf.py:164-229, modeling.py:1151-1169).
//
// gfst_centroid_cell_commit: one CTA per block, one thread per (cell, dim)
// sum, exact IEEE operations in the reference's order (no contraction).
//
// gfst_centroid_readout: one CTA per (stream, query).  The candidate cells of
// the selected blocks (count > 0) are compacted in selection order; per
// centroid head the raw cell scores, robust z-scores (lower medians of the
// scores and of their absolute deviations by bitonic sorts in shared memory),
// count penalty and self field; the cells ordered by z (descending, lower
// index first), the BH-FDR cut on their p-values 0.5 erfc(z / sqrt 2), the
// minimum-count fallback, softmax weights and the activation mass of each
// (block, cell); then one thread per candidate token: base score q . k, token
// mass, centroid-recall log-sum-exp over (head, selected cell), final score;
// last the collapse by token id and the best group.  p-values fall as z
// rises, so ranking cells by z orders them as the reference's p-value sort
// does (they differ only among cells whose p-values round equal).
#include <math.h>
#include <cuda_fp16.h>

#include "gfst_common.cuh"

namespace gfst {
namespace {

// ---------------------------------------------------------------------------
// cell write
// ---------------------------------------------------------------------------
constexpr int kCellThreads = 256;
constexpr int kMaxCellTokens = 1024;  // L * W

__global__ void __launch_bounds__(kCellThreads) centroid_cell_commit_kernel(
    const int32_t* __restrict__ cell_ids, const float* __restrict__ cell_weights, const float* __restrict__ keys,
    const float* __restrict__ values, int L, int W, int C, int dk, int dv, uint8_t* __restrict__ out_ids,
    uint8_t* __restrict__ out_wq, __half* __restrict__ cell_keys, int8_t* __restrict__ cell_values_q,
    int16_t* __restrict__ cell_counts) {
  __shared__ int s_id[kMaxCellTokens];
  __shared__ float s_w[kMaxCellTokens];  // q / 255, 0 when q == 0
  const int64_t blk = blockIdx.x;
  const int tid = threadIdx.x;
  const int n = L * W;
  for (int i = tid; i < n; i += kCellThreads) {
    int id = cell_ids[blk * n + i];
    id = id < 0 ? 0 : (id > C - 1 ? C - 1 : id);
    float qf = rintf(__fmul_rn(cell_weights[blk * n + i], 255.f));
    qf = qf > 0.f ? (qf < 255.f ? qf : 255.f) : 0.f;  // NaN -> 0
    const uint8_t q = (uint8_t)qf;
    out_ids[blk * n + i] = (uint8_t)id;
    out_wq[blk * n + i] = q;
    s_id[i] = id;
    s_w[i] = q > 0 ? __fdiv_rn((float)q, 255.f) : 0.f;
  }
  __syncthreads();
  // counts (state.py:413), then keys and values (state.py:411-412)
  for (int c = tid; c < C; c += kCellThreads) {
    float cnt = 0.f;
    for (int i = 0; i < n; ++i)
      if (s_id[i] == c && s_w[i] > 0.f) cnt = __fadd_rn(cnt, s_w[i]);
    cell_counts[blk * C + c] = (int16_t)fminf(fmaxf(rintf(__fmul_rn(cnt, 32.f)), 0.f), 32767.f);
  }
  for (int j = tid; j < C * (dk + dv); j += kCellThreads) {
    const bool is_key = j < C * dk;
    const int c = is_key ? j / dk : (j - C * dk) / dv;
    const int e = is_key ? j % dk : (j - C * dk) % dv;
    float sum = 0.f, cnt = 0.f;
    for (int i = 0; i < n; ++i) {
      if (s_id[i] == c && s_w[i] > 0.f) {
        const int t = i / W;
        const float x = is_key ? keys[(blk * L + t) * dk + e] : values[(blk * L + t) * dv + e];
        sum = __fadd_rn(sum, __fmul_rn(s_w[i], x));
        cnt = __fadd_rn(cnt, s_w[i]);
      }
    }
    const float mean = cnt > 0.f ? __fdiv_rn(sum, fmaxf(cnt, 1.f)) : 0.f;  // state.py:528-537
    if (is_key) {
      cell_keys[(blk * C + c) * dk + e] = __float2half_rn(mean);
    } else {
      cell_values_q[(blk * C + c) * dv + e] = (int8_t)fminf(fmaxf(rintf(__fmul_rn(mean, 32.f)), -127.f), 127.f);
    }
  }
}

// ---------------------------------------------------------------------------
// readout
// ---------------------------------------------------------------------------
constexpr int kRThreads = 256;
constexpr int kMaxEntries = 32;   // K
constexpr int kMaxCells = 512;    // K * C candidate cells
constexpr int kMaxHeads = 8;
constexpr int kMaxDk = 64;
constexpr int kMaxDv = 32;
constexpr int kMaxWidth = 16;
constexpr int kMaxCand = 2048;    // K * L candidate tokens
constexpr int kMaxDq = 256;
constexpr int kPairsPerLane = kMaxHeads * kMaxWidth / 32;
constexpr int kRegDv = 16;  // value dims held in registers on the register recall path
static_assert(kMaxCand + (kRThreads / 32) * kMaxHeads * kMaxDv <= kMaxHeads * kMaxCells,
              "token-phase buffers fit the z-score area");
constexpr float kSqrt2 = 1.41421356237309515f;  // (float) math.sqrt(2.0)

__device__ __forceinline__ uint32_t orderable(float x) {  // ascending float order as u32
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ascending bitonic sort of key[0, n_pow2) by the whole block
__device__ void block_sort(unsigned long long* key, int n_pow2) {
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int e = threadIdx.x; e < n_pow2; e += blockDim.x) {
        const int partner = e ^ stride;
        if (partner > e) {
          const bool up = (e & size) == 0;
          const unsigned long long a = key[e], b = key[partner];
          if ((a > b) == up) {
            key[e] = b;
            key[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

struct __align__(16) ReadoutSmem {
  float q[kMaxDq];
  float qh[kMaxHeads * kMaxDk];
  int s_sel[kMaxEntries], s_prefix[kMaxEntries];
  float s_score[kMaxEntries];
  int s_count[kMaxCells];
  int e_slot[kMaxEntries], e_k[kMaxEntries], e_prefix[kMaxEntries], e_nvalid[kMaxEntries], e_base[kMaxEntries];
  float e_score[kMaxEntries], e_selfmean[kMaxEntries];
  int c_entry[kMaxCells], c_cell[kMaxCells];
  float c_count[kMaxCells];  // count_q / 32
  float c_self[kMaxCells];   // log1p(count_q) - block mean
  union {
    float z[kMaxHeads][kMaxCells];  // selection phase
    struct {                        // token phase
      float cand[kMaxCand];
      float feat[kRThreads / 32][kMaxHeads * kMaxDv];
    };
  };
  unsigned long long key[kMaxCand];
  int sel[kMaxHeads][kMaxWidth];  // selected cell (index into the compacted list)
  float sel_alpha[kMaxHeads][kMaxWidth], sel_logalpha[kMaxHeads][kMaxWidth];
  alignas(16) float sel_val[kMaxHeads][kMaxWidth][kMaxDv + 4];  // 16-byte rows, spread over banks
  int pair_h[kMaxHeads * kMaxWidth], pair_j[kMaxHeads * kMaxWidth];
  int sel_count[kMaxHeads];
  float h_entropy[kMaxHeads], h_margin[kMaxHeads], h_signif[kMaxHeads];
  float mass[kMaxEntries * 32];
  float wlut[256];  // q / 255
  float red[kRThreads / 32];
  int n_entries, n_cells, upto, n_pairs;
  float conf;
};

__global__ void __launch_bounds__(kRThreads, 3) centroid_readout_kernel(
    const float* __restrict__ Q, const float* __restrict__ query_heads, const int32_t* __restrict__ sel_idx,
    const float* __restrict__ sel_scores, const int32_t* __restrict__ prefix_len, const float* __restrict__ tok_keys,
    const float* __restrict__ tok_feats, const int32_t* __restrict__ tok_ids, const uint8_t* __restrict__ tok_cell,
    const uint8_t* __restrict__ tok_wq, const __half* __restrict__ cell_keys, const int8_t* __restrict__ cell_vals,
    const int16_t* __restrict__ cell_counts, int Nq, int NB, int L, int dq, int H, int dk, int dv, int C, int W, int K,
    gfst_centroid_params prm, float sqrt_dk, float sqrt_dv, float* __restrict__ cand_out,
    int32_t* __restrict__ best_id, float* __restrict__ best_score, int32_t* __restrict__ best_block,
    int32_t* __restrict__ best_pos, int32_t* __restrict__ out_sel_block, int32_t* __restrict__ out_sel_cell,
    float* __restrict__ out_sel_alpha, float* __restrict__ out_head_stats, float* __restrict__ out_conf) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ReadoutSmem& sm = *reinterpret_cast<ReadoutSmem*>(smem_raw);
  const int64_t sq = blockIdx.x;
  const int64_t s = sq / Nq;
  const int tid = threadIdx.x;
  const int width = prm.top_cells_per_head;

  for (int i = tid; i < dq; i += kRThreads) sm.q[i] = Q[sq * dq + i];
  for (int i = tid; i < H * dk; i += kRThreads) sm.qh[i] = query_heads[sq * H * dk + i];
  // selections and their cell counts, staged by all threads (global loads in
  // parallel), then the entry list in selection order (modeling.py:1091-1108)
  for (int k = tid; k < K; k += kRThreads) {
    const int b = sel_idx[sq * K + k];
    int p = prefix_len ? prefix_len[sq * K + k] : L;
    p = p > L ? L : p;
    sm.s_sel[k] = (b < 0 || b >= NB || p <= 0) ? -1 : b;
    sm.s_prefix[k] = p;
    sm.s_score[k] = sel_scores[sq * K + k];
  }
  __syncthreads();
  for (int i = tid; i < K * C; i += kRThreads) {
    const int b = sm.s_sel[i / C];
    sm.s_count[i] = b >= 0 ? cell_counts[((s * NB) + b) * C + i % C] : 0;
  }
  __syncthreads();
  if (tid == 0) {
    int ne = 0, nc = 0;
    for (int k = 0; k < K; ++k) {
      if (sm.s_sel[k] < 0) continue;
      sm.e_slot[ne] = sm.s_sel[k];
      sm.e_k[ne] = k;
      sm.e_prefix[ne] = sm.s_prefix[k];
      sm.e_score[ne] = sm.s_score[k];
      sm.e_base[ne] = nc;
      int nv = 0;
      for (int c = 0; c < C; ++c) nv += sm.s_count[k * C + c] > 0 ? 1 : 0;
      sm.e_nvalid[ne] = nv;
      nc += nv;
      ++ne;
    }
    sm.n_entries = ne;
    sm.n_cells = nc;
  }
  __syncthreads();
  const int ne = sm.n_entries, N = sm.n_cells;
  for (int i = tid; i < kMaxEntries * 32; i += kRThreads) sm.mass[i] = 0.f;
  // compacted cells (modeling.py:690-727) and the per-block self field
  for (int e = tid; e < ne; e += kRThreads) {
    const int* cc = sm.s_count + sm.e_k[e] * C;
    int o = sm.e_base[e];
    float lsum = 0.f;
    for (int c = 0; c < C; ++c) {
      if (cc[c] <= 0) continue;
      sm.c_entry[o] = e;
      sm.c_cell[o] = c;
      sm.c_count[o] = __fdiv_rn((float)cc[c], 32.f);
      sm.c_self[o] = log1pf(fmaxf((float)cc[c], 0.f));
      lsum += sm.c_self[o];
      ++o;
    }
    sm.e_selfmean[e] = sm.e_nvalid[e] > 0 ? __fdiv_rn(lsum, (float)sm.e_nvalid[e]) : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < N; i += kRThreads) sm.c_self[i] = sm.c_self[i] - sm.e_selfmean[sm.c_entry[i]];
  // raw scores (modeling.py:739-745): one thread per cell, every head, the
  // cell's key read once
  for (int n = tid; n < N; n += kRThreads) {
    const int e = sm.c_entry[n];
    const __half* key = cell_keys + (((s * NB) + sm.e_slot[e]) * C + sm.c_cell[n]) * dk;
    float acc[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) acc[h] = 0.f;
    for (int j = 0; j < dk; ++j) {
      const float kj = __half2float(key[j]);
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < H) acc[h] = fmaf(sm.qh[h * dk + j], kj, acc[h]);
    }
    const float bias = __fmul_rn(prm.block_score_lambda, sm.e_score[e]);
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h)
      if (h < H) sm.z[h][n] = __fadd_rn(__fdiv_rn(acc[h], sqrt_dk), bias);
  }
  __syncthreads();
  bool centroid_on = N > 0 && width > 0;
  int n_pow2 = 1;
  while (n_pow2 < N) n_pow2 <<= 1;
  if (centroid_on) {
    for (int h = 0; h < H; ++h) {
      // robust z-score (modeling.py:747-760)
      float med = 0.f;
      if (prm.background_subtract) {
        for (int i = tid; i < n_pow2; i += kRThreads)
          sm.key[i] = i < N ? ((unsigned long long)orderable(sm.z[h][i]) << 32) : ~0ull;
        __syncthreads();
        block_sort(sm.key, n_pow2);
        const uint32_t u = (uint32_t)(sm.key[(N - 1) / 2] >> 32);
        med = __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
      }
      for (int i = tid; i < n_pow2; i += kRThreads)
        sm.key[i] = i < N ? ((unsigned long long)orderable(fabsf(__fsub_rn(sm.z[h][i], med))) << 32) : ~0ull;
      __syncthreads();
      block_sort(sm.key, n_pow2);
      const uint32_t um = (uint32_t)(sm.key[(N - 1) / 2] >> 32);
      const float mad = __uint_as_float((um & 0x80000000u) ? (um & 0x7fffffffu) : ~um);
      const float sigma = fmaxf(__fmul_rn(1.4826f, mad), 1e-4f);
      for (int i = tid; i < N; i += kRThreads) {
        float zz = __fdiv_rn(__fsub_rn(sm.z[h][i], med), sigma);
        zz = __fsub_rn(zz, __fmul_rn(prm.count_penalty, log1pf(fmaxf(sm.c_count[i], 0.f))));
        zz = __fadd_rn(zz, __fmul_rn(prm.self_field_weight, sm.c_self[i]));
        sm.z[h][i] = zz;
      }
      __syncthreads();
      // order by z descending, index ascending; BH-FDR cut (modeling.py:805-821)
      for (int i = tid; i < n_pow2; i += kRThreads)
        sm.key[i] = i < N ? (((unsigned long long)(~orderable(sm.z[h][i]))) << 32) | (uint32_t)i : ~0ull;
      if (tid == 0) sm.upto = 0;
      __syncthreads();
      block_sort(sm.key, n_pow2);
      int my_upto = 0;
      for (int r = tid; r < N; r += kRThreads) {
        const float zz = sm.z[h][(int)(uint32_t)sm.key[r]];
        const float p = __fmul_rn(0.5f, erfcf(__fdiv_rn(zz, kSqrt2)));
        const float thr = __fmul_rn(prm.fdr_q, __fdiv_rn((float)(r + 1), (float)N));
        if (p <= thr) my_upto = r + 1;
      }
      atomicMax(&sm.upto, my_upto);
      __syncthreads();
      const int topk = min(width, N);
      int kept = sm.upto;
      if (kept < prm.min_selected) kept = min(prm.min_selected, topk);  // modeling.py:826-830
      const int kc = min(width, kept);
      if (tid == 0) {
        sm.sel_count[h] = kc;
        float m = -INFINITY;
        for (int j = 0; j < kc; ++j) m = fmaxf(m, __fdiv_rn(sm.z[h][(int)(uint32_t)sm.key[j]], prm.temperature));
        float sum = 0.f;
        float ex[kMaxWidth];
        for (int j = 0; j < kc; ++j) {
          ex[j] = expf(__fsub_rn(__fdiv_rn(sm.z[h][(int)(uint32_t)sm.key[j]], prm.temperature), m));
          sum += ex[j];
        }
        float ent = 0.f, sig = 0.f;
        for (int j = 0; j < kMaxWidth; ++j) {
          if (j < kc) {
            const int n = (int)(uint32_t)sm.key[j];
            const float a = __fdiv_rn(ex[j], sum);
            sm.sel[h][j] = n;
            sm.sel_alpha[h][j] = a;
            sm.sel_logalpha[h][j] = logf(fmaxf(a, 1e-8f));
            const float ac = fmaxf(a, 1e-8f);
            ent += ac * logf(ac);
            const float p = __fmul_rn(0.5f, erfcf(__fdiv_rn(sm.z[h][n], kSqrt2)));
            sig += -log10f(fmaxf(p, 1e-12f));
          } else {
            sm.sel[h][j] = -1;
            sm.sel_alpha[h][j] = 0.f;
            sm.sel_logalpha[h][j] = -INFINITY;
          }
        }
        sm.h_entropy[h] = kc > 1 ? __fdiv_rn(-ent, (float)log((double)kc)) : 0.f;
        sm.h_margin[h] = kc > 1 ? __fsub_rn(sm.z[h][(int)(uint32_t)sm.key[0]], sm.z[h][(int)(uint32_t)sm.key[1]])
                                : 0.f;
        sm.h_signif[h] = kc > 0 ? __fdiv_rn(sig, (float)kc) : 0.f;
        // activation mass (modeling.py:856-864), heads in order
        for (int j = 0; j < kc; ++j) {
          const int n = sm.sel[h][j];
          sm.mass[sm.c_entry[n] * 32 + sm.c_cell[n]] += sm.sel_alpha[h][j];
        }
      }
      __syncthreads();
      for (int i = tid; i < kMaxWidth * dv; i += kRThreads) {
        const int j = i / dv, e = i % dv;
        float v = 0.f;
        if (j < sm.sel_count[h]) {
          const int n = sm.sel[h][j];
          const int8_t* cv = cell_vals + (((s * NB) + sm.e_slot[sm.c_entry[n]]) * C + sm.c_cell[n]) * dv;
          v = __fdiv_rn((float)cv[e], 32.f);
        }
        sm.sel_val[h][j][e] = v;
      }
      __syncthreads();
    }
    // confidence (modeling.py:867-895)
    if (tid == 0) {
      float se = 0.f, ss = 0.f;
      int used = 0;
      for (int h = 0; h < H; ++h) {
        if (sm.sel_count[h] > 0) {
          se += sm.h_entropy[h];
          ss += sm.h_signif[h];
          ++used;
        }
      }
      int np = 0;
      for (int h = 0; h < H; ++h) {
        for (int j = 0; j < sm.sel_count[h]; ++j) {
          sm.pair_h[np] = h;
          sm.pair_j[np] = j;
          ++np;
        }
      }
      sm.n_pairs = np;
      float conf = -1.f;
      if (used > 0) {
        const float me = __fdiv_rn(se, (float)used), ms = __fdiv_rn(ss, (float)used);
        const float ec = fminf(fmaxf(__fdiv_rn(__fsub_rn(prm.entropy_high, me),
                                               fmaxf(1e-6f, __fsub_rn(prm.entropy_high, prm.entropy_low))), 0.f), 1.f);
        const float sc = fminf(fmaxf(__fdiv_rn(ms, 3.f), 0.f), 1.f);
        conf = __fmul_rn(ec, sc);
      }
      sm.conf = conf;
    }
    __syncthreads();
    centroid_on = sm.conf >= 0.f;
  }
  // candidate tokens (modeling.py:904-962; _score_block_tokens 599-657)
  const float gm = centroid_on ? __fmul_rn(prm.gamma_m, sm.conf) : 0.f;
  const float gr = centroid_on ? __fmul_rn(prm.gamma_r, sm.conf) : 0.f;
  const int n_cand = ne * L;
  int c_pow2 = 1;
  while (c_pow2 < n_cand) c_pow2 <<= 1;
  // one warp per candidate token: coalesced key / feature rows, lanes split the
  // base dot product and the (head, selected cell) recall terms
  const int lane = tid & 31, warp = tid >> 5;
  for (int ci = n_cand + tid; ci < c_pow2; ci += kRThreads) sm.key[ci] = ~0ull;
  for (int i = tid; i < 256; i += kRThreads) sm.wlut[i] = __fdiv_rn((float)i, 255.f);
  float qreg[kMaxDq / 32];
#pragma unroll
  for (int t = 0; t < kMaxDq / 32; ++t) qreg[t] = lane + 32 * t < dq ? sm.q[lane + 32 * t] : 0.f;
  // register path of the recall terms: one (head, selected cell) pair per lane,
  // its value row and log-weight in registers
  const bool reg_pairs = centroid_on && sm.n_pairs <= 32 && dv <= kRegDv && (dv & 3) == 0;
  float sv[kRegDv];
  float my_logalpha = -INFINITY;
  int my_h = 0;
  if (reg_pairs) {
    const bool mine = lane < sm.n_pairs;
    const int h = mine ? sm.pair_h[lane] : 0, j = mine ? sm.pair_j[lane] : 0;
#pragma unroll
    for (int u = 0; u < kRegDv; ++u) sv[u] = (mine && u < dv) ? sm.sel_val[h][j][u] : 0.f;
    my_logalpha = mine ? sm.sel_logalpha[h][j] : -INFINITY;
    my_h = h;
  }
  __syncthreads();  // weight table
  // Score of one candidate token from its rows (this lane's part of the key
  // row kx[t] = key[lane + 32 t], of the feature row fx[t]) and its membership
  // (lanes w < W hold cell id and weight w).
  auto finish_token = [&](int ci, int e, int64_t tok, const float* kx, int nkx, const float* fx, int nfx, int tid_tok,
                          int mcell, int mwq) {
    float part = 0.f;
    for (int t = 0; t < nkx; ++t) part = fmaf(kx[t], qreg[t], part);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const float base = part;
    float score = base;
    if (centroid_on) {
      float* fb = sm.feat[warp];
      for (int t = 0; t < nfx; ++t)
        if (lane + 32 * t < H * dv) fb[lane + 32 * t] = fx[t];
      __syncwarp();
      float seed[kPairsPerLane];
      float mx = -INFINITY;
      if (reg_pairs) {
        const float4* f4 = reinterpret_cast<const float4*>(fb + my_h * dv);
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
        for (int u = 0; u < kRegDv; u += 4) {
          if (u < dv) {
            const float4 f = f4[u / 4];
            d0 = fmaf(f.x, sv[u], d0);
            d1 = fmaf(f.y, sv[u + 1], d1);
            d2 = fmaf(f.z, sv[u + 2], d2);
            d3 = fmaf(f.w, sv[u + 3], d3);
          }
        }
        seed[0] = lane < sm.n_pairs ? __fadd_rn(__fdiv_rn((d0 + d1) + (d2 + d3), sqrt_dv), my_logalpha) : -INFINITY;
        mx = seed[0];
#pragma unroll
        for (int t = 1; t < kPairsPerLane; ++t) seed[t] = -INFINITY;
      } else {
#pragma unroll
        for (int t = 0; t < kPairsPerLane; ++t) {
          const int pi = lane + 32 * t;
          seed[t] = -INFINITY;
          if (pi < sm.n_pairs) {
            const int h = sm.pair_h[pi], j = sm.pair_j[pi];
            float d = 0.f;
            for (int u = 0; u < dv; ++u) d = fmaf(fb[h * dv + u], sm.sel_val[h][j][u], d);
            seed[t] = __fadd_rn(__fdiv_rn(d, sqrt_dv), sm.sel_logalpha[h][j]);
            mx = fmaxf(mx, seed[t]);
          }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float se = 0.f;
#pragma unroll
      for (int t = 0; t < kPairsPerLane; ++t)
        if (seed[t] != -INFINITY) se += expf(__fsub_rn(seed[t], mx));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
      const float recall = __fadd_rn(mx, logf(se));
      float tm = 0.f;
      for (int w = 0; w < W; ++w) {  // modeling.py:929-938, memberships in order
        int c = __shfl_sync(0xffffffffu, mcell, w);
        const int q8 = __shfl_sync(0xffffffffu, mwq, w);
        c = c > C - 1 ? C - 1 : c;
        tm = __fadd_rn(tm, __fmul_rn(sm.mass[e * 32 + c], sm.wlut[q8]));
      }
      score = __fadd_rn(__fadd_rn(base, __fmul_rn(gm, tm)), __fmul_rn(gr, recall));
      __syncwarp();  // every lane is done with fb before the next token's rows
    }
    unsigned long long kv = ~0ull;
    if (tid_tok >= 0 && score == score) kv = ((unsigned long long)(uint32_t)tid_tok << 32) | (uint32_t)ci;
    if (lane == 0) {
      sm.cand[ci] = score;
      sm.key[ci] = kv;
      if (cand_out) cand_out[(sq * K + sm.e_k[e]) * L + ci % L] = score;
    }
  };
  auto dead_token = [&](int ci, int e) {
    if (lane == 0) {
      sm.cand[ci] = -INFINITY;
      sm.key[ci] = ~0ull;
      if (cand_out) cand_out[(sq * K + sm.e_k[e]) * L + ci % L] = -INFINITY;
    }
  };
  // Pair path for 4 heads of 16 value dims (the reference's defaults): two
  // threads per candidate token, each with half the key row and two heads'
  // feature rows in registers, the recall log-sum-exp kept online (running
  // max and scaled sum) and merged across the pair by one shuffle.
  const bool pair_path = H == 4 && dv == 16 && (dq & 7) == 0 && dq <= kMaxDq &&
                         ((reinterpret_cast<uintptr_t>(tok_keys) | reinterpret_cast<uintptr_t>(tok_feats)) & 15) == 0;
  if (pair_path) {
    const int half = tid & 1;
    const int dqh = dq / 2;
    for (int cb = 0; cb < n_cand; cb += kRThreads / 2) {
      const int ci = cb + (tid >> 1);
      const bool inb = ci < n_cand;
      const int e = inb ? ci / L : 0, p = inb ? ci % L : 0;
      const bool live = inb && p < sm.e_prefix[e];
      const int64_t tok = live ? ((s * NB) + sm.e_slot[e]) * L + p : 0;
      float score = -INFINITY;
      if (live) {
        const float4* kr = reinterpret_cast<const float4*>(tok_keys + tok * dq + half * dqh);
        const float4* q4 = reinterpret_cast<const float4*>(sm.q + half * dqh);
        float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        for (int j = 0; j < dqh / 4; ++j) {
          const float4 k = kr[j], qq = q4[j];
          b0 = fmaf(k.x, qq.x, b0);
          b1 = fmaf(k.y, qq.y, b1);
          b2 = fmaf(k.z, qq.z, b2);
          b3 = fmaf(k.w, qq.w, b3);
        }
        score = (b0 + b1) + (b2 + b3);
      }
      score += __shfl_xor_sync(0xffffffffu, score, 1);  // base (both halves)
      float m = -INFINITY, ssum = 0.f;
      if (live && centroid_on) {
        const float4* fr = reinterpret_cast<const float4*>(tok_feats + tok * 64 + half * 32);
        float f[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 v = fr[u];
          f[4 * u] = v.x;
          f[4 * u + 1] = v.y;
          f[4 * u + 2] = v.z;
          f[4 * u + 3] = v.w;
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int h = 2 * half + hh;
          for (int j = 0; j < sm.sel_count[h]; ++j) {
            const float4* sv4 = reinterpret_cast<const float4*>(sm.sel_val[h][j]);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float4 v = sv4[u];
              d0 = fmaf(f[16 * hh + 4 * u], v.x, d0);
              d1 = fmaf(f[16 * hh + 4 * u + 1], v.y, d1);
              d2 = fmaf(f[16 * hh + 4 * u + 2], v.z, d2);
              d3 = fmaf(f[16 * hh + 4 * u + 3], v.w, d3);
            }
            const float x = __fadd_rn(__fdiv_rn((d0 + d1) + (d2 + d3), sqrt_dv), sm.sel_logalpha[h][j]);
            if (x > m) {
              ssum = fmaf(ssum, expf(m - x), 1.f);
              m = x;
            } else {
              ssum += expf(x - m);
            }
          }
        }
      }
      // every thread takes part in the pair exchange (the two threads of a
      // token agree on live)
      const float m2 = __shfl_xor_sync(0xffffffffu, m, 1), s2 = __shfl_xor_sync(0xffffffffu, ssum, 1);
      if (live && centroid_on) {
        const float mm = fmaxf(m, m2);
        const float se = (m == -INFINITY ? 0.f : ssum * expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mm));
        const float recall = __fadd_rn(mm, logf(se));
        float tm = 0.f;
        for (int w = 0; w < W; ++w) {  // modeling.py:929-938, memberships in order
          int c = tok_cell[tok * W + w];
          c = c > C - 1 ? C - 1 : c;
          tm = __fadd_rn(tm, __fmul_rn(sm.mass[e * 32 + c], sm.wlut[tok_wq[tok * W + w]]));
        }
        score = __fadd_rn(__fadd_rn(score, __fmul_rn(gm, tm)), __fmul_rn(gr, recall));
      }
      if (inb && half == 0) {
        unsigned long long kv = ~0ull;
        if (live) {
          const int id = tok_ids[tok];
          if (id >= 0 && score == score) kv = ((unsigned long long)(uint32_t)id << 32) | (uint32_t)ci;
        }
        sm.cand[ci] = live ? score : -INFINITY;
        sm.key[ci] = kv;
        if (cand_out) cand_out[(sq * K + sm.e_k[e]) * L + p] = live ? score : -INFINITY;
      }
    }
  }
  for (int ci = pair_path ? n_cand : warp; ci < n_cand; ci += kRThreads / 32) {
    const int e = ci / L, p = ci % L;
    if (p >= sm.e_prefix[e]) {
      dead_token(ci, e);
      continue;
    }
    const int64_t tok = ((s * NB) + sm.e_slot[e]) * L + p;
    const float* kr = tok_keys + tok * dq;
    const float* fr = tok_feats + tok * H * dv;
    float kx[kMaxDq / 32], fx[kMaxHeads * kMaxDv / 32];
#pragma unroll
    for (int t = 0; t < kMaxDq / 32; ++t) kx[t] = lane + 32 * t < dq ? kr[lane + 32 * t] : 0.f;
#pragma unroll
    for (int t = 0; t < kMaxHeads * kMaxDv / 32; ++t)
      fx[t] = (centroid_on && lane + 32 * t < H * dv) ? fr[lane + 32 * t] : 0.f;
    finish_token(ci, e, tok, kx, kMaxDq / 32, fx, kMaxHeads * kMaxDv / 32, tok_ids[tok],
                 lane < W ? tok_cell[tok * W + lane] : 0, lane < W ? tok_wq[tok * W + lane] : 0);
  }
  if (cand_out) {  // selections that are not valid entries
    for (int i = tid; i < K * L; i += kRThreads) {
      const int k = i / L;
      bool valid = false;
      for (int e = 0; e < ne; ++e) valid |= sm.e_k[e] == k;
      if (!valid) cand_out[sq * K * L + i] = -INFINITY;
    }
  }
  __syncthreads();
  block_sort(sm.key, c_pow2);
  // collapse by token id: group max, first occurrence, LSE (perf.py:164-229)
  float bs = -INFINITY;
  int bid = 0x7fffffff, bcand = -1;
  for (int i = tid; i < n_cand; i += kRThreads) {
    const unsigned long long kv = sm.key[i];
    if (kv == ~0ull) continue;
    const uint32_t id = (uint32_t)(kv >> 32);
    if (i > 0 && sm.key[i - 1] != ~0ull && (uint32_t)(sm.key[i - 1] >> 32) == id) continue;
    float m = -INFINITY;
    int first = -1, end = i;
    for (; end < n_cand && sm.key[end] != ~0ull && (uint32_t)(sm.key[end] >> 32) == id; ++end) {
      const int ci = (int)(uint32_t)sm.key[end];
      if (sm.cand[ci] > m) {
        m = sm.cand[ci];
        first = ci;
      }
    }
    float sum = 0.f;
    for (int j = i; j < end; ++j) sum += expf(sm.cand[(int)(uint32_t)sm.key[j]] - m);
    const float g = m + logf(fmaxf(sum, 1e-8f));
    if (g > bs || (g == bs && (int)id < bid)) {
      bs = g;
      bid = (int)id;
      bcand = first;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bid, o);
    const int c2 = __shfl_xor_sync(0xffffffffu, bcand, o);
    if (s2 > bs || (s2 == bs && i2 < bid)) {
      bs = s2;
      bid = i2;
      bcand = c2;
    }
  }
  __shared__ float r_s[kRThreads / 32];
  __shared__ int r_i[kRThreads / 32], r_c[kRThreads / 32];
  if ((tid & 31) == 0) {
    r_s[tid >> 5] = bs;
    r_i[tid >> 5] = bid;
    r_c[tid >> 5] = bcand;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kRThreads / 32; ++w) {
      if (r_s[w] > bs || (r_s[w] == bs && r_i[w] < bid)) {
        bs = r_s[w];
        bid = r_i[w];
        bcand = r_c[w];
      }
    }
    const bool found = bcand >= 0;
    best_id[sq] = found ? bid : -1;
    best_score[sq] = found ? bs : -INFINITY;
    best_block[sq] = found ? sm.e_slot[bcand / L] : -1;
    best_pos[sq] = found ? bcand % L : -1;
    if (out_conf) out_conf[sq] = centroid_on ? sm.conf : -1.f;
  }
  // diagnostics (modeling.py:966-981): selected entry index / cell / alpha per head
  if (out_sel_block || out_sel_cell || out_sel_alpha) {
    for (int i = tid; i < H * width; i += kRThreads) {
      const int h = i / width, j = i % width;
      const bool on = centroid_on && j < kMaxWidth && j < sm.sel_count[h];
      const int n = on ? sm.sel[h][j] : -1;
      if (out_sel_block) out_sel_block[sq * H * width + i] = on ? sm.c_entry[n] : -1;
      if (out_sel_cell) out_sel_cell[sq * H * width + i] = on ? sm.c_cell[n] : -1;
      if (out_sel_alpha) out_sel_alpha[sq * H * width + i] = on ? sm.sel_alpha[h][j] : 0.f;
    }
  }
  if (out_head_stats) {
    for (int h = tid; h < H; h += kRThreads) {
      out_head_stats[(sq * H + h) * 3 + 0] = centroid_on ? sm.h_entropy[h] : 0.f;
      out_head_stats[(sq * H + h) * 3 + 1] = centroid_on ? sm.h_margin[h] : 0.f;
      out_head_stats[(sq * H + h) * 3 + 2] = centroid_on ? (float)sm.sel_count[h] : 0.f;
    }
  }
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_centroid_cell_commit(const int32_t* cell_ids, const float* cell_weights, const float* cell_keys,
                                         const float* cell_values, int64_t n_blocks, int L, int W, int C, int dk,
                                         int dv, uint8_t* token_cell_ids, uint8_t* token_cell_weights_q,
                                         void* block_cell_keys, int8_t* block_cell_values_q,
                                         int16_t* block_cell_counts, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_blocks >= 0 && L >= 1 && W >= 1 && C >= 1 && dk >= 1 && dv >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE((int64_t)L * W <= kMaxCellTokens, GFST_ERR_SHAPE, "L * W = %lld exceeds %d", (long long)L * W,
               kMaxCellTokens);
  GFST_REQUIRE(C <= 256, GFST_ERR_SHAPE, "cells_per_block %d exceeds 256 (u8 cell ids)", C);
  if (n_blocks == 0) return GFST_OK;
  GFST_REQUIRE(n_blocks <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many blocks");
  GFST_REQUIRE(cell_ids && cell_weights && cell_keys && cell_values && token_cell_ids && token_cell_weights_q &&
                   block_cell_keys && block_cell_values_q && block_cell_counts,
               GFST_ERR_ARG, "null buffer");
  centroid_cell_commit_kernel<<<(unsigned)n_blocks, kCellThreads, 0, stream>>>(
      cell_ids, cell_weights, cell_keys, cell_values, L, W, C, dk, dv, token_cell_ids, token_cell_weights_q,
      static_cast<__half*>(block_cell_keys), block_cell_values_q, block_cell_counts);
  return check_launch("centroid_cell_commit_kernel");
}

extern "C" int gfst_centroid_readout(const float* Q, const float* query_heads, const int32_t* sel_idx,
                                     const float* sel_scores, const int32_t* prefix_len, const float* token_keys,
                                     const float* token_features, const int32_t* token_ids,
                                     const uint8_t* token_cell_ids, const uint8_t* token_cell_weights_q,
                                     const void* cell_keys, const int8_t* cell_values_q, const int16_t* cell_counts,
                                     int64_t n_streams, int n_queries, int n_slots, int L, int dq, int H, int dk,
                                     int dv, int C, int W, int K, const gfst_centroid_params* params,
                                     float* cand_scores, int32_t* best_id, float* best_score, int32_t* best_block,
                                     int32_t* best_pos, int32_t* sel_block, int32_t* sel_cell, float* sel_alpha,
                                     float* head_stats, float* confidence, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(params != nullptr, GFST_ERR_ARG, "params must be non-null");
  const gfst_centroid_params prm = *params;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_slots >= 1 && L >= 1, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(K >= 1 && K <= kMaxEntries, GFST_ERR_SHAPE, "K=%d outside [1, %d]", K, kMaxEntries);
  GFST_REQUIRE(C >= 1 && C <= 32 && K * C <= kMaxCells, GFST_ERR_SHAPE, "C=%d (K*C <= %d, C <= 32)", C, kMaxCells);
  GFST_REQUIRE((int64_t)K * L <= kMaxCand, GFST_ERR_SHAPE, "K * L = %lld exceeds %d", (long long)K * L, kMaxCand);
  GFST_REQUIRE(H >= 1 && H <= kMaxHeads && dk >= 1 && dk <= kMaxDk && dv >= 1 && dv <= kMaxDv, GFST_ERR_SHAPE,
               "heads %d (<= %d), key dim %d (<= %d), value dim %d (<= %d)", H, kMaxHeads, dk, kMaxDk, dv, kMaxDv);
  GFST_REQUIRE(dq >= 1 && dq <= kMaxDq && W >= 1 && W <= 8, GFST_ERR_SHAPE, "query dim %d / membership %d", dq, W);
  GFST_REQUIRE(prm.top_cells_per_head >= 0 && prm.top_cells_per_head <= kMaxWidth, GFST_ERR_SHAPE,
               "top_cells_per_head %d outside [0, %d]", prm.top_cells_per_head, kMaxWidth);
  GFST_REQUIRE(prm.temperature > 0.f, GFST_ERR_ARG, "selection temperature must be positive");
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(Q && query_heads && sel_idx && sel_scores && token_keys && token_features && token_ids &&
                   token_cell_ids && token_cell_weights_q && cell_keys && cell_values_q && cell_counts && best_id &&
                   best_score && best_block && best_pos,
               GFST_ERR_ARG, "null buffer");
  GFST_REQUIRE(n_streams * (int64_t)n_queries <= 0x7fffffffLL, GFST_ERR_SHAPE, "too many queries");
  const size_t smem = sizeof(ReadoutSmem);
  cudaError_t e = cudaFuncSetAttribute(centroid_readout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const float sqrt_dk = (float)sqrt((double)dk), sqrt_dv = (float)sqrt((double)dv);
  centroid_readout_kernel<<<(unsigned)(n_streams * n_queries), kRThreads, smem, stream>>>(
      Q, query_heads, sel_idx, sel_scores, prefix_len, token_keys, token_features, token_ids, token_cell_ids,
      token_cell_weights_q, static_cast<const __half*>(cell_keys), cell_values_q, cell_counts, n_queries, n_slots, L,
      dq, H, dk, dv, C, W, K, prm, sqrt_dk, sqrt_dv, cand_scores, best_id, best_score, best_block, best_pos, sel_block,
      sel_cell, sel_alpha, head_stats, confidence);
  return check_launch("centroid_readout_kernel");
}
