// MPUC recurrent scan: the token loop of MpucGfstHmbBlock._forward_sequence_tensors
// (src/gfst_hmb_mpuc/modeling.py:4449-4476 of pkhairkh/gfst-hmb-public) with its
// cell _token_step (4363-4411), _update_band (4343-4356) and the low-rank
// bridges up(silu(down(x))) (4182-4183).  The reference's own native op
// (mpuc_recurrent_scan_forward, csrc/sm120_stub.cu:210-224) takes no weights
// and returns zeros; this one takes the cell's weights.
//
// Per token and batch element, with F, M, S the fast / mid / slow widths and
// C the bridge rank, nine dependent matrix-vector stages:
//   A  d_fm = silu(D_fm M),  d_fs = silu(D_fs S),  d_ms = silu(D_ms S)     [3C]
//   B  f    = x_fast[t] + U_fm d_fm + U_fs d_fs                            [F]
//   C  g = sigmoid(W_fg f + b), c = tanh(W_fc f + b), F <- (1-g) F + g c   [F]
//   D  d_mf = silu(D_mf F),  d_sf = silu(D_sf F)                           [2C]
//   E  m    = x_mid[t] + U_mf d_mf + U_ms d_ms                             [M]
//   F  gate / candidate of m: M <- (1-g) M + g c                           [M]
//   G  d_sm = silu(D_sm M)                                                 [C]
//   H  s    = x_slow[t] + U_sf d_sf + U_sm d_sm                            [S]
//   I  boundary logit from (mean g_fast, mean g_mid, rms(m - M_prev),
//      rms(s - S_prev)) through the two-layer MLP; S <- (1-g) S + g c with
//      g = sigmoid(W_sg s + b) * sigmoid(logit)                            [S]
// The fused output projection (fusion_proj + the semantic residual) does not
// feed back, so it is not here: it is one batched product over all tokens.
//
// Design: one cooperative launch of one CTA per SM walks all tokens.  Each
// stage's output rows are spread over every warp of the grid (a warp computes
// whole rows, lanes split the dot product, every batch element at once); the
// stage's input vectors are staged in shared memory by each CTA; stages are
// separated by a grid barrier (a monotonically counting word in the caller's
// workspace).  The weights stay in L2 across tokens.  Sums for the boundary
// features are reduced per CTA in warp order and then over CTAs in CTA order:
// the result does not depend on timing.
//
// Every barrier wait is bounded: a CTA whose wait gives up records
// GFST_ERR_TIMEOUT in this file's device error word, raises an abort word that
// the other CTAs' waits also watch, and returns.
#include <algorithm>

#include "gfst_common.cuh"

namespace gfst {

GFST_DEFINE_ERROR_WORD(g_scan_error, read_scan_error, "recurrent scan")

namespace {

constexpr int kScanWarps = 8;
constexpr int kScanThreads = kScanWarps * 32;
constexpr int kScanBatch = 8;                       // batch elements per launch
constexpr long long kScanWaitCycles = 2000000000LL;  // about a second

struct ScanParams {
  gfst_mpuc_weights w;
  int F, M, S, C, BH;
  int B, T;
  const float* x_fast;  // [B, T, F]
  const float* x_mid;   // [B, T, M]
  const float* x_slow;  // [B, T, S]
  float* states;        // [B, T, F + M + S]
  float* logits;        // [B, T]
  float* st_fast;       // [B, F] live state (initial in, final out)
  float* st_mid;        // [B, M]
  float* st_slow;       // [B, S]
  float* ws;            // stage outputs and per-CTA partial sums
  unsigned* bar;        // [0]: barrier arrivals, [1]: abort
};

// workspace (floats): d_fm, d_fs, d_ms, d_mf, d_sf, d_sm [B][C] each; f [B][F];
// m [B][M]; s [B][S]; partial sums [4][grid][B]
struct ScanWs {
  float *d_fm, *d_fs, *d_ms, *d_mf, *d_sf, *d_sm, *f, *m, *s, *part;
  __device__ ScanWs(const ScanParams& p) {
    const int B = p.B, C = p.C;
    d_fm = p.ws;
    d_fs = d_fm + B * C;
    d_ms = d_fs + B * C;
    d_mf = d_ms + B * C;
    d_sf = d_mf + B * C;
    d_sm = d_sf + B * C;
    f = d_sm + B * C;
    m = f + B * p.F;
    s = m + B * p.M;
    part = s + B * p.S;
  }
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }

__device__ __forceinline__ void red_add_release_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier number `k` (0-based) of this launch: every CTA has arrived
// k + 1 times.  The arrival is a release add (it orders the CTA's stage
// outputs, made CTA-visible by the bar.sync before it, ahead of itself); the
// wait is acquire loads of the count, with the abort word checked every 64
// polls.  False when the wait gave up (or another CTA's did).
__device__ bool grid_barrier(unsigned* bar, unsigned k, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    red_add_release_u32(&bar[0], 1u);
    const unsigned target = (k + 1u) * gridDim.x;
    int ok = 1;
    if (ld_acquire_u32(&bar[0]) < target) {
      const long long t0 = clock64();
      unsigned polls = 0;
      while (ld_acquire_u32(&bar[0]) < target) {
        if ((++polls & 63u) == 0u &&
            (ld_acquire_u32(&bar[1]) != 0u || clock64() - t0 > kScanWaitCycles)) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) {
      atomicExch(&bar[1], 1u);
      atomicExch(&g_scan_error, (unsigned)GFST_ERR_TIMEOUT);
    }
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// Stage the rows [b][0, n) of src (row stride ld floats, other CTAs' writes:
// read past L1) into xs[b][off, off + n) (row stride xld).
// n, ld, off and xld are multiples of 4: float4 moves.
__device__ __forceinline__ void stage_in(float* xs, int xld, int off, const float* src, int ld, int n, int B) {
  const int n4 = n >> 2;
  for (int e = threadIdx.x; e < B * n4; e += kScanThreads) {
    const int b = e / n4, i = e - b * n4;
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (size_t)b * ld) + i);
    *reinterpret_cast<float4*>(xs + b * xld + off + 4 * i) = v;
  }
}

// acc[b] += W_row . xs[b][off, off + K) for b < B; K % 4 == 0; lanes split k.
__device__ __forceinline__ void warp_dot(const float* __restrict__ wrow, const float* xs, int xld, int off, int K,
                                         int B, float (&acc)[kScanBatch], int lane) {
  const float4* w4 = reinterpret_cast<const float4*>(wrow);
  for (int k4 = lane; k4 < K / 4; k4 += 32) {
    const float4 w = __ldg(w4 + k4);
#pragma unroll
    for (int b = 0; b < kScanBatch; ++b) {
      if (b < B) {
        const float4 x = *reinterpret_cast<const float4*>(xs + b * xld + off + 4 * k4);
        acc[b] = fmaf(w.x, x.x, acc[b]);
        acc[b] = fmaf(w.y, x.y, acc[b]);
        acc[b] = fmaf(w.z, x.z, acc[b]);
        acc[b] = fmaf(w.w, x.w, acc[b]);
      }
    }
  }
}

__device__ __forceinline__ void warp_allreduce(float (&acc)[kScanBatch], int B) {
#pragma unroll
  for (int b = 0; b < kScanBatch; ++b) {
    if (b < B) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
    }
  }
}

__device__ __forceinline__ void zero(float (&acc)[kScanBatch]) {
#pragma unroll
  for (int b = 0; b < kScanBatch; ++b) acc[b] = 0.f;
}

// Per-CTA sums of per-warp partials (warp order) into part[kind][blockIdx.x][b].
__device__ __forceinline__ void cta_partial(float* wsum, const float (&mine)[kScanBatch], float* part, int kind,
                                            int B, int warp, int lane) {
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < kScanBatch; ++b)
      if (b < B) wsum[warp * kScanBatch + b] = mine[b];
  }
  __syncthreads();
  if (threadIdx.x < B) {
    float s = 0.f;
    for (int w = 0; w < kScanWarps; ++w) s += wsum[w * kScanBatch + threadIdx.x];
    part[((size_t)kind * gridDim.x + blockIdx.x) * B + threadIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kScanThreads, 1) mpuc_scan_kernel(ScanParams p) {
  extern __shared__ __align__(16) float scan_smem[];
  __shared__ float wsum[4 * kScanBatch * 8];  // per-warp partials; then the stage-I sums
  __shared__ float gate_scale[kScanBatch];
  __shared__ int bar_ok;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * kScanWarps + warp, GW = gridDim.x * kScanWarps;
  const int F = p.F, M = p.M, S = p.S, C = p.C, B = p.B, H = F + M + S;
  const gfst_mpuc_weights& w = p.w;
  ScanWs ws(p);
  float* xs = scan_smem;  // [B][xld]
  const int xld = max(max(F, M + S), 2 * C);
  unsigned nb = 0;        // barriers passed in this launch
  float acc[kScanBatch], acc2[kScanBatch], mine[kScanBatch];

  for (int t = 0; t < p.T; ++t) {
    // ---- A: d_fm, d_fs, d_ms from M, S ---------------------------------------
    stage_in(xs, xld, 0, p.st_mid, M, M, B);
    stage_in(xs, xld, M, p.st_slow, S, S, B);
    __syncthreads();
    for (int j = gw; j < 3 * C; j += GW) {
      const int which = j / C, r = j - which * C;
      const float* wr = which == 0 ? w.fm_down + (size_t)r * M : (which == 1 ? w.fs_down : w.ms_down) + (size_t)r * S;
      zero(acc);
      warp_dot(wr, xs, xld, which == 0 ? 0 : M, which == 0 ? M : S, B, acc, lane);
      warp_allreduce(acc, B);
      float* dst = which == 0 ? ws.d_fm : (which == 1 ? ws.d_fs : ws.d_ms);
      if (lane < B) {
        float v = 0.f;
#pragma unroll
        for (int b = 0; b < kScanBatch; ++b) v = (b == lane) ? acc[b] : v;
        dst[lane * C + r] = siluf_(v);
      }
    }
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- B: fast drive ---------------------------------------------------------
    stage_in(xs, xld, 0, ws.d_fm, C, C, B);
    stage_in(xs, xld, C, ws.d_fs, C, C, B);
    __syncthreads();
    for (int j = gw; j < F; j += GW) {
      zero(acc);
      warp_dot(w.fm_up + (size_t)j * C, xs, xld, 0, C, B, acc, lane);
      warp_dot(w.fs_up + (size_t)j * C, xs, xld, C, C, B, acc, lane);
      warp_allreduce(acc, B);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b)
        if (b < B && lane == b) ws.f[b * F + j] = __ldg(p.x_fast + ((size_t)b * p.T + t) * F + j) + acc[b];
    }
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- C: fast band -----------------------------------------------------------
    stage_in(xs, xld, 0, ws.f, F, F, B);
    __syncthreads();
    zero(mine);
    for (int j = gw; j < F; j += GW) {
      zero(acc);
      zero(acc2);
      warp_dot(w.fast_gate_w + (size_t)j * F, xs, xld, 0, F, B, acc, lane);
      warp_dot(w.fast_cand_w + (size_t)j * F, xs, xld, 0, F, B, acc2, lane);
      warp_allreduce(acc, B);
      warp_allreduce(acc2, B);
      const float bg = __ldg(w.fast_gate_b + j), bc = __ldg(w.fast_cand_b + j);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b) {
        if (b < B) {
          const float g = sigmoidf_(acc[b] + bg);
          const float c = tanhf(acc2[b] + bc);
          mine[b] += g;
          if (lane == b) {
            const float prev = __ldcg(p.st_fast + (size_t)b * F + j);
            const float nv = (1.f - g) * prev + g * c;
            p.st_fast[(size_t)b * F + j] = nv;
            p.states[((size_t)b * p.T + t) * H + j] = nv;
          }
        }
      }
    }
    cta_partial(wsum, mine, ws.part, 0, B, warp, lane);
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- D: d_mf, d_sf from the new F --------------------------------------------
    stage_in(xs, xld, 0, p.st_fast, F, F, B);
    __syncthreads();
    for (int j = gw; j < 2 * C; j += GW) {
      const int which = j / C, r = j - which * C;
      zero(acc);
      warp_dot((which == 0 ? w.mf_down : w.sf_down) + (size_t)r * F, xs, xld, 0, F, B, acc, lane);
      warp_allreduce(acc, B);
      float* dst = which == 0 ? ws.d_mf : ws.d_sf;
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b)
        if (b < B && lane == b) dst[b * C + r] = siluf_(acc[b]);
    }
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- E: mid drive, with the squared change against the previous M -------------
    stage_in(xs, xld, 0, ws.d_mf, C, C, B);
    stage_in(xs, xld, C, ws.d_ms, C, C, B);
    __syncthreads();
    zero(mine);
    for (int j = gw; j < M; j += GW) {
      zero(acc);
      warp_dot(w.mf_up + (size_t)j * C, xs, xld, 0, C, B, acc, lane);
      warp_dot(w.ms_up + (size_t)j * C, xs, xld, C, C, B, acc, lane);
      warp_allreduce(acc, B);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b) {
        if (b < B) {
          const float v = __ldg(p.x_mid + ((size_t)b * p.T + t) * M + j) + acc[b];
          const float dlt = v - __ldcg(p.st_mid + (size_t)b * M + j);
          mine[b] += dlt * dlt;
          if (lane == b) ws.m[b * M + j] = v;
        }
      }
    }
    cta_partial(wsum, mine, ws.part, 2, B, warp, lane);
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- F: mid band --------------------------------------------------------------
    stage_in(xs, xld, 0, ws.m, M, M, B);
    __syncthreads();
    zero(mine);
    for (int j = gw; j < M; j += GW) {
      zero(acc);
      zero(acc2);
      warp_dot(w.mid_gate_w + (size_t)j * M, xs, xld, 0, M, B, acc, lane);
      warp_dot(w.mid_cand_w + (size_t)j * M, xs, xld, 0, M, B, acc2, lane);
      warp_allreduce(acc, B);
      warp_allreduce(acc2, B);
      const float bg = __ldg(w.mid_gate_b + j), bc = __ldg(w.mid_cand_b + j);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b) {
        if (b < B) {
          const float g = sigmoidf_(acc[b] + bg);
          const float c = tanhf(acc2[b] + bc);
          mine[b] += g;
          if (lane == b) {
            const float prev = __ldcg(p.st_mid + (size_t)b * M + j);
            const float nv = (1.f - g) * prev + g * c;
            p.st_mid[(size_t)b * M + j] = nv;
            p.states[((size_t)b * p.T + t) * H + F + j] = nv;
          }
        }
      }
    }
    cta_partial(wsum, mine, ws.part, 1, B, warp, lane);
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- G: d_sm from the new M -----------------------------------------------------
    stage_in(xs, xld, 0, p.st_mid, M, M, B);
    __syncthreads();
    for (int j = gw; j < C; j += GW) {
      zero(acc);
      warp_dot(w.sm_down + (size_t)j * M, xs, xld, 0, M, B, acc, lane);
      warp_allreduce(acc, B);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b)
        if (b < B && lane == b) ws.d_sm[b * C + j] = siluf_(acc[b]);
    }
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- H: slow drive, with the squared change against the previous S ----------------
    stage_in(xs, xld, 0, ws.d_sf, C, C, B);
    stage_in(xs, xld, C, ws.d_sm, C, C, B);
    __syncthreads();
    zero(mine);
    for (int j = gw; j < S; j += GW) {
      zero(acc);
      warp_dot(w.sf_up + (size_t)j * C, xs, xld, 0, C, B, acc, lane);
      warp_dot(w.sm_up + (size_t)j * C, xs, xld, C, C, B, acc, lane);
      warp_allreduce(acc, B);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b) {
        if (b < B) {
          const float v = __ldg(p.x_slow + ((size_t)b * p.T + t) * S + j) + acc[b];
          const float dlt = v - __ldcg(p.st_slow + (size_t)b * S + j);
          mine[b] += dlt * dlt;
          if (lane == b) ws.s[b * S + j] = v;
        }
      }
    }
    cta_partial(wsum, mine, ws.part, 3, B, warp, lane);
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;

    // ---- I: boundary logit, then the slow band ----------------------------------------
    // per (kind, b): eight threads sum the CTAs' partials c = sub, sub + 8, ...
    // in order, then one thread adds the eight in order (fixed association)
    {
      const int pair = threadIdx.x >> 3, sub = threadIdx.x & 7;
      if (pair < 4 * B) {
        const int kind = pair / B, b = pair - kind * B;
        float s = 0.f;
        for (int c = sub; c < (int)gridDim.x; c += 8) s += __ldcg(ws.part + ((size_t)kind * gridDim.x + c) * B + b);
        wsum[threadIdx.x] = s;
      }
    }
    __syncthreads();
    if (threadIdx.x < B) {
      const int b = threadIdx.x;
      float sums[4];
      for (int kind = 0; kind < 4; ++kind) {
        float s = 0.f;
        for (int sub = 0; sub < 8; ++sub) s += wsum[(kind * B + b) * 8 + sub];
        sums[kind] = s;
      }
      const float feat[4] = {sums[0] / (float)F, sums[1] / (float)M, sqrtf(sums[2] / (float)M + 1e-6f),
                             sqrtf(sums[3] / (float)S + 1e-6f)};
      float logit = __ldg(w.bnd_b2);
      for (int h = 0; h < p.BH; ++h) {
        float z = __ldg(w.bnd_b1 + h);
        for (int q = 0; q < 4; ++q) z = fmaf(__ldg(w.bnd_w1 + h * 4 + q), feat[q], z);
        logit = fmaf(__ldg(w.bnd_w2 + h), siluf_(z), logit);
      }
      gate_scale[b] = sigmoidf_(logit);
      if (blockIdx.x == 0) p.logits[(size_t)b * p.T + t] = logit;
    }
    stage_in(xs, xld, 0, ws.s, S, S, B);
    __syncthreads();
    for (int j = gw; j < S; j += GW) {
      zero(acc);
      zero(acc2);
      warp_dot(w.slow_gate_w + (size_t)j * S, xs, xld, 0, S, B, acc, lane);
      warp_dot(w.slow_cand_w + (size_t)j * S, xs, xld, 0, S, B, acc2, lane);
      warp_allreduce(acc, B);
      warp_allreduce(acc2, B);
      const float bg = __ldg(w.slow_gate_b + j), bc = __ldg(w.slow_cand_b + j);
#pragma unroll
      for (int b = 0; b < kScanBatch; ++b) {
        if (b < B && lane == b) {
          const float g = sigmoidf_(acc[b] + bg) * gate_scale[b];
          const float c = tanhf(acc2[b] + bc);
          const float prev = __ldcg(p.st_slow + (size_t)b * S + j);
          const float nv = (1.f - g) * prev + g * c;
          p.st_slow[(size_t)b * S + j] = nv;
          p.states[((size_t)b * p.T + t) * H + F + M + j] = nv;
        }
      }
    }
    if (!grid_barrier(p.bar, nb++, &bar_ok)) return;
  }
}

size_t workspace_floats(int64_t B, int F, int M, int S, int C, int grid) {
  return (size_t)B * (6 * (size_t)C + F + M + S) + 4 * (size_t)grid * B;
}

// One CTA per SM of the current device.
int scan_grid(int* grid_out) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "device attributes: %s", cudaGetErrorString(e));
  *grid_out = sms;
  return GFST_OK;
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_mpuc_scan_workspace_bytes(int64_t batch, int fast_dim, int mid_dim, int slow_dim, int cross_rank,
                                              size_t* bytes) {
  using namespace gfst;
  GFST_REQUIRE(bytes != nullptr, GFST_ERR_ARG, "bytes must be non-null");
  GFST_REQUIRE(batch >= 0 && fast_dim > 0 && mid_dim > 0 && slow_dim > 0 && cross_rank > 0, GFST_ERR_ARG,
               "bad sizes");
  int grid = 0;
  const int st = scan_grid(&grid);
  if (st != GFST_OK) return st;
  const int64_t chunk = std::min<int64_t>(batch, kScanBatch);
  // two words of barrier state in front, then the floats (16-byte aligned)
  *bytes = 16 + workspace_floats(chunk, fast_dim, mid_dim, slow_dim, cross_rank, grid) * sizeof(float);
  return GFST_OK;
}

extern "C" int gfst_mpuc_recurrent_scan(const gfst_mpuc_weights* w, int fast_dim, int mid_dim, int slow_dim,
                                        int cross_rank, int boundary_hidden, const float* fast_in,
                                        const float* mid_in, const float* slow_in, int64_t batch, int T,
                                        float* states_out, float* boundary_out, float* fast_state,
                                        float* mid_state, float* slow_state, void* workspace,
                                        size_t workspace_bytes, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(w != nullptr, GFST_ERR_ARG, "weights must be non-null");
  const int F = fast_dim, M = mid_dim, S = slow_dim, C = cross_rank;
  GFST_REQUIRE(F > 0 && M > 0 && S > 0 && C > 0 && boundary_hidden > 0, GFST_ERR_ARG, "bad sizes");
  GFST_REQUIRE(F % 4 == 0 && M % 4 == 0 && S % 4 == 0 && C % 4 == 0, GFST_ERR_SHAPE,
               "fast, mid, slow widths and the bridge rank must be multiples of 4 (%d %d %d %d)", F, M, S, C);
  GFST_REQUIRE(std::max(std::max(F, M + S), 2 * C) <= 6144, GFST_ERR_SHAPE,
               "stage inputs of %d floats per batch element exceed the shared-memory stage",
               std::max(std::max(F, M + S), 2 * C));
  GFST_REQUIRE(batch >= 0 && T >= 0 && T <= (1 << 20), GFST_ERR_ARG, "batch >= 0 and 0 <= T <= 2^20");
  if (batch == 0 || T == 0) return GFST_OK;
  const float* ptrs[] = {w->fast_gate_w, w->fast_gate_b, w->fast_cand_w, w->fast_cand_b, w->mid_gate_w,
                         w->mid_gate_b,  w->mid_cand_w,  w->mid_cand_b,  w->slow_gate_w, w->slow_gate_b,
                         w->slow_cand_w, w->slow_cand_b, w->fm_down,     w->fm_up,       w->fs_down,
                         w->fs_up,       w->mf_down,     w->mf_up,       w->ms_down,     w->ms_up,
                         w->sf_down,     w->sf_up,       w->sm_down,     w->sm_up,       w->bnd_w1,
                         w->bnd_b1,      w->bnd_w2,      w->bnd_b2};
  for (const float* q : ptrs) GFST_REQUIRE(q != nullptr, GFST_ERR_ARG, "every weight pointer must be non-null");
  const float* mats[] = {w->fast_gate_w, w->fast_cand_w, w->mid_gate_w, w->mid_cand_w, w->slow_gate_w,
                         w->slow_cand_w, w->fm_down,     w->fm_up,      w->fs_down,    w->fs_up,
                         w->mf_down,     w->mf_up,       w->ms_down,    w->ms_up,      w->sf_down,
                         w->sf_up,       w->sm_down,     w->sm_up};
  for (const float* q : mats) GFST_REQUIRE(aligned16(q), GFST_ERR_ALIGN, "weight matrices must be 16-byte aligned");
  GFST_REQUIRE(fast_in && mid_in && slow_in && states_out && boundary_out && fast_state && mid_state && slow_state,
               GFST_ERR_ARG, "inputs, outputs and states must be non-null");
  int grid = 0;
  int st = scan_grid(&grid);
  if (st != GFST_OK) return st;
  const int64_t chunk = std::min<int64_t>(batch, kScanBatch);
  const size_t need = 16 + workspace_floats(chunk, F, M, S, C, grid) * sizeof(float);
  GFST_REQUIRE(workspace != nullptr && workspace_bytes >= need, GFST_ERR_ARG,
               "workspace of %zu bytes needed (gfst_mpuc_scan_workspace_bytes), %zu given", need, workspace_bytes);
  GFST_REQUIRE(aligned16(workspace), GFST_ERR_ALIGN, "workspace must be 16-byte aligned");
  const int xld = std::max(std::max(F, M + S), 2 * C);
  const size_t smem = (size_t)kScanBatch * xld * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(mpuc_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mpuc_scan_kernel, kScanThreads, smem);
  GFST_REQUIRE(e == cudaSuccess && per_sm >= 1, GFST_ERR_DEVICE, "the scan kernel does not fit on an SM");
  const int H = F + M + S;
  for (int64_t b0 = 0; b0 < batch; b0 += kScanBatch) {
    ScanParams p;
    p.w = *w;
    p.F = F;
    p.M = M;
    p.S = S;
    p.C = C;
    p.BH = boundary_hidden;
    p.B = (int)std::min<int64_t>(kScanBatch, batch - b0);
    p.T = T;
    p.x_fast = fast_in + b0 * T * (int64_t)F;
    p.x_mid = mid_in + b0 * T * (int64_t)M;
    p.x_slow = slow_in + b0 * T * (int64_t)S;
    p.states = states_out + b0 * T * (int64_t)H;
    p.logits = boundary_out + b0 * T;
    p.st_fast = fast_state + b0 * F;
    p.st_mid = mid_state + b0 * M;
    p.st_slow = slow_state + b0 * S;
    p.bar = static_cast<unsigned*>(workspace);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + 16);
    e = cudaMemsetAsync(workspace, 0, 16, stream);  // barrier count and abort word
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_DEVICE, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    void* args[] = {&p};
    e = cudaLaunchCooperativeKernel((const void*)mpuc_scan_kernel, dim3(grid), dim3(kScanThreads), args, smem,
                                    stream);
    GFST_REQUIRE(e == cudaSuccess, GFST_ERR_LAUNCH, "cooperative launch of mpuc_scan_kernel: %s",
                 cudaGetErrorString(e));
  }
  return GFST_OK;
}
