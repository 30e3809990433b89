/*
 * gfst_b200.h -- C ABI of the B200 (sm_100a) GFST-HMB streaming hot path.
 *
 * Every entry point takes raw device pointers, plain sizes and a cudaStream_t,
 * returns an int status (GFST_OK == 0), allocates nothing unless stated, and
 * never synchronises the host.  Work is enqueued on `stream`; results are
 * valid once that stream has reached the enqueued work.  Callers own every
 * buffer.  Layouts are dense row-major (C order) unless stated.
 *
 * The entry points replace these reference interfaces (paths are relative to
 * the reference project pkhairkh/gfst-hmb-public):
 *   gfst_frame_update_qr   <- gfst_local_qr_sm120_forward(candidate[B,m,n], eps_sign)
 *                             src/gfst_hmb_mpuc/csrc/mathdx/mathdx_extension.cpp:20-22,
 *                             src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:665-671, and the
 *                             torch path gfst.canonical_qr_batched / update_basis_candidate_batched
 *                             src/gfst_hmb_mpuc/gfst.py:26-46, 115-140
 *   gfst_frame_stream      <- the per-token loop GfstHmbSublayer._update_local_bases
 *                             src/gfst_hmb_mpuc/modeling.py:2299-2423 (largest level), with the
 *                             frame kept on chip across tokens
 *   gfst_local_tracker_stream <- GfstHmbSublayer._update_local_bases (all flag levels, rule
 *                             residual_rank_one_v1) + _local_alignment_features, per token
 *                             src/gfst_hmb_mpuc/modeling.py:2284-2437, gfst.py:91-112
 *   gfst_block_commit_mean <- GfstDecodeState.append_exact_token block commit
 *                             src/gfst_hmb_mpuc/state.py:651-815 and the block summary of
 *                             GfstHmbSublayer._update_block_memory modeling.py:3482-3535
 *                             (summary key = mean of the block's token keys)
 *   gfst_block_tracker_stream <- the per-token block tracker of GfstHmbSublayer._update_block_memory
 *                             modeling.py:3460-3479 (rule update + QR, projector_sum += U U^T,
 *                             reduced_sum += x)
 *   gfst_block_commit_eig  <- runtime_backends.gfst_block_commit(projector_sum, reduced_sum,
 *                             token_count, max_flag_dim, flag_dims) and its torch path
 *                             top_eig_summary, modeling.py:3482-3507, gfst.py:172-430,
 *                             diagnostics/block_commit_replay.py:97-181
 *   gfst_global_features   <- GfstHmbSublayer._resolve_single_global_request (torch branch)
 *                             modeling.py:2996-3108: global sketch, top_eig_summary,
 *                             alignment_components (gfst.py:389-430, 580-588)
 *   gfst_exact_readout_collapse <- the readout with perf.collapse_logsumexp_scores_and_occurrence
 *                             (src/gfst_hmb_mpuc/perf.py:164-229) and the select of
 *                             modeling.py:1151-1169 (duplicate token ids collapsed)
 *   gfst_block_topk        <- FaissGpuRetriever.search / exact_topk
 *                             src/gfst_hmb_mpuc/retrieval.py:136-172
 *   gfst_exact_topk        <- FaissGpuRetriever.exact_topk (one query, any k)
 *                             src/gfst_hmb_mpuc/retrieval.py:165-172
 *   gfst_exact_readout     <- ExactRecallReadout._score_block_tokens + top-1 select
 *                             src/gfst_hmb_mpuc/modeling.py:599-657, 1151-1169
 *   gfst_open_block_readout <- the current (open) block appended to the retrieved blocks
 *                             with its prefix length, modeling.py:2948-2963 (token appended
 *                             first, modeling.py:3807 / state.py:651-815, retrieval at :3853)
 *   gfst_segmented_max     <- runtime_backends segmented_max_by_group(scores, inverse, group_count)
 *                             src/gfst_hmb_mpuc/csrc/sm120_stub.cu:16-40, 150-172, called by
 *                             perf.collapse_max_scores_by_group perf.py:136-161
 *   gfst_segmented_logsumexp_occurrence <- runtime_backends segmented_logsumexp_occurrence(
 *                             scores, inverse, occurrence_blocks, occurrence_positions, group_count)
 *                             src/gfst_hmb_mpuc/csrc/sm120_stub.cu:42-111, 174-208, called by
 *                             perf.collapse_logsumexp_scores_and_occurrence perf.py:164-229
 *   gfst_exact_block_materialize <- runtime_backends exact_block_materialize(packed, start, end)
 *                             src/gfst_hmb_mpuc/csrc/sm120_stub.cu:225-245, called at
 *                             state.py:568 (_materialize_exact_block)
 *   gfst_heev              <- runtime_backends gfst_heev(matrices) / native gfst_heev_sm120_forward
 *                             src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:113-170, 620-650, 750-780
 *                             (batched symmetric eigendecomposition, called at modeling.py:3181)
 *   gfst_exact_block_score <- runtime_backends exact_block_score(query, token_features, W), the
 *                             projection exact_block_project_forward
 *                             src/gfst_hmb_mpuc/csrc/sm120_cutlass_exact_block_score.cu:42-129
 *                             and its dot with the query, modeling.py:640-651
 */
#ifndef GFST_B200_H_
#define GFST_B200_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define GFST_API __attribute__((visibility("default")))
#else
#define GFST_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
enum gfst_status {
  GFST_OK = 0,
  GFST_ERR_ARG = 1,         /* null pointer or negative size                          */
  GFST_ERR_SHAPE = 2,       /* shape outside what the kernels support                 */
  GFST_ERR_ALIGN = 3,       /* pointer or row pitch not aligned as required           */
  GFST_ERR_LAUNCH = 4,      /* the CUDA launch itself failed (cudaGetLastError)       */
  GFST_ERR_DEVICE = 5,      /* device is not sm_100 or a CUDA runtime call failed     */
  GFST_ERR_TIMEOUT = 6,     /* a bounded device-side wait gave up                     */
  GFST_ERR_DTYPE = 7,       /* unsupported element type                               */
  GFST_ERR_NUMERIC = 8      /* a device-side numerical routine did not converge      */
};

/* Sign convention applied to every column of a thin-QR factor Q. */
enum gfst_sign_mode {
  /* Reference rule (gfst.py:35-46): find the first row whose |q| > eps_sign;
   * if that entry is negative, negate the column.  Columns with no such entry
   * are left as they are. */
  GFST_SIGN_FIRST_SIGNIFICANT = 0,
  /* Q * sign(diag(R)) with sign(0) = +1: every R_jj >= 0. */
  GFST_SIGN_R_DIAG_POSITIVE = 1
};

/* QR algorithm of the streaming frame pass (gfst_frame_stream_ex). */
enum gfst_qr_method {
  /* CholeskyQR2 for 32 < d <= 128 with 8 < r <= 32 (split over warps while
   * every split CTA is resident: up to 2 frames per SM for d = 128, 4 for
   * d <= 64) and for 8 < d <= 128 with r <= 8, Householder otherwise. */
  GFST_QR_AUTO = 0,
  /* LAPACK-order Householder (geqrf/orgqr) for every token. */
  GFST_QR_HOUSEHOLDER = 1,
  /* Two Cholesky QR passes per token (G = C^T C = R^T R, C <- C R^{-1});
   * a frame whose pivot R_jj^2 falls below 1e-2 * G_jj (or is not finite)
   * takes the Householder path for that token.  Same Q as Householder with
   * R_jj > 0 to fp32 rounding; shapes outside the AUTO range are rejected.
   * With r <= 8 a frame is split over 8 or 16 lanes and a failed pivot test
   * sends the frames of the whole warp (2 or 4) through Householder. */
  GFST_QR_CHOLESKY2 = 2,
  /* GFST_QR_CHOLESKY2 with each frame split over d/32 warps (a CTA per frame):
   * shorter per-token latency for batches too small to fill the GPU with one
   * frame per warp.  AUTO takes it up to 2 frames per SM (d = 128) or 4
   * (d <= 64): 296 or 592 frames on B200. */
  GFST_QR_CHOLESKY2_SPLIT = 3
};

/* Element types of key / value / query / summary buffers. */
enum gfst_dtype { GFST_F32 = 0, GFST_BF16 = 1, GFST_F64 = 2 };

/* Human-readable text of a status code (static storage). */
GFST_API const char* gfst_status_string(int status);
/* ABI version of this library, (major << 16) | minor. */
GFST_API int gfst_abi_version(void);
/* Detail text of the last non-OK status returned on the calling host thread
 * (empty string if none). */
GFST_API const char* gfst_last_error(void);

/* ---- frames: rank-m update + thin QR ----------------------------------- *
 * For every frame f in [0, n_frames):
 *     C   = beta * U[f] + A[f] * B[f]^T        (U: d x r, A: d x m, B: r x m)
 *     Q   = thin Q of Householder QR(C) (LAPACK geqrf/orgqr order), sign-fixed
 *     Uout[f] = Q                               (d x r)
 * Frames of 8 < d <= 128 rows and r <= 8 columns take CholeskyQR2 (the same
 * Q to fp32 rounding; Householder for a warp whose frames fail the pivot
 * test of GFST_QR_CHOLESKY2).
 * m == 0 is a plain batched QR of U (A and B may be NULL).  U and Uout may alias.
 * Limits: 1 <= r <= d, r <= 32, d <= 128 (d <= 256 when r <= 16), 0 <= m <= 8.
 * fp32 throughout; no fast-math.                                            */
GFST_API int gfst_frame_update_qr(const float* U, const float* A, const float* B, float beta,
                         float* Uout, int64_t n_frames, int d, int r, int m,
                         float eps_sign, int sign_mode, cudaStream_t stream);

/* ---- frames: T-token streaming pass, frame resident on chip ---------------
 * For t in [0, T):  U[f] <- QR_signfixed(beta * U[f] + A[f,t] * B[f,t]^T)
 * U: [n_frames, d, r] (in/out), A: [n_frames, T, d, m], B: [n_frames, T, r, m].
 * If frames_out != NULL and out_every > 0, the frame after token t is written
 * to frames_out[(t+1)/out_every - 1] (layout [T/out_every, n_frames, d, r])
 * whenever (t+1) % out_every == 0.  Same shape limits as gfst_frame_update_qr;
 * m >= 1; A and B rows need 16-byte alignment (d*m and r*m multiples of 4).  */
GFST_API int gfst_frame_stream(float* U, const float* A, const float* B, float beta,
                      int64_t n_frames, int T, int d, int r, int m,
                      float eps_sign, int sign_mode,
                      float* frames_out, int out_every, cudaStream_t stream);

/* gfst_frame_stream with the QR algorithm chosen explicitly (gfst_qr_method);
 * gfst_frame_stream is this call with GFST_QR_AUTO.  No reference
 * counterpart: the reference factorises every token with torch.linalg.qr. */
GFST_API int gfst_frame_stream_ex(float* U, const float* A, const float* B, float beta,
                         int64_t n_frames, int T, int d, int r, int m,
                         float eps_sign, int sign_mode,
                         float* frames_out, int out_every, int qr_method, cudaStream_t stream);

/* ---- local tracker: all flag levels + alignment features, T tokens --------
 * Per stream s and token t (x = x[s,t], a d-vector), with the reference rule
 * residual_rank_one_v1 (gfst.py:91-112) on a basis B and a vector v at rate a:
 *     w = B^T v,  s = (v - B w) / sqrt(||v||^2 + eps_update^2),
 *     B <- QR_signfixed((1 - a) B + a v w^T + a s e_last^T)
 *   U <- rule(U, x, rates[n_levels]);  p = U^T x;
 *   V_l <- rule(V_l, p, rates[l]) for l < n_levels (thin Q keeps dims[l] columns);
 *   features[s,t] = (c_0, c_0, c_1, c_1 - c_0, ..., c_L, c_L - c_{L-1}) with
 *     c_l = ||V_l^T p||^2 / max(||x||^2, eps) (l < L), c_L = ||p||^2 / max(||x||^2, eps).
 * U: [n_streams, d, r] (in/out, r = the largest flag dim); nested:
 * [n_streams, n_levels, r, r] (in/out; level l occupies columns [0, dims[l]),
 * other columns are ignored on input and zero on output); x: [n_streams, T, d]
 * (16-byte aligned, d % 4 == 0); dims: host array of n_levels strictly
 * increasing sizes in [1, r); rates: host array of n_levels + 1 forgetting
 * rates (nested levels, then U); features: [n_streams, T, 2 (n_levels + 1)] or
 * NULL.  Limits: r <= 32, d as gfst_frame_update_qr, n_levels <= 4.  fp32.   */
GFST_API int gfst_local_tracker_stream(float* U, float* nested, const float* x, int64_t n_streams,
                              int T, int d, int r, int n_levels, const int32_t* dims,
                              const double* rates, double eps, double eps_update,
                              float eps_sign, int sign_mode, float* features,
                              cudaStream_t stream);

/* ---- block tracker: per-token accumulation of a block's commit inputs -----
 * Per stream s and token t (x = x[s,t]): U <- QR_signfixed((1 - rate) U +
 * rate x w^T + rate s e_last^T) with the rule of gfst_local_tracker_stream;
 * projector_sum[s] += U U^T (d x d); reduced_sum[s] += x.  Inputs are updated
 * in place, so a block can be fed in several calls; a new block starts from
 * U = eye(d, r) and zero sums.  Replaces the per-token part of
 * GfstHmbSublayer._update_block_memory (modeling.py:3460-3479) of the reference.
 * Limits: d <= 64, d % 4 == 0, r % 4 == 0, r <= 32; x 16-byte aligned.      */
GFST_API int gfst_block_tracker_stream(float* U, float* projector_sum, float* reduced_sum,
                              const float* x, int64_t n_streams, int T, int d, int r,
                              double rate, double eps_update, float eps_sign, int sign_mode,
                              cudaStream_t stream);

/* ---- block commit ----------------------------------------------------------
 * For every stream s in [0, n_streams):
 *   pool_K[s, slot] = K[s]   (L x d),  pool_V[s, slot] = V[s]   (L x dv)
 *   summary[s, slot, :] = mean over the L rows of K[s]   (fp32 sum in token
 *                         order, divided by L, rounded once to `dtype`)
 * K: [n_streams, L, d], V: [n_streams, L, dv]; pool_K: [n_streams, n_slots, L, d];
 * pool_V: [n_streams, n_slots, L, dv]; summary: [n_streams, n_slots, d].
 * V / pool_V may be NULL (keys only).  dtype is GFST_F32 or GFST_BF16 for all
 * five buffers.  Rows need 16-byte alignment.                               */
GFST_API int gfst_block_commit_mean(const void* K, const void* V, void* pool_K, void* pool_V,
                           void* summary, int64_t n_streams, int n_slots, int slot,
                           int L, int d, int dv, int dtype, cudaStream_t stream);

/* ---- reference-faithful block commit: eigen summary of a closed block ------
 * For every stream s (fp32 in, fp32 out, float64 eigenproblem):
 *   average_projector[s] = projector_sum[s] / token_count        (d x d)
 *   reduced_mean[s]      = reduced_sum[s] / token_count          (d)
 *   eigenpairs of (average + average^T) / 2 in float64; eigenvalue clusters
 *   (|a - b| <= 1e-9 + 1e-7 |b|) taken from the top until T = max(max_flag_dim,
 *   max(flag_dims), 1) columns are filled, each replaced by its canonical basis
 *   (Gram-Schmidt over the cluster projector's columns in descending-diagonal
 *   order, signs by the first entry with |x| > eps_sign), cast to fp32, signs
 *   fixed again;
 *   summary_basis[s] = columns [0, max_flag_dim)  (d x max_flag_dim), top_vector[s] = column 0.
 * projector_sum: [n_streams, d, d]; reduced_sum: [n_streams, d]; flag_dims: host
 * array of n_flags sizes.  Limits: d <= 64, 1 <= max_flag_dim <= d.  An
 * eigensolver that does not converge, or a cluster basis short of its rank,
 * records GFST_ERR_NUMERIC for gfst_check_device_errors().                    */
GFST_API int gfst_block_commit_eig(const float* projector_sum, const float* reduced_sum,
                          int64_t n_streams, int d, int token_count, int max_flag_dim,
                          const int32_t* flag_dims, int n_flags, double eps_sign,
                          float* summary_basis, float* reduced_mean, float* top_vector,
                          float* average_projector, cudaStream_t stream);

/* ---- exact readout with the token-id log-sum-exp collapse ------------------
 * Candidates of query (s, q): the tokens of its selected blocks in selection
 * order (a block listed twice counts once; entries < 0 or >= n_slots skipped),
 * score = key . query (fp32 accumulate).  Grouped by token_ids[s, block, pos]
 * (ids < 0 and NaN scores take no part): group score = m + log(max(sum
 * exp(score - m), 1e-8)) with m the group max; the occurrence is the first
 * candidate (selection order, then position) scoring m.  Output the best group
 * (score descending, token id ascending): best_id, best_score, best_block,
 * best_pos [n_streams, n_queries] (-1 / -inf when nothing qualifies).
 * Q: [n_streams, n_queries, d]; pool_K: [n_streams, n_slots, L, d];
 * token_ids: [n_streams, n_slots, L] int32; top_idx: [n_streams, n_queries, k].
 * Limits: k * L <= 2048, d <= 256; dtype GFST_F32 or GFST_BF16.              */
GFST_API int gfst_exact_readout_collapse(const void* Q, const void* pool_K, const int32_t* token_ids,
                          const int32_t* top_idx, int64_t n_streams, int n_queries, int n_slots,
                          int L, int d, int k, int dtype, int32_t* best_id, float* best_score,
                          int32_t* best_block, int32_t* best_pos, cudaStream_t stream);

/* ---- global sketch features per query --------------------------------------
 * For every stream s and query q, over the selections j with 0 <= sel_idx[s,q,j]
 * < n_blocks: w = softmax(sel_scores[s,q,j] * temperature); sketch = sum_j w_j
 * projector_bank[s, sel_idx[s,q,j]] (d x d); B = the canonical top basis of the
 * sketch (as gfst_block_commit_eig, T = max(max_flag_dim, max(flag_dims)));
 * for each flag dim m: c_m = x^T B_m B_m^T x / (x . x + eps);
 * features[s,q] = (c_0, c_0, c_1, c_1 - c_0, ...) (2 n_flags floats; zeros when
 * no selection is valid).  Optional outputs: sketch_out [S, Nq, d, d],
 * basis_out [S, Nq, d, max_flag_dim].  projector_bank: [n_streams, n_blocks, d, d];
 * sel_idx, sel_scores: [n_streams, n_queries, k]; x: [n_streams, n_queries, d].
 * Limits: d <= 64, k <= 32, 1 <= n_flags <= 8.                              */
GFST_API int gfst_global_features(const float* projector_bank, const int32_t* sel_idx,
                          const float* sel_scores, const float* x, int64_t n_streams,
                          int n_queries, int n_blocks, int d, int k, float temperature,
                          int max_flag_dim, const int32_t* flag_dims, int n_flags, float eps,
                          double eps_sign, float* features, float* sketch_out, float* basis_out,
                          cudaStream_t stream);

/* ---- centroid path: cell write at block commit ---------------------------
 * GfstDecodeState._append_exact_token_cuda_packed (state.py:315-470) for the L
 * tokens of a block and _finalise_block_cells (state.py:501-551), for each of
 * n_blocks blocks.  Inputs [n_blocks, L, W] cell_ids (int32, clamped to
 * [0, C-1]) and cell_weights (float32); [n_blocks, L, dk] cell_keys and
 * [n_blocks, L, dv] cell_values (float32).  Outputs: token_cell_ids and
 * token_cell_weights_q [n_blocks, L, W] u8 (round(w * 255) clamped to
 * [0, 255], NaN -> 0); block_cell_keys [n_blocks, C, dk] fp16 (mean key of the
 * cell's tokens weighted by q/255, 0 for an empty cell), block_cell_values_q
 * [n_blocks, C, dv] int8 (round(mean value * 32) clamped to [-127, 127]),
 * block_cell_counts [n_blocks, C] int16 (round(weight sum * 32) clamped to
 * [0, 32767]).  Sums run in token then membership order in IEEE fp32, as the
 * reference's index_add_ does on the CPU.  Limits: L * W <= 1024, C <= 256. */
GFST_API int gfst_centroid_cell_commit(const int32_t* cell_ids, const float* cell_weights,
                              const float* cell_keys, const float* cell_values,
                              int64_t n_blocks, int L, int W, int C, int dk, int dv,
                              uint8_t* token_cell_ids, uint8_t* token_cell_weights_q,
                              void* block_cell_keys, int8_t* block_cell_values_q,
                              int16_t* block_cell_counts, cudaStream_t stream);

/* Parameters of the centroid readout: the ExactRecallReadout attributes of the
 * same names (modeling.py:371-448, config defaults in brackets). */
typedef struct gfst_centroid_params {
  float block_score_lambda;  /* centroid_block_score_lambda [0.10]             */
  int background_subtract;   /* centroid_background_subtract [1]               */
  float count_penalty;       /* centroid_count_penalty [0.5]                   */
  float self_field_weight;   /* centroid_self_field_weight [0.15]              */
  int top_cells_per_head;    /* centroid_top_cells_per_head [8], <= 16         */
  float fdr_q;               /* centroid_fdr_q [0.10]                          */
  int min_selected;          /* centroid_min_selected_cells_per_head [2]       */
  float temperature;         /* centroid_selection_temperature [1.0], > 0      */
  float entropy_low;         /* centroid_gain_entropy_low [0.35]               */
  float entropy_high;        /* centroid_gain_entropy_high [0.75]              */
  float gamma_m;             /* centroid_gamma_m [1.0]                         */
  float gamma_r;             /* centroid_gamma_r [1.0]                         */
} gfst_centroid_params;

/* ---- centroid path: significance-gated readout ---------------------------
 * ExactRecallReadout._build_centroid_candidates (modeling.py:659-982) for every
 * (stream, query), then the log-sum-exp collapse by token id and the best
 * group (perf.py:164-229, modeling.py:1151-1169).  Per query: the valid
 * selections (0 <= sel_idx < n_slots, prefix > 0) in order are the block
 * entries; their cells with count > 0 are scored per centroid head
 * (query_heads . key / sqrt(dk) + lambda * block score), robust-z-scored,
 * selected by BH-FDR (minimum-count fallback), weighted by softmax; every
 * token of an entry (positions < prefix) gets
 *   base + gamma_m * conf * token_mass + gamma_r * conf * recall
 * with base = token_keys . Q.  With no candidate cell or no selection the
 * centroid terms are off (base only, confidence -1), as the reference falls
 * back to _score_block_tokens.
 * Q [S, Nq, dq]; query_heads [S, Nq, H, dk] (centroid_query_proj(query));
 * sel_idx int32 / sel_scores float32 / prefix_len int32 (or NULL: full blocks)
 * [S, Nq, K]; token_keys [S, n_slots, L, dq] (within_block_proj of the stored
 * tokens); token_features [S, n_slots, L, H, dv] (centroid_token_proj of the
 * stored tokens); token_ids [S, n_slots, L]; token_cell_ids /
 * token_cell_weights_q [S, n_slots, L, W] u8 and cell_keys (fp16) /
 * cell_values_q / cell_counts [S, n_slots, C, ...] as gfst_centroid_cell_commit
 * writes them.  Outputs: best_id / best_score / best_block (slot) / best_pos
 * [S, Nq] (-1 / -inf when nothing is valid); optional (NULL to skip):
 * cand_scores [S, Nq, K, L] (final token scores, -inf where no token),
 * sel_block (entry index) / sel_cell / sel_alpha [S, Nq, H, top_cells_per_head],
 * head_stats [S, Nq, H, 3] (entropy, margin, selected count), confidence
 * [S, Nq].  Limits: K <= 32, C <= 32, K * C <= 512, K * L <= 2048, H <= 8,
 * dk <= 64, dv <= 32, dq <= 256, W <= 8.  fp32 throughout.                 */
GFST_API int gfst_centroid_readout(const float* Q, const float* query_heads, const int32_t* sel_idx,
                          const float* sel_scores, const int32_t* prefix_len,
                          const float* token_keys, const float* token_features,
                          const int32_t* token_ids, const uint8_t* token_cell_ids,
                          const uint8_t* token_cell_weights_q, const void* cell_keys,
                          const int8_t* cell_values_q, const int16_t* cell_counts,
                          int64_t n_streams, int n_queries, int n_slots, int L, int dq, int H,
                          int dk, int dv, int C, int W, int K, const gfst_centroid_params* params,
                          float* cand_scores, int32_t* best_id, float* best_score,
                          int32_t* best_block, int32_t* best_pos, int32_t* sel_block,
                          int32_t* sel_cell, float* sel_alpha, float* head_stats,
                          float* confidence, cudaStream_t stream);

/* ---- coarse block retrieval: score + top-k ---------------------------------
 * For every stream s and query q:
 *   score[b] = Q[s,q,:] . Ksum[s,b,:]   for b in [0, n_blocks)   (fp32 accumulate)
 *   top_idx[s,q,0..k) / top_scores[s,q,0..k) = the k best blocks in the total
 *   order (score descending, block index ascending).  Blocks scoring NaN or
 *   -inf are never selected; unfilled slots hold index -1 and score -inf.
 * Q: [n_streams, n_queries, d]; Ksum: [n_streams, n_blocks_stride, d] of which the
 * first n_blocks rows are scored.  dtype GFST_F32 computes with fp32 FMAs;
 * GFST_BF16 runs the tcgen05 tensor-core path (bf16 operands, fp32 accumulate).
 * Limits: 1 <= k <= 32; d a multiple of 8 (bf16) or 4 (f32), d <= 256;
 * bf16: n_streams <= 65535, Q and Ksum 16-byte aligned.                     */
GFST_API int gfst_block_topk(const void* Q, const void* Ksum, int64_t n_streams, int n_queries,
                    int n_blocks, int n_blocks_stride, int d, int k, int dtype,
                    float* top_scores, int32_t* top_idx, cudaStream_t stream);

/* ---- exact top-k of one query, any k -----------------------------------------
 * scores[i] = keys[i,:] . query (fp32 accumulate; with dtype GFST_BF16 and
 * round_scores != 0 each score is rounded to bf16, as the reference's bf16
 * `keys @ q` returns it); out_scores[0..k) / out_idx[0..k) = the k best in the
 * total order (score descending, index ascending; NaN ranks last, -0 == +0).
 * keys: [count, d] (16-byte aligned), query: [d], same dtype (GFST_F32 or
 * GFST_BF16).  Replaces FaissGpuRetriever.exact_topk
 * src/gfst_hmb_mpuc/retrieval.py:165-172 (torch.topk over keys @ q), which is
 * also the oracle the reference's tests compare FAISS search against.
 * Banks of more than 16,384 keys need a caller-provided workspace of
 * gfst_exact_topk_workspace_bytes(count, k) bytes (8-byte aligned; 0 bytes
 * below that size) and k <= 8192.  Limits: 1 <= k <= count < 2^32, d <= 1024,
 * d a multiple of 4 (fp32) or 8 (bf16).                                     */
GFST_API size_t gfst_exact_topk_workspace_bytes(int64_t count, int k);
GFST_API int gfst_exact_topk(const void* keys, const void* query, int64_t count, int d, int k, int dtype,
                    int round_scores, float* out_scores, int64_t* out_idx, void* workspace,
                    size_t workspace_bytes, cudaStream_t stream);

/* ---- exact top-k without allocation -------------------------------------------
 * No counterpart in the reference.  gfst_exact_topk with its workspace taken
 * from a static 1 MiB device array instead of the caller: for callers that
 * cannot allocate device memory per call -- a host whose device memory is
 * reserved up front by its own pool allocator (a raw cudaMalloc would go
 * around that pool and fails once the pool holds the free memory), or a
 * latency-bound loop that cannot take the device-wide synchronisation that
 * cudaFree implies.  The caller still passes keys, query and outputs.
 * Limit: 2 * ceil(count / 16384) * k <= 131072 (the workspace of
 * gfst_exact_topk must fit in 1 MiB); larger requests return GFST_ERR_SHAPE.
 * Every device that loads the library holds the 1 MiB until the process
 * exits.  The first call on a device looks up the array's device address
 * (once per device); make that first call before any stream capture.  All
 * calls share the array, so calls that overlap on the GPU race (serialise
 * them on one stream); nothing in it has to start at zero, since every pass
 * writes the candidates the next one reads.  Same results as gfst_exact_topk. */
GFST_API int gfst_exact_topk_noalloc(const void* keys, const void* query, int64_t count, int d, int k,
                            int dtype, int round_scores, float* out_scores, int64_t* out_idx,
                            cudaStream_t stream);

/* ---- candidate merge ----------------------------------------------------------
 * For every row: the k best of the row's n_cand (score, index) candidates in the
 * total order (score descending, index ascending); candidates with index < 0,
 * NaN or -inf scores are skipped; unfilled slots hold (-inf, -1).  scores/idx:
 * [rows, n_cand]; out: [rows, k].  Merges per-GPU candidate lists after an
 * all-gather when the block memory is sharded by block range (no counterpart
 * in the reference, which runs on one device).  Limits: 1 <= k <= 32.       */
GFST_API int gfst_topk_merge(const float* scores, const int32_t* idx, int64_t rows, int n_cand,
                             int k, float* out_scores, int32_t* out_idx, cudaStream_t stream);

/* ---- device-side failure report ---------------------------------------------
 * Kernels that wait on one another inside a CTA (the tensor-core retrieval
 * pipeline) bound every wait; a wait that gives up records GFST_ERR_TIMEOUT in
 * a sticky per-device word and the kernel returns without hanging.  This call
 * synchronises with the current device's work, returns GFST_OK or the
 * recorded status, and clears the word when `clear` is non-zero.            */
GFST_API int gfst_check_device_errors(int clear);

/* ---- failure-path probe ------------------------------------------------------
 * Launches one CTA that waits on an mbarrier nothing arrives at, for at most
 * `cycles` SM clock cycles (1 <= cycles <= 2e9, about a second at B200
 * clocks), then gives up exactly as a pipeline wait does: GFST_ERR_TIMEOUT is
 * recorded for gfst_check_device_errors and the kernel returns, leaving the
 * context usable.  For testing the failure path without a fault; no
 * counterpart in the reference.                                              */
GFST_API int gfst_debug_bounded_wait(int64_t cycles, cudaStream_t stream);

/* ---- exact-token readout ------------------------------------------------------
 * For every stream s and query q, over the tokens of the k blocks top_idx[s,q,:]
 * (entries < 0 or >= n_slots are skipped; a block listed twice counts once):
 *   score(b, p) = Q[s,q,:] . pool_K[s,b,p,:]        (fp32 accumulate)
 *   best = argmax in the total order (score descending, token index ascending),
 *          token index = b * L + p
 *   best_tok[s,q] = best (or -1 when no block is valid), best_score[s,q] = its score,
 *   out_V[s,q,:] = pool_V[s,best_b,best_p,:] (zeros when no block is valid)
 * Q: [n_streams, n_queries, d]; pool_K: [n_streams, n_slots, L, d];
 * pool_V: [n_streams, n_slots, L, dv] (may be NULL together with out_V);
 * top_idx: [n_streams, n_queries, k].  dtype applies to Q, pool_K, pool_V, out_V.
 * Limits: 1 <= k <= 32, d a multiple of 8, d <= 256, L >= 1.                     */
GFST_API int gfst_exact_readout(const void* Q, const void* pool_K, const void* pool_V,
                       const int32_t* top_idx, int64_t n_streams, int n_queries,
                       int n_slots, int L, int d, int dv, int k, int dtype,
                       int32_t* best_tok, float* best_score, void* out_V,
                       cudaStream_t stream);

/* ---- open-block readout ------------------------------------------------------
 * The exact readout over the prefix of the block still being written, merged
 * into a result over the committed blocks (gfst_exact_readout's outputs, in
 * place).  Replaces the current-block part of the reference's readout
 * (modeling.py:2948-2963: the open block and its prefix length are appended to
 * the retrieved blocks; the token is appended to the exact store,
 * modeling.py:3807 / state.py:651-815, before its own retrieval at :3853).
 * For every stream s and query q with n = open_len(s, q) > 0:
 *   score(p) = Q[s,q,:] . K_open[s,p,:] for p in [0, n)        (fp32 accumulate)
 *   the best open position (score descending, position ascending; NaN never
 *   wins) has token index open_base + p; it replaces (best_tok, best_score,
 *   out_V) of (s, q) when best_tok[s,q] < 0 or it ranks first in (score
 *   descending, token index ascending); out_V[s,q,:] = V_open[s,p,:].
 * open_len: [n_streams, n_queries] int32 (clamped to [0, L_open]), or NULL for
 *   the streaming rule: query q sees positions [0, q] while q < L_open - 1 and
 *   none from q = L_open - 1 on (the reference closes a block in the exact
 *   store at its last token, before that token's retrieval, and appends its
 *   summary only after it).
 * Q: [n_streams, n_queries, d]; K_open: [n_streams, L_open, d]; V_open:
 * [n_streams, L_open, dv] (may be NULL together with out_V); best_tok,
 * best_score: [n_streams, n_queries]; out_V: [n_streams, n_queries, dv].
 * dtype (GFST_F32 or GFST_BF16) applies to Q, K_open, V_open, out_V.
 * Limits: d a multiple of 4, d <= 256; open_base + L_open < 2^31.         */
GFST_API int gfst_open_block_readout(const void* Q, const void* K_open, const void* V_open,
                            const int32_t* open_len, int64_t n_streams, int n_queries, int L_open,
                            int d, int dv, int64_t open_base, int dtype, int32_t* best_tok,
                            float* best_score, void* out_V, cudaStream_t stream);

/* ---- segmented reductions over group ids -------------------------------------
 * inverse[i] in [0, group_count) names element i's group (elements outside
 * that range take no part).  gfst_segmented_max: grouped[g] = max of the
 * group's scores (fmaxf: NaN scores are ignored; -inf for an empty group).
 * gfst_segmented_logsumexp_occurrence: with m the group max, grouped_scores[g]
 * = m + logf(fmaxf(sum exp(s - m), 1e-8)) when m is finite, m + logf(1e-8)
 * otherwise; grouped_blocks[g] / grouped_positions[g] = occurrence_blocks /
 * occurrence_positions of the group's lowest-index element scoring m (-1 when
 * m is not finite or the group is empty).  Each group's sum runs in element
 * order.  All arrays are 1-D; outputs have group_count entries.
 * Limits: n <= 16384, group_count <= 16384 (one CTA; the reference calls them
 * on one query's candidate list).                                            */
GFST_API int gfst_segmented_max(const float* scores, const int64_t* inverse, int64_t n,
                       int64_t group_count, float* grouped, cudaStream_t stream);
GFST_API int gfst_segmented_logsumexp_occurrence(const float* scores, const int64_t* inverse,
                       const int64_t* occurrence_blocks, const int64_t* occurrence_positions,
                       int64_t n, int64_t group_count, float* grouped_scores,
                       int64_t* grouped_blocks, int64_t* grouped_positions, cudaStream_t stream);

/* ---- block token scores through the within-block projection ------------------
 * scores[t] = sum_j key[t, j] * query[j], key[t, j] = sum_c token_features[t, c] *
 * weight[j, c] (fp32 accumulate).  GFST_BF16: key rounded to bf16 and the score
 * rounded to bf16 before widening, as proj(F) @ q in bf16 is; GFST_F32: no
 * rounding.  query: [n]; token_features: [m, k]; weight: [n, k] (the Linear
 * weight, no bias); scores: [m] fp32.  m == 0 is a no-op.                    */
GFST_API int gfst_exact_block_score(const void* query, const void* token_features, const void* weight,
                       int64_t m, int n, int k, int dtype, float* scores, cudaStream_t stream);

/* ---- batched symmetric eigendecomposition -----------------------------------
 * For each of `batch` d x d matrices (row-major, the lower triangle is read):
 * eigenvalues ascending [batch, d]; eigenvectors [batch, d, d] with column j
 * the unit eigenvector of eigenvalue j, signed so that its largest-magnitude
 * entry (lowest index on ties) is positive.  Computed in float64 (cyclic
 * Jacobi); dtype GFST_F32 or GFST_F64 for inputs and outputs.  info (may be
 * NULL): [batch] int32, 0 = converged, 1 = not converged in 40 sweeps (also
 * recorded as GFST_ERR_NUMERIC for gfst_check_device_errors).  1 <= d <= 64. */
GFST_API int gfst_heev(const void* matrices, int64_t batch, int d, int dtype, void* eigenvalues,
                       void* eigenvectors, int32_t* info, cudaStream_t stream);

/* ---- slice of a packed store ------------------------------------------------
 * out[0 : end - start] = packed[start : end], elements of elem_size bytes
 * (packed holds n_elements).  0 <= start <= end <= n_elements; an empty range
 * is a no-op.                                                                 */
GFST_API int gfst_exact_block_materialize(const void* packed, int64_t n_elements, int elem_size, int64_t start,
                       int64_t end, void* out, cudaStream_t stream);

/* ---- exact readout with an int8 first look ---------------------------------
 * gfst_block_commit_i8 writes the int8 copy of one bf16 block per stream
 * (K [n_streams, L, d]) into slot `slot` of pool_K8 [n_streams, n_slots, L, d]
 * int8, and into k8_scale [n_streams, n_slots, L + 4] float32 the per-token
 * scales s (k8 = round(k / s), s = max|k| / 127) followed by the block's
 * (E, N, 0, 0): E >= max |k - s k8|_2 and N >= max |k|_2 over its tokens
 * (rounded up; +inf when a key has a non-finite value).
 * gfst_exact_readout_i8 returns what gfst_exact_readout returns for bf16
 * pools (same arguments, plus pool_K8 and k8_scale of every committed slot):
 * it streams the int8 copies, bounds each (query, token) score by A +- b from
 * the exact integer product of the int8 values and the error norms, and
 * re-scores from pool_K only the tokens whose upper bound reaches the best
 * lower bound of their query (a query with more than 32 such tokens, with
 * non-finite or all-zero values, or selecting a block with a non-finite key,
 * is scored in full).  No reference counterpart: a B200 path for the readout
 * of modeling.py:599-657, 1151-1169.
 * Limits: d = 128 or 256; L % 16 == 0, L <= 256; k <= 32; n_slots L < 2^24. */
GFST_API int gfst_block_commit_i8(const void* K, int8_t* pool_K8, float* k8_scale, int64_t n_streams, int n_slots,
                                  int slot, int L, int d, cudaStream_t stream);
GFST_API int gfst_exact_readout_i8(const void* Q, const void* pool_K, const int8_t* pool_K8, const float* k8_scale,
                                   const void* pool_V, const int32_t* top_idx, int64_t n_streams, int n_queries,
                                   int n_slots, int L, int d, int dv, int k, int32_t* best_tok, float* best_score,
                                   void* out_V, cudaStream_t stream);

/* ---- MPUC recurrent scan ------------------------------------------------------
 * The token loop of MpucGfstHmbBlock._forward_sequence_tensors
 * (src/gfst_hmb_mpuc/modeling.py:4449-4476; cell _token_step 4363-4411,
 * _update_band 4343-4356, bridges up(silu(down(x))) 4182-4183).  Replaces the
 * reference's native mpuc_recurrent_scan_forward(normalized, fast_inputs,
 * mid_inputs, slow_inputs) (csrc/sm120_stub.cu:210-224, caller
 * modeling.py:4424), which takes no weights and returns zeros: this entry
 * point takes the cell's weights.  Widths: fast F, mid M, slow S, bridge rank
 * C, boundary MLP hidden width Bh.  Weights are fp32 in nn.Linear layout
 * ([out, in] row-major, 16-byte aligned matrices):                           */
typedef struct gfst_mpuc_weights {
  const float *fast_gate_w, *fast_gate_b, *fast_cand_w, *fast_cand_b; /* [F, F], [F]     */
  const float *mid_gate_w, *mid_gate_b, *mid_cand_w, *mid_cand_b;     /* [M, M], [M]     */
  const float *slow_gate_w, *slow_gate_b, *slow_cand_w, *slow_cand_b; /* [S, S], [S]     */
  const float *fm_down, *fm_up; /* fast_from_mid:  [C, M], [F, C]                      */
  const float *fs_down, *fs_up; /* fast_from_slow: [C, S], [F, C]                      */
  const float *mf_down, *mf_up; /* mid_from_fast:  [C, F], [M, C]                      */
  const float *ms_down, *ms_up; /* mid_from_slow:  [C, S], [M, C]                      */
  const float *sf_down, *sf_up; /* slow_from_fast: [C, F], [S, C]                      */
  const float *sm_down, *sm_up; /* slow_from_mid:  [C, M], [S, C]                      */
  const float *bnd_w1, *bnd_b1, *bnd_w2, *bnd_b2; /* boundary MLP: [Bh, 4], [Bh], [1, Bh], [1] */
} gfst_mpuc_weights;

/* Workspace bytes gfst_mpuc_recurrent_scan needs for this batch and widths. */
GFST_API int gfst_mpuc_scan_workspace_bytes(int64_t batch, int fast_dim, int mid_dim, int slow_dim,
                                            int cross_rank, size_t* bytes);

/* For each batch element b and token t in order (fp32 throughout):
 *   the recurrence of _token_step on fast_in [batch, T, F], mid_in
 *   [batch, T, M], slow_in [batch, T, S] (the three branch outputs);
 *   states_out [batch, T, F + M + S] = (fast, mid, slow) after token t;
 *   boundary_out [batch, T] = the boundary logit of token t.
 * fast_state [batch, F], mid_state [batch, M], slow_state [batch, S] hold the
 * states before the first token on entry (zeros for a new sequence, as
 * _forward_sequence_tensors starts) and after the last on return.  The output
 * projection (fusion_proj + semantic residual) is not applied: it does not
 * feed back and is one batched product over all tokens.  workspace: at least
 * gfst_mpuc_scan_workspace_bytes (16-byte aligned); it also carries the grid
 * barrier, so concurrent calls need separate workspaces.  One cooperative
 * launch (one CTA per SM) per 8 batch elements.  Limits: F, M, S, C multiples
 * of 4; max(F, M + S, 2 C) <= 6144; T <= 2^20.                               */
GFST_API int gfst_mpuc_recurrent_scan(const gfst_mpuc_weights* weights, int fast_dim, int mid_dim,
                                      int slow_dim, int cross_rank, int boundary_hidden,
                                      const float* fast_in, const float* mid_in, const float* slow_in,
                                      int64_t batch, int T, float* states_out, float* boundary_out,
                                      float* fast_state, float* mid_state, float* slow_state,
                                      void* workspace, size_t workspace_bytes, cudaStream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GFST_B200_H_ */
