"""CPU restatement of the reference's GFST-HMB hot path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline /
reference arm, never by the product package.  Every function names the
reference file:line (pkhairkh/gfst-hmb-public) it restates.  Arrays are numpy;
the QR uses torch's CPU LAPACK binding, which is the exact call the reference
makes (``torch.linalg.qr(..., mode="reduced")``, src/gfst_hmb_mpuc/gfst.py:29).
"""
from __future__ import annotations

import numpy as np
import torch

SIGN_FIRST_SIGNIFICANT = 0
SIGN_R_DIAG_POSITIVE = 1


# ---------------------------------------------------------------------------
# bf16 helpers (round to nearest even, as torch / CUDA do)
# ---------------------------------------------------------------------------
def to_bf16_f32(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 and widen back to float32."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def as_f32(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", torch.float32).numpy()
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# frames
# ---------------------------------------------------------------------------
def canonicalize_qr_column_signs(q: np.ndarray, eps_sign: float = 1e-8) -> np.ndarray:
    """gfst.py:35-46: per column, the first row with |q| > eps_sign decides the
    sign; a negative entry flips the column; columns without one stay."""
    q = np.asarray(q)
    mask = np.abs(q) > np.float32(eps_sign)
    first = np.argmax(mask, axis=-2)  # first True row (0 if none)
    first_vals = np.take_along_axis(q, first[..., None, :], axis=-2)[..., 0, :]
    flip = mask.any(axis=-2) & (first_vals < 0)
    sign = np.where(flip, -1.0, 1.0).astype(q.dtype)
    return q * sign[..., None, :]


def qr_reference(matrices: np.ndarray, eps_sign: float = 1e-8,
                 sign_mode: int = SIGN_FIRST_SIGNIFICANT) -> np.ndarray:
    """gfst.py:26-32 (canonical_qr_batched): reduced Householder QR in float32
    through LAPACK, then the sign rule.  ``SIGN_R_DIAG_POSITIVE`` multiplies each
    column by sign(R_jj) (sign(0) = +1) instead."""
    a = torch.from_numpy(np.ascontiguousarray(matrices, dtype=np.float32))
    if a.numel() == 0:
        return np.zeros(matrices.shape, dtype=np.float32)
    q, r = torch.linalg.qr(a, mode="reduced")
    q = q.numpy()
    if sign_mode == SIGN_R_DIAG_POSITIVE:
        diag = np.diagonal(r.numpy(), axis1=-2, axis2=-1)
        return q * np.where(diag < 0, -1.0, 1.0).astype(np.float32)[..., None, :]
    return canonicalize_qr_column_signs(q, eps_sign)


def qr_fp64(matrices: np.ndarray, eps_sign: float = 1e-8, sign_mode: int = SIGN_FIRST_SIGNIFICANT) -> np.ndarray:
    """Same as qr_reference in float64 (error analysis: distance to the exact Q)."""
    a = torch.from_numpy(np.ascontiguousarray(matrices, dtype=np.float64))
    q, r = torch.linalg.qr(a, mode="reduced")
    q = q.numpy()
    if sign_mode == SIGN_R_DIAG_POSITIVE:
        diag = np.diagonal(r.numpy(), axis1=-2, axis2=-1)
        return q * np.where(diag < 0, -1.0, 1.0)[..., None, :]
    return canonicalize_qr_column_signs(q, eps_sign)


def frame_candidate(U: np.ndarray, A: np.ndarray | None, B: np.ndarray | None, beta: float = 1.0) -> np.ndarray:
    """beta*U + A B^T in float32: the candidate form of gfst.py:136-140, which
    also covers the plain rank-m update U + sum_i u_i v_i^T of the streaming
    workloads (beta = 1)."""
    U = np.asarray(U, dtype=np.float32)
    c = (np.float32(beta) * U) if beta != 1.0 else U.copy()
    if A is not None:
        c = c + np.matmul(np.asarray(A, np.float32), np.swapaxes(np.asarray(B, np.float32), -1, -2))
    return c.astype(np.float32)


def residual_rank_one_candidate(U: np.ndarray, x: np.ndarray, alpha: float, eps_update: float = 1e-6) -> np.ndarray:
    """gfst.py:115-140 (update_basis_candidate_batched, rule residual_rank_one_v1)."""
    Ut = torch.from_numpy(np.asarray(U, np.float32))
    xt = torch.from_numpy(np.asarray(x, np.float32))
    weights = torch.matmul(Ut.transpose(-2, -1), xt.unsqueeze(-1)).squeeze(-1)
    projection = torch.matmul(Ut, weights.unsqueeze(-1)).squeeze(-1)
    residual = xt - projection
    norm = torch.linalg.vector_norm(xt, dim=-1, keepdim=True)
    scaled = residual / torch.sqrt(norm.square() + float(eps_update) ** 2)
    novelty = torch.zeros_like(weights)
    novelty[..., -1] = 1.0
    out = (1.0 - alpha) * Ut + alpha * xt.unsqueeze(-1) * weights.unsqueeze(-2) \
        + alpha * scaled.unsqueeze(-1) * novelty.unsqueeze(-2)
    return out.numpy()


def stream_frames(U0: np.ndarray, A: np.ndarray, B: np.ndarray, beta: float = 1.0, eps_sign: float = 1e-8,
                  sign_mode: int = SIGN_FIRST_SIGNIFICANT, out_every: int = 0):
    """Per-token loop of modeling.py:2355-2374 (update candidate, canonical QR)
    over frames [F, d, r] with inputs A [F, T, d, m], B [F, T, r, m].
    Returns (final frames, snapshots [T//out_every, F, d, r] or None)."""
    U = np.array(U0, dtype=np.float32, copy=True)
    T = A.shape[1]
    snaps = []
    for t in range(T):
        U = qr_reference(frame_candidate(U, A[:, t], B[:, t], beta), eps_sign, sign_mode)
        if out_every and (t + 1) % out_every == 0:
            snaps.append(U.copy())
    return U, (np.stack(snaps) if snaps else None)


def _residual_rank_one_candidate_2d(basis: torch.Tensor, value: torch.Tensor, alpha: float,
                                    eps_update: float) -> torch.Tensor:
    """gfst.py:91-112 (update_basis_candidate): the unbatched form, with the
    matrix-vector products of one tracker."""
    weights = basis.transpose(0, 1) @ value
    residual = value - basis @ weights
    norm = torch.linalg.vector_norm(value)
    scaled = residual / torch.sqrt(norm.square() + float(eps_update) ** 2)
    novelty = torch.zeros_like(weights)
    novelty[-1] = 1.0
    return (1.0 - alpha) * basis + alpha * torch.outer(value, weights) + alpha * torch.outer(scaled, novelty)


def _canonical_qr_1(candidate: torch.Tensor, eps_sign: float, sign_mode: int) -> torch.Tensor:
    """gfst.py:26-32 on a batch of one, as the tracker calls it."""
    return torch.from_numpy(qr_reference(candidate.unsqueeze(0).numpy(), eps_sign, sign_mode)[0])


def local_tracker_stream(U0: np.ndarray, nested0: list, xs: np.ndarray, flag_dims, forgetting_rates,
                         eps: float = 1e-6, eps_update: float = 1e-6, eps_sign: float = 1e-8,
                         sign_mode: int = SIGN_FIRST_SIGNIFICANT, out_every: int = 0):
    """Per-token local tracker of modeling.py:2299-2423 (_update_local_bases)
    followed by modeling.py:2425-2437 (_local_alignment_features), one tracker
    per stream, in the reference's own unbatched torch calls.

    U0 [S, d, r] (r = max flag dim); nested0: list of [S, r, dim_l] for the
    flag levels but the last; xs [S, T, d].  Per token: the largest basis takes
    the residual_rank_one_v1 candidate at rate forgetting_rates[-1] and its
    canonical QR; p = U^T x; nested level l takes the same rule on p at
    forgetting_rates[l]; features = (cumulative, increment) pairs of
    ||V_l^T p||^2 / max(||x||^2, eps), then ||p||^2 / max(||x||^2, eps).
    Returns (U, nested list, features [S, T, 2 (L + 1)], snapshots [T//out_every, S, d, r] or None).
    """
    xs = np.asarray(xs, np.float32)
    S, T, _ = xs.shape
    nl = len(nested0)
    U_out = np.array(U0, np.float32, copy=True)
    V_out = [np.array(v, np.float32, copy=True) for v in nested0]
    feats = np.zeros((S, T, 2 * (nl + 1)), np.float32)
    snaps = np.zeros((T // out_every if out_every else 0, S) + U_out.shape[1:], np.float32)
    for s in range(S):
        U = torch.from_numpy(U_out[s].copy())
        V = [torch.from_numpy(v[s].copy()) for v in V_out]
        for t in range(T):
            x = torch.from_numpy(xs[s, t].copy())
            U = _canonical_qr_1(_residual_rank_one_candidate_2d(U, x, float(forgetting_rates[-1]), eps_update),
                                eps_sign, sign_mode)
            p = U.transpose(0, 1) @ x
            for lvl in range(nl):
                cand = _residual_rank_one_candidate_2d(V[lvl], p, float(forgetting_rates[lvl]), eps_update)
                V[lvl] = _canonical_qr_1(cand, eps_sign, sign_mode)[:, : int(flag_dims[lvl])]
            p = U.transpose(0, 1) @ x
            den = torch.clamp(x.square().sum(), min=float(eps))
            cum = [(Vl.transpose(0, 1) @ p).square().sum() / den for Vl in V]
            cum.append(p.square().sum() / den)
            c = torch.stack(cum)
            prev = torch.cat((torch.zeros_like(c[:1]), c[:-1]))
            feats[s, t] = torch.stack((c, c - prev), dim=-1).reshape(-1).numpy()
            if out_every and (t + 1) % out_every == 0:
                snaps[(t + 1) // out_every - 1, s] = U.numpy()
        U_out[s] = U.numpy()
        for lvl in range(nl):
            V_out[lvl][s] = V[lvl].numpy()
    return U_out, V_out, feats, (snaps if out_every else None)


def block_tracker_stream(U0: np.ndarray, projector_sum0: np.ndarray, reduced_sum0: np.ndarray, xs: np.ndarray,
                         rate: float, eps_update: float = 1e-6, eps_sign: float = 1e-8,
                         sign_mode: int = SIGN_FIRST_SIGNIFICANT):
    """Per-token part of the block tracker, modeling.py:3460-3479: the rule
    update at ``rate`` (forgetting_rates[-1]) and canonical QR of the block
    basis, projector_sum += basis_projector(U) (gfst.py:143-144), reduced_sum +=
    x; one tracker per stream in the reference's unbatched torch calls.
    U0 [S, d, r], projector_sum0 [S, d, d], reduced_sum0 [S, d], xs [S, T, d]."""
    xs = np.asarray(xs, np.float32)
    S, T, _ = xs.shape
    U_out = np.array(U0, np.float32, copy=True)
    P_out = np.array(projector_sum0, np.float32, copy=True)
    R_out = np.array(reduced_sum0, np.float32, copy=True)
    for s in range(S):
        U = torch.from_numpy(U_out[s].copy())
        P = torch.from_numpy(P_out[s].copy())
        R = torch.from_numpy(R_out[s].copy())
        for t in range(T):
            x = torch.from_numpy(xs[s, t].copy())
            U = _canonical_qr_1(_residual_rank_one_candidate_2d(U, x, float(rate), eps_update), eps_sign, sign_mode)
            P = P + U @ U.transpose(0, 1)
            R = R + x
        U_out[s], P_out[s], R_out[s] = U.numpy(), P.numpy(), R.numpy()
    return U_out, P_out, R_out


# frame metrics ---------------------------------------------------------------
def orthogonality_error(Q: np.ndarray) -> np.ndarray:
    """max |Q^T Q - I| per frame (float64 arithmetic)."""
    Q = np.asarray(Q, np.float64)
    g = np.matmul(np.swapaxes(Q, -1, -2), Q)
    eye = np.eye(Q.shape[-1])
    return np.abs(g - eye).max(axis=(-1, -2))


def subspace_distance(Q1: np.ndarray, Q2: np.ndarray, prefix: int | None = None) -> np.ndarray:
    """Principal-angle distance max sin(theta) between span(Q1[:, :p]) and
    span(Q2[:, :p]) per frame, in float64.  Both bases are re-orthonormalised in
    float64 first (so fp32 orthogonality error does not masquerade as angle),
    then sin(theta_max) = ||(I - Q2 Q2^T) Q1||_2, which has no cancellation for
    small angles."""
    Q1 = np.asarray(Q1, np.float64)
    Q2 = np.asarray(Q2, np.float64)
    if prefix is not None:
        Q1 = Q1[..., :prefix]
        Q2 = Q2[..., :prefix]
    Q1 = np.linalg.qr(Q1)[0]
    Q2 = np.linalg.qr(Q2)[0]
    resid = Q1 - np.matmul(Q2, np.matmul(np.swapaxes(Q2, -1, -2), Q1))
    return np.linalg.svd(resid, compute_uv=False).max(axis=-1)


def max_prefix_subspace_distance(Q1: np.ndarray, Q2: np.ndarray) -> np.ndarray:
    """Largest principal-angle distance over every leading-column prefix 1..r
    (the nested flag subspaces of modeling.py:2380-2417)."""
    r = Q1.shape[-1]
    return np.max(np.stack([subspace_distance(Q1, Q2, p) for p in range(1, r + 1)]), axis=0)


# ---------------------------------------------------------------------------
# block commit
# ---------------------------------------------------------------------------
def block_commit_mean(K_block: np.ndarray, bf16: bool) -> np.ndarray:
    """Summary key of a block = mean of its L token keys (the mean-of-keys summary
    of the streaming workloads; the reference's eigen-based block summary is
    modeling.py:3496-3507).  Sum in token
    order in float32, divide by L in float32, round once to bf16 when the memory
    is bf16.  K_block: [..., L, d] float32 (bf16-representable for bf16 memory)."""
    K = np.asarray(K_block, np.float32)
    acc = np.zeros(K.shape[:-2] + K.shape[-1:], np.float32)
    for t in range(K.shape[-2]):
        acc = (acc + K[..., t, :]).astype(np.float32)
    mean = (acc / np.float32(K.shape[-2])).astype(np.float32)
    return to_bf16_f32(mean) if bf16 else mean


EIG_CLUSTER_ATOL = 1e-9   # gfst.py:6
EIG_CLUSTER_RTOL = 1e-7   # gfst.py:7


def _first_significant_signs(q: torch.Tensor, eps_sign: float) -> torch.Tensor:
    """gfst.py:35-46 on a torch tensor of any float dtype."""
    mask = q.abs() > float(eps_sign)
    first = torch.argmax(mask.to(torch.int64), dim=-2)
    vals = torch.gather(q, -2, first.unsqueeze(-2)).squeeze(-2)
    sign = torch.where(mask.any(dim=-2) & vals.lt(0), -torch.ones_like(vals), torch.ones_like(vals))
    return q * sign.unsqueeze(-2)


def _cluster_basis(cluster: torch.Tensor, target_rank: int, eps: float, eps_sign: float) -> torch.Tensor:
    """gfst.py:172-214 (_canonical_basis_from_cluster_space): Gram-Schmidt over the
    cluster projector's columns taken in descending-diagonal order (ties: lower
    axis first), then over the cluster's own columns if that falls short; signs
    by the first significant entry.  float64."""
    projector = cluster @ cluster.transpose(0, 1)
    diag = torch.diag(projector)
    order = sorted(range(projector.shape[0]), key=lambda a: (-float(diag[a].item()), a))
    cols: list[torch.Tensor] = []

    def append(candidate):
        v = candidate.clone()
        for c in cols:
            v = v - torch.dot(c, v) * c
        n = torch.linalg.norm(v)
        if float(n.item()) > eps:
            cols.append(v / n)

    for a in order:
        if len(cols) >= target_rank:
            break
        append(projector[:, a])
    for j in range(cluster.shape[1]):
        if len(cols) >= target_rank:
            break
        append(cluster[:, j])
    if len(cols) < target_rank:
        raise RuntimeError("cluster basis short of its rank")
    return _first_significant_signs(torch.stack(cols[:target_rank], dim=1), eps_sign)


def _canonical_top_basis(sketch: torch.Tensor, target: int, eps_sign: float) -> torch.Tensor:
    """gfst.py:389-430 (top_eig_summary's full_basis): symmetrise in float32,
    float64 eigh, clusters walked from the top, each replaced by its canonical
    basis (gfst.py:232-297), float32 with signs fixed again."""
    sym = (0.5 * (sketch + sketch.transpose(0, 1))).to(torch.float64)
    vals, vecs = torch.linalg.eigh(sym)
    rank = max(0, min(int(target), vecs.shape[0]))
    parts, remaining, end = [], rank, vals.shape[0] - 1
    while end >= 0 and remaining > 0:
        start = end
        while start > 0 and abs(float(vals[start - 1]) - float(vals[start])) <= \
                EIG_CLUSTER_ATOL + EIG_CLUSTER_RTOL * abs(float(vals[start])):
            start -= 1
        take = min(end - start + 1, remaining)
        parts.append(_cluster_basis(vecs[:, start:end + 1], take, 1e-9, eps_sign))
        remaining -= take
        end = start - 1
    return _first_significant_signs(torch.cat(parts, dim=1).to(torch.float32), eps_sign)


def global_features(bank, sel_idx, sel_scores, x, temperature: float, flag_dims, max_flag_dim: int,
                    eps: float = 1e-6, eps_sign: float = 1e-8):
    """Global sketch features per (stream, query), the torch branch of
    _resolve_single_global_request (modeling.py:2996-3108): w = softmax(scores *
    temperature) over the valid selections, sketch = sum_k w_k P[idx_k],
    top_eig_summary's canonical basis B, prefix projectors 0.5 (B_m B_m^T +
    (B_m B_m^T)^T), alignment_components (gfst.py:580-588).  bank [S, NB, d, d],
    sel_idx / sel_scores [S, Nq, K], x [S, Nq, d].  Returns (features [S, Nq, 2F],
    basis [S, Nq, d, max_flag_dim])."""
    bank = torch.as_tensor(np.asarray(bank, np.float32))
    sel_idx = np.asarray(sel_idx)
    scores = torch.as_tensor(np.asarray(sel_scores, np.float32))
    x = torch.as_tensor(np.asarray(x, np.float32))
    S, Nq, _ = sel_idx.shape
    d = bank.shape[-1]
    target = max(int(max_flag_dim), max(int(m) for m in flag_dims), 1)
    feats = np.zeros((S, Nq, 2 * len(flag_dims)), np.float32)
    bases = np.zeros((S, Nq, d, int(max_flag_dim)), np.float32)
    for s in range(S):
        for q in range(Nq):
            valid = [j for j in range(sel_idx.shape[2]) if 0 <= int(sel_idx[s, q, j]) < bank.shape[1]]
            if not valid:
                continue
            w = torch.softmax(scores[s, q, valid] * float(temperature), dim=0)
            sketch = torch.einsum("k,kij->ij", w, bank[s, [int(sel_idx[s, q, j]) for j in valid]])
            full = _canonical_top_basis(sketch, target, eps_sign)
            v = x[s, q]
            denom = torch.dot(v, v) + eps
            cum = []
            for m in flag_dims:
                p = full[:, : int(m)] @ full[:, : int(m)].transpose(0, 1)
                p = 0.5 * (p + p.transpose(0, 1))
                cum.append(torch.dot(v, p @ v) / denom)
            c = torch.stack(cum)
            prev = torch.cat((torch.zeros_like(c[:1]), c[:-1]))
            feats[s, q] = torch.stack((c, c - prev), dim=-1).reshape(-1).numpy()
            bases[s, q] = full[:, : int(max_flag_dim)].numpy()
    return feats, bases


def block_commit_eig(projector_sum, reduced_sum, token_count: int, max_flag_dim: int, flag_dims,
                     eps_sign: float = 1e-8):
    """Reference-faithful block commit for one block: replay_block_commit_bundle
    native path (diagnostics/block_commit_replay.py:97-139) = average projector,
    top_eig_summary (gfst.py:389-430: symmetrise in the input dtype, float64
    eigh, clusters of eigenvalues equal within atol 1e-9 / rtol 1e-7 walked from
    the top, each replaced by its canonical basis, gfst.py:232-297), reduced mean.
    projector_sum [d, d] float32, reduced_sum [d] float32.  Returns numpy float32
    (summary_basis [d, max_flag_dim], reduced_mean [d], top_vector [d],
    average_projector [d, d])."""
    ps = torch.as_tensor(np.asarray(projector_sum, np.float32))
    rs = torch.as_tensor(np.asarray(reduced_sum, np.float32))
    avg = ps / float(token_count)
    mean = rs / float(token_count)
    target = max(int(max_flag_dim), max((int(b) for b in flag_dims), default=0), 1)
    full = _canonical_top_basis(avg, target, eps_sign)
    basis = full[:, : max(0, min(int(max_flag_dim), full.shape[1]))]
    top = full[:, 0] if full.shape[1] > 0 else torch.zeros(ps.shape[0])
    return basis.numpy(), mean.numpy(), top.numpy(), avg.numpy()


def collapse_logsumexp(scores, token_ids, blocks, positions):
    """perf.py:164-229 (collapse_logsumexp_scores_and_occurrence, native
    branch), restated: unique token ids ascending; per group m = max, score =
    m + log(max(sum exp(s - m), 1e-8)) with the sum in element order; the
    occurrence is the first element scoring m.  float32."""
    s = torch.as_tensor(np.asarray(scores, np.float32))
    ids = torch.as_tensor(np.asarray(token_ids, np.int64))
    uid, inv = torch.unique(ids, sorted=True, return_inverse=True)
    g = int(uid.numel())
    mx = s.new_full((g,), float("-inf"))
    mx.scatter_reduce_(0, inv, s, reduce="amax", include_self=True)
    stable = torch.exp(s - mx.index_select(0, inv))
    sumexp = s.new_zeros((g,))
    sumexp.scatter_add_(0, inv, stable)
    gs = mx + sumexp.clamp_min(1e-8).log()
    flat = torch.arange(s.numel())
    cand = torch.where(s.eq(mx.index_select(0, inv)), flat, torch.full_like(flat, s.numel()))
    first = torch.full((g,), s.numel(), dtype=torch.long)
    first.scatter_reduce_(0, inv, cand, reduce="amin", include_self=True)
    b = torch.as_tensor(np.asarray(blocks, np.int64)).index_select(0, first)
    p = torch.as_tensor(np.asarray(positions, np.int64)).index_select(0, first)
    return uid.numpy(), gs.numpy(), b.numpy(), p.numpy()


def segmented_max(scores, inverse, group_count):
    """sm120_stub.cu:16-40 (segmented_max_kernel), restated: per group the max
    of its scores with fmaxf semantics (NaN ignored), -inf for an empty group;
    elements whose group lies outside [0, group_count) take no part.  float32."""
    s = np.asarray(scores, np.float32)
    inv = np.asarray(inverse, np.int64)
    out = np.full(int(group_count), -np.inf, np.float32)
    for i in range(s.size):
        g = int(inv[i])
        if 0 <= g < group_count and not np.isnan(s[i]):
            out[g] = max(out[g], s[i])
    return out


def segmented_logsumexp_occurrence(scores, inverse, blocks, positions, group_count):
    """sm120_stub.cu:42-111 (segmented_logsumexp_occurrence_kernel), restated:
    m = the group max (segmented_max); when m is finite, sum = sum exp(s - m)
    over the group in element order and the occurrence is the lowest index with
    s == m; otherwise sum = 0 and no occurrence (-1, -1).  score = m +
    log(max(sum, 1e-8)), where a NaN sum counts as below 1e-8 (fmaxf).
    float32 arithmetic throughout."""
    s = np.asarray(scores, np.float32)
    inv = np.asarray(inverse, np.int64)
    bl = np.asarray(blocks, np.int64)
    po = np.asarray(positions, np.int64)
    m = segmented_max(s, inv, group_count)
    gs = np.empty(int(group_count), np.float32)
    gb = np.full(int(group_count), -1, np.int64)
    gp = np.full(int(group_count), -1, np.int64)
    with np.errstate(invalid="ignore", over="ignore"):
        for g in range(int(group_count)):
            total, best = np.float32(0.0), -1
            if np.isfinite(m[g]):
                for i in np.nonzero(inv == g)[0]:
                    total = np.float32(total + np.exp(np.float32(s[i] - m[g]), dtype=np.float32))
                    if best < 0 and s[i] == m[g]:
                        best = int(i)
            clamped = np.float32(1e-8) if not total >= np.float32(1e-8) else total
            gs[g] = np.float32(m[g] + np.log(clamped, dtype=np.float32))
            if best >= 0:
                gb[g], gp[g] = bl[best], po[best]
    return gs, gb, gp


def exact_readout_collapse(Q, pool_K, token_ids, top_idx):
    """Readout with the token-id collapse: candidates = tokens of the selected
    blocks in selection order (modeling.py:599-657; a block listed twice counts
    once; ids < 0 and NaN scores left out), float32 scores key . q,
    collapse_logsumexp, then the best group (score descending, id ascending;
    modeling.py:1151-1169).  Returns (best_id, best_score, best_block, best_pos)."""
    Q = np.asarray(Q, np.float32)
    K = np.asarray(pool_K, np.float32)
    ids = np.asarray(token_ids)
    S, Nq, _ = Q.shape
    L = K.shape[2]
    out = (np.full((S, Nq), -1, np.int32), np.full((S, Nq), -np.inf, np.float32), np.full((S, Nq), -1, np.int32),
           np.full((S, Nq), -1, np.int32))
    for s in range(S):
        for q in range(Nq):
            seen, blocks = set(), []
            for b in top_idx[s, q]:
                b = int(b)
                if 0 <= b < K.shape[1] and b not in seen:
                    seen.add(b)
                    blocks.append(b)
            if not blocks:
                continue
            keys = torch.as_tensor(np.concatenate([K[s, b] for b in blocks]))
            sc = (keys @ torch.as_tensor(Q[s, q])).numpy()
            tid = np.concatenate([ids[s, b] for b in blocks])
            blk = np.repeat(np.array(blocks), L)
            pos = np.tile(np.arange(L), len(blocks))
            keep = (tid >= 0) & ~np.isnan(sc)
            if not keep.any():
                continue
            uid, gs, gb, gp = collapse_logsumexp(sc[keep], tid[keep], blk[keep], pos[keep])
            w = int(np.lexsort((uid, -gs))[0])
            out[0][s, q], out[1][s, q], out[2][s, q], out[3][s, q] = uid[w], gs[w], gb[w], gp[w]
    return out


# ---------------------------------------------------------------------------
# top-k block select
# ---------------------------------------------------------------------------
def _order_desc_idx_asc(scores: np.ndarray) -> np.ndarray:
    """Indices sorting the last axis by (score desc, index asc); NaN last."""
    s = np.where(np.isnan(scores), -np.inf, scores)
    n = s.shape[-1]
    idx = np.broadcast_to(np.arange(n), s.shape)
    # lexsort: last key is primary
    order = np.lexsort((idx, -s), axis=-1)
    return order


def block_scores(Q: np.ndarray, Ksum: np.ndarray) -> np.ndarray:
    """scores[s, q, b] = Q[s,q] . Ksum[s,b] in float64 (exact enough to rank
    bf16/fp32 inputs; retrieval.py:165-172 computes keys @ q)."""
    return np.matmul(np.asarray(Q, np.float64), np.swapaxes(np.asarray(Ksum, np.float64), -1, -2))


def block_topk(Q: np.ndarray, Ksum: np.ndarray, k: int):
    """retrieval.py:165-172 (exact_topk) batched over streams and queries, with
    the deterministic total order (score desc, block index asc).  Blocks
    scoring NaN or -inf are never selected.  Returns (top_scores f32 [S,Nq,k],
    top_idx int32 [S,Nq,k], margin_ok bool [S,Nq]); unfilled slots hold
    (-inf, -1).  margin_ok is False when the k-th and (k+1)-th scores are within
    1e-3 relative, where either order of the boundary is acceptable."""
    scores = block_scores(Q, Ksum)
    scores = np.where(np.isnan(scores), -np.inf, scores)
    nb = scores.shape[-1]
    order = _order_desc_idx_asc(scores)
    kk = min(k, nb)
    top_idx = np.full(scores.shape[:-1] + (k,), -1, np.int32)
    top_sc = np.full(scores.shape[:-1] + (k,), -np.inf, np.float32)
    sel_sc = np.take_along_axis(scores, order[..., :kk], axis=-1)
    live = np.isfinite(sel_sc) | (sel_sc > 0)
    top_idx[..., :kk] = np.where(live, order[..., :kk], -1)
    top_sc[..., :kk] = np.where(live, sel_sc, -np.inf).astype(np.float32)
    margin_ok = np.ones(scores.shape[:-1], bool)
    if nb > kk:
        sk = np.take_along_axis(scores, order[..., kk - 1:kk], axis=-1)[..., 0]
        sn = np.take_along_axis(scores, order[..., kk:kk + 1], axis=-1)[..., 0]
        margin_ok = np.abs(sk - sn) > 1e-3 * np.maximum(np.abs(sk), 1e-30)
    return top_sc, top_idx, margin_ok


def exact_topk(keys: np.ndarray, query: np.ndarray, k: int, round_bf16: bool = False):
    """retrieval.py:165-172 (FaissGpuRetriever.exact_topk): scores = keys @ q,
    the best min(k, count) as (indices int64, scores float32), in the total
    order (score desc, index asc; NaN last).  round_bf16: the scores of a bf16
    bank, which the reference's bf16 matmul returns rounded to bf16 (here the
    float64 dot rounded to float32, then to bf16)."""
    sc = np.asarray(keys, np.float64) @ np.asarray(query, np.float64)
    sc = sc.astype(np.float32)
    if round_bf16:
        sc = to_bf16_f32(sc)
    key = np.where(np.isnan(sc), -np.inf, sc).astype(np.float64)
    nan_last = np.isnan(sc).astype(np.int8)
    idx = np.arange(sc.shape[0])
    order = np.lexsort((idx, -key, nan_last))
    kk = min(int(k), sc.shape[0])
    return order[:kk].astype(np.int64), sc[order[:kk]]


def same_topk_up_to_ties(idx_a, sc_a, idx_b, sc_b, all_scores) -> bool:
    """Two top-k answers agree when their score lists are equal and, for every
    score value, the same keys were chosen -- except at the k-th score, where
    any keys of that score are a valid completion (the reference's torch.topk
    orders equal scores arbitrarily)."""
    sc_a, sc_b = np.asarray(sc_a, np.float32), np.asarray(sc_b, np.float32)
    if sc_a.shape != sc_b.shape or not np.array_equal(sc_a, sc_b, equal_nan=True):
        return False
    if sc_a.size == 0:
        return True
    kth = sc_a[-1]
    inner = sc_a != kth
    if set(np.asarray(idx_a)[inner].tolist()) != set(np.asarray(idx_b)[inner].tolist()):
        return False
    all_scores = np.asarray(all_scores, np.float32)
    for ia, ib in zip(np.asarray(idx_a)[~inner], np.asarray(idx_b)[~inner]):
        if all_scores[int(ia)] != kth or all_scores[int(ib)] != kth:
            return False
    return True


# ---------------------------------------------------------------------------
# exact-token readout
# ---------------------------------------------------------------------------
def exact_readout(Q: np.ndarray, pool_K: np.ndarray, pool_V: np.ndarray | None, top_idx: np.ndarray,
                  open_K: np.ndarray | None = None, open_V: np.ndarray | None = None,
                  open_len: np.ndarray | None = None, open_base: int = 0):
    """modeling.py:599-657 (_score_block_tokens: token score = key . query) and
    modeling.py:1151-1169 (best token = first of the scores sorted descending),
    with token index b*L + p and the total order (score desc, index asc); NaN
    scores never win and a block listed twice counts once.
    Q [S,Nq,d]; pool_K [S,NB,L,d]; pool_V [S,NB,L,dv]; top_idx [S,Nq,k] int.
    Optionally the open block (modeling.py:2948-2963: the current block is
    appended to the retrieved blocks with its prefix length): open_K [S,Lo,d],
    open_V [S,Lo,dv], open_len [S,Nq] (positions [0, n) of the open block are
    candidates too, with token index open_base + p).
    Returns (best_tok int32 [S,Nq], best_score f32 [S,Nq], out_V [S,Nq,dv] or None,
    margin_ok bool [S,Nq] -- False when the runner-up is within 1e-3 relative)."""
    S, Nq, _ = Q.shape
    L = pool_K.shape[2]
    NB = pool_K.shape[1]
    best_tok = np.full((S, Nq), -1, np.int32)
    best_score = np.full((S, Nq), -np.inf, np.float32)
    margin_ok = np.ones((S, Nq), bool)
    dv = pool_V.shape[-1] if pool_V is not None else 0
    out_V = np.zeros((S, Nq, dv), np.float32) if pool_V is not None else None
    for s in range(S):
        for q in range(Nq):
            blocks = sorted({int(b) for b in top_idx[s, q] if 0 <= b < NB})
            key_parts = [pool_K[s, b] for b in blocks]
            tok_parts = [b * L + np.arange(L) for b in blocks]
            n_open = 0 if open_K is None else int(min(max(int(open_len[s, q]), 0), open_K.shape[1]))
            if n_open > 0:
                key_parts.append(open_K[s, :n_open])
                tok_parts.append(open_base + np.arange(n_open))
            if not key_parts:
                continue
            keys = np.concatenate(key_parts, axis=0).astype(np.float64)
            toks = np.concatenate(tok_parts)
            sc = keys @ np.asarray(Q[s, q], np.float64)
            keep = ~np.isnan(sc)  # NaN scores never win
            if not keep.any():
                continue
            keys, toks, sc = keys[keep], toks[keep], sc[keep]
            order = np.lexsort((toks, -sc))
            w = order[0]
            best_tok[s, q] = toks[w]
            best_score[s, q] = np.float32(sc[w])
            if len(order) > 1:
                s1, s2 = sc[order[0]], sc[order[1]]
                margin_ok[s, q] = abs(s1 - s2) > 1e-3 * max(abs(s1), 1e-30)
            if pool_V is not None:
                tw = int(toks[w])
                out_V[s, q] = open_V[s, tw - open_base] if tw >= open_base and n_open > 0 else \
                    pool_V[s, tw // L, tw % L]
    return best_tok, best_score, out_V, margin_ok


def streaming_open_len(n_queries: int, block_len: int) -> np.ndarray:
    """Open-block prefix each query of a block sees (modeling.py:2948-2963 with
    the exact-store append at modeling.py:3807 before the retrieval at :3853):
    query p sees positions [0, p] while p < L - 1; at p = L - 1 append_exact_token
    has already closed the block (state.py:749-815) and its summary is appended
    only after the retrieval (modeling.py:3632), so that query sees none."""
    p = np.arange(n_queries)
    return np.where(p < block_len - 1, p + 1, 0).astype(np.int32)


def streaming_pass(U0, A, B, K, V, Q, *, block_len: int, n_slots: int, k: int, memory_bf16: bool,
                   sign_mode: int = SIGN_R_DIAG_POSITIVE, eps_sign: float = 1e-8):
    """The streaming step composed token by token in the reference's order
    (GfstHmbSublayer, modeling.py:3590-3640 and 3790-3870), with the
    benchmark's simplifications (update U + A B^T, mean-of-keys block summary,
    identity within-block projection, token keys / values / queries given):

      for each token t (position p = t mod L of its block):
        1. frame update + thin QR (modeling.py:3600-3607; gfst.py:26-46, 115-140)
        2. append the token to the open block of the exact store
           (modeling.py:3807; state.py:651-815); at p = L - 1 the block closes
        3. retrieval: top-k over the committed summaries (modeling.py:3853 ->
           2714-2920; retrieval.py:165-172)
        4. readout: the tokens of the selected blocks and positions [0, p] of the
           open block while p < L - 1 (modeling.py:2948-2963, 599-657, 1151-1169)
        5. at p = L - 1, after the retrieval, the block's summary is appended
           (modeling.py:3632 -> 3401-3571) and the block joins the memory.

    The memory holds the last n_slots committed blocks, block b in slot
    b mod n_slots (the reference keeps every block; both agree while fewer than
    n_slots + 1 blocks are committed).  Committed token index = slot * L + p;
    open-block position p = n_slots * L + p.
    U0 [S,d,r]; A [S,T,d,m]; B [S,T,r,m]; K, V, Q [S,T,d] float32 (bf16-valued
    when memory_bf16).  Returns a dict of per-token arrays: frames [S,T,d,r],
    top_idx [S,T,k], top_ok [S,T], best_tok [S,T], best_score [S,T], value
    [S,T,dv], read_ok [S,T]."""
    U = np.array(U0, np.float32, copy=True)
    A, B = np.asarray(A, np.float32), np.asarray(B, np.float32)
    K, V, Q = (np.asarray(x, np.float32) for x in (K, V, Q))
    S, T, d, _ = A.shape
    L = int(block_len)
    dv = V.shape[-1]
    pool_K = np.zeros((S, n_slots, L, d), np.float32)
    pool_V = np.zeros((S, n_slots, L, dv), np.float32)
    summary = np.zeros((S, n_slots, d), np.float32)
    open_K = np.zeros((S, L, d), np.float32)
    open_V = np.zeros((S, L, dv), np.float32)
    committed = 0
    out = {"frames": np.zeros((S, T) + U.shape[1:], np.float32),
           "top_idx": np.full((S, T, k), -1, np.int32), "top_ok": np.ones((S, T), bool),
           "best_tok": np.full((S, T), -1, np.int32), "best_score": np.full((S, T), -np.inf, np.float32),
           "value": np.zeros((S, T, dv), np.float32), "read_ok": np.ones((S, T), bool)}
    for t in range(T):
        p = t % L
        U = qr_reference(frame_candidate(U, A[:, t], B[:, t]), eps_sign, sign_mode)
        out["frames"][:, t] = U
        open_K[:, p], open_V[:, p] = K[:, t], V[:, t]
        n_open = p + 1 if p < L - 1 else 0
        n_valid = min(committed, n_slots)
        top_i = np.full((S, 1, k), -1, np.int32)
        if n_valid > 0:
            _, top_i, ok = block_topk(Q[:, t:t + 1], summary[:, :n_valid], k)
            out["top_ok"][:, t] = ok[:, 0]
        out["top_idx"][:, t] = top_i[:, 0]
        bt, bs, bv, rok = exact_readout(Q[:, t:t + 1], pool_K, pool_V, top_i, open_K, open_V,
                                        np.full((S, 1), n_open, np.int32), n_slots * L)
        out["best_tok"][:, t], out["best_score"][:, t] = bt[:, 0], bs[:, 0]
        out["value"][:, t], out["read_ok"][:, t] = bv[:, 0], rok[:, 0]
        if p == L - 1:
            slot = committed % n_slots
            pool_K[:, slot], pool_V[:, slot] = open_K, open_V
            summary[:, slot] = block_commit_mean(open_K, memory_bf16)
            committed += 1
    return out
