"""Exact-token readout inside the selected blocks, on the sm_100a kernel.

Reference (pkhairkh/gfst-hmb-public): ExactRecallReadout._score_block_tokens
(src/gfst_hmb_mpuc/modeling.py:599-657) scores every token of each retrieved
block against the query, and the best-scoring token is the copy target
(modeling.py:1151-1169).  Token ids here are positions (block * L + p), so the
reference's log-sum-exp collapse by token id is the identity; the collapse by
stored token ids runs fused (exact_readout_collapse) or as the reference's
standalone segmented reductions (segmented_max_by_group,
segmented_logsumexp_occurrence).  exact_block_score scores a block's tokens
through the within-block projection.
"""
from __future__ import annotations

import torch

from . import _native as nat


def exact_readout(Q: torch.Tensor, pool_K: torch.Tensor, pool_V: torch.Tensor | None, top_idx: torch.Tensor,
                  *, k8: tuple | None = None):
    """Q [S, Nq, d]; pool_K [S, n_slots, L, d]; pool_V [S, n_slots, L, dv] or None;
    top_idx [S, Nq, k] int32 (entries < 0 skipped).
    Returns (best_tok int32 [S,Nq] (-1 if nothing valid), best_score f32 [S,Nq],
    out_V [S,Nq,dv] or None).

    ``k8`` = (pool_K8 int8 [S, n_slots, L, d], k8_scale float32 [S, n_slots, L + 4]),
    the int8 copies of the keys written by ``block_commit_i8`` (BlockMemory with
    ``int8_keys=True``): the kernel then streams the int8 copies, bounds every
    token's exact score from them and re-scores only the tokens the bound does
    not rule out from the bf16 keys -- the same best token and score, about
    half the bytes (bf16 pools, d = 128 or 256, L % 16 == 0, L <= 256)."""
    nat.require_cuda(Q, pool_K, pool_V, top_idx, what="exact_readout")
    if Q.ndim != 3 or pool_K.ndim != 4 or top_idx.ndim != 3:
        raise ValueError("exact_readout expects Q [S,Nq,d], pool_K [S,slots,L,d], top_idx [S,Nq,k]")
    S, Nq, d = Q.shape
    _, n_slots, L, dk = pool_K.shape
    if dk != d or pool_K.shape[0] != S or tuple(top_idx.shape[:2]) != (S, Nq):
        raise ValueError("exact_readout: shape mismatch")
    if Q.dtype != pool_K.dtype or (pool_V is not None and pool_V.dtype != Q.dtype):
        raise RuntimeError("exact_readout: Q, pool_K and pool_V must share a dtype")
    k = top_idx.shape[2]
    dv = pool_V.shape[-1] if pool_V is not None else 0
    if not pool_K.is_contiguous() or (pool_V is not None and not pool_V.is_contiguous()):
        raise ValueError("exact_readout: pools must be contiguous")
    Q = Q.contiguous()
    top_idx = top_idx.to(torch.int32).contiguous()
    best_tok = torch.empty((S, Nq), dtype=torch.int32, device=Q.device)
    best_score = torch.empty((S, Nq), dtype=torch.float32, device=Q.device)
    out_V = torch.empty((S, Nq, dv), dtype=Q.dtype, device=Q.device) if pool_V is not None else None
    if k8 is not None:
        pool_K8, k8_scale = k8
        nat.require_cuda(pool_K8, k8_scale, what="exact_readout")
        if Q.dtype != torch.bfloat16:
            raise RuntimeError("exact_readout: the int8 first look needs bf16 pools")
        if tuple(pool_K8.shape) != tuple(pool_K.shape) or pool_K8.dtype != torch.int8 or \
                tuple(k8_scale.shape) != (S, n_slots, L + 4) or k8_scale.dtype != torch.float32:
            raise ValueError("exact_readout: k8 must be (int8 [S, slots, L, d], float32 [S, slots, L + 4])")
        if not (pool_K8.is_contiguous() and k8_scale.is_contiguous()):
            raise ValueError("exact_readout: int8 copies must be contiguous")
        with torch.cuda.device(Q.device):
            nat.call("gfst_exact_readout_i8", nat.ptr(Q), nat.ptr(pool_K), nat.ptr(pool_K8), nat.ptr(k8_scale),
                     nat.ptr(pool_V), nat.ptr(top_idx), S, Nq, n_slots, L, d, dv, k, nat.ptr(best_tok),
                     nat.ptr(best_score), nat.ptr(out_V), nat.stream_of(Q))
        return best_tok, best_score, out_V
    with torch.cuda.device(Q.device):
        nat.call("gfst_exact_readout", nat.ptr(Q), nat.ptr(pool_K), nat.ptr(pool_V), nat.ptr(top_idx), S, Nq,
                 n_slots, L, d, dv, k, nat.dtype_code(Q.dtype, "exact_readout"), nat.ptr(best_tok),
                 nat.ptr(best_score), nat.ptr(out_V), nat.stream_of(Q))
    return best_tok, best_score, out_V


def open_block_readout(Q: torch.Tensor, K_open: torch.Tensor, V_open: torch.Tensor | None, best_tok: torch.Tensor,
                       best_score: torch.Tensor, out_V: torch.Tensor | None, *, open_base: int,
                       open_len: torch.Tensor | None = None) -> None:
    """Merge the readout over the open block's prefix into a committed-block
    result, in place (the current block appended to the retrieved blocks with
    its prefix length, modeling.py:2948-2963; the token is appended to the exact
    store before its own retrieval, modeling.py:3807 vs 3853).

    Q [S, Nq, d]; K_open [S, L_open, d]; V_open [S, L_open, dv] or None;
    best_tok int32 / best_score f32 [S, Nq] and out_V [S, Nq, dv] as
    exact_readout returns them.  Query q scores open positions [0, n) with
    n = open_len[s, q] ([S, Nq] int32), or by default n = q + 1 while
    q < L_open - 1 and n = 0 from q = L_open - 1 on (the reference closes the
    block in the exact store at its last token, and its summary becomes
    retrievable only after that token's retrieval).  The best open position p
    (token index open_base + p) replaces the result when it ranks first in
    (score descending, token index ascending)."""
    nat.require_cuda(Q, K_open, V_open, best_tok, best_score, out_V, open_len, what="open_block_readout")
    if Q.ndim != 3 or K_open.ndim != 3 or K_open.shape[0] != Q.shape[0] or K_open.shape[2] != Q.shape[2]:
        raise ValueError("open_block_readout expects Q [S,Nq,d], K_open [S,L_open,d]")
    S, Nq, d = Q.shape
    Lo = K_open.shape[1]
    if tuple(best_tok.shape) != (S, Nq) or tuple(best_score.shape) != (S, Nq):
        raise ValueError("open_block_readout: best_tok / best_score must be [S, Nq]")
    if best_tok.dtype != torch.int32 or best_score.dtype != torch.float32:
        raise RuntimeError("open_block_readout: best_tok must be int32 and best_score float32")
    if (V_open is None) != (out_V is None):
        raise ValueError("open_block_readout: V_open and out_V go together")
    dv = 0
    if V_open is not None:
        dv = V_open.shape[-1]
        if tuple(V_open.shape) != (S, Lo, dv) or tuple(out_V.shape) != (S, Nq, dv):
            raise ValueError("open_block_readout: V_open / out_V shapes do not match")
        if V_open.dtype != Q.dtype or out_V.dtype != Q.dtype:
            raise RuntimeError("open_block_readout: Q, K_open, V_open and out_V must share a dtype")
    if K_open.dtype != Q.dtype:
        raise RuntimeError("open_block_readout: Q and K_open must share a dtype")
    for t in (best_tok, best_score, out_V):
        if t is not None and not t.is_contiguous():
            raise ValueError("open_block_readout: outputs must be contiguous")
    if open_len is not None:
        if tuple(open_len.shape) != (S, Nq):
            raise ValueError("open_block_readout: open_len must be [S, Nq]")
        open_len = open_len.to(torch.int32).contiguous()
    Q, K_open = Q.contiguous(), K_open.contiguous()
    V_open = V_open.contiguous() if V_open is not None else None
    with torch.cuda.device(Q.device):
        nat.call("gfst_open_block_readout", nat.ptr(Q), nat.ptr(K_open), nat.ptr(V_open), nat.ptr(open_len), S, Nq,
                 Lo, d, dv, int(open_base), nat.dtype_code(Q.dtype, "open_block_readout"), nat.ptr(best_tok),
                 nat.ptr(best_score), nat.ptr(out_V), nat.stream_of(Q))


def exact_readout_collapse(Q: torch.Tensor, pool_K: torch.Tensor, token_ids: torch.Tensor, top_idx: torch.Tensor):
    """The readout with the reference's log-sum-exp collapse of duplicate token
    ids (perf.py:164-229 collapse_logsumexp_scores_and_occurrence, then the
    select of modeling.py:1151-1169): Q [S, Nq, d]; pool_K [S, n_slots, L, d];
    token_ids [S, n_slots, L] int32 (the id stored at each position, < 0 =
    padding); top_idx [S, Nq, k].  Returns (best_id, best_score, best_block,
    best_pos), each [S, Nq]: the winning token id, its group score and the
    (block, position) of its best occurrence."""
    nat.require_cuda(Q, pool_K, token_ids, top_idx, what="exact_readout_collapse")
    S, Nq, d = Q.shape
    _, n_slots, L, dk = pool_K.shape
    if dk != d or tuple(token_ids.shape) != (S, n_slots, L) or tuple(top_idx.shape[:2]) != (S, Nq):
        raise ValueError("exact_readout_collapse: shape mismatch")
    if Q.dtype != pool_K.dtype:
        raise RuntimeError("exact_readout_collapse: Q and pool_K must share a dtype")
    k = top_idx.shape[2]
    Q, pool_K = Q.contiguous(), pool_K.contiguous()
    ids = token_ids.to(torch.int32).contiguous()
    sel = top_idx.to(torch.int32).contiguous()
    out = [torch.empty((S, Nq), dtype=dt, device=Q.device)
           for dt in (torch.int32, torch.float32, torch.int32, torch.int32)]
    with torch.cuda.device(Q.device):
        nat.call("gfst_exact_readout_collapse", nat.ptr(Q), nat.ptr(pool_K), nat.ptr(ids), nat.ptr(sel), S, Nq,
                 n_slots, L, d, k, nat.dtype_code(Q.dtype, "exact_readout_collapse"), *(nat.ptr(t) for t in out),
                 nat.stream_of(Q))
    return tuple(out)


SEGMENTED_MAX_ELEMENTS = 16384


def _rank1(what: str, *tensors: torch.Tensor) -> int:
    if any(t.ndim != 1 for t in tensors):
        raise ValueError(f"{what}: inputs must be rank-1 tensors")
    n = int(tensors[0].numel())
    if any(int(t.numel()) != n for t in tensors):
        raise ValueError(f"{what}: inputs must have matching element counts")
    return n


def segmented_max_by_group(scores: torch.Tensor, inverse: torch.Tensor, group_count: int) -> torch.Tensor:
    """Per-group max of ``scores`` (runtime backend ``segmented_max_by_group``,
    src/gfst_hmb_mpuc/csrc/sm120_stub.cu:16-40, 150-172): ``inverse[i]`` in
    ``[0, group_count)`` names element i's group.  NaN scores are ignored (fmaxf);
    an empty group gets -inf.  Returns float32 [group_count]."""
    nat.require_cuda(scores, inverse, what="segmented_max_by_group")
    n = _rank1("segmented_max_by_group", scores, inverse)
    scores = scores.float().contiguous()
    inverse = inverse.to(torch.int64).contiguous()
    out = torch.empty((int(group_count),), dtype=torch.float32, device=scores.device)
    with torch.cuda.device(scores.device):
        nat.call("gfst_segmented_max", nat.ptr(scores), nat.ptr(inverse), n, int(group_count), nat.ptr(out),
                 nat.stream_of(scores))
    return out


def segmented_logsumexp_occurrence(scores: torch.Tensor, inverse: torch.Tensor, occurrence_blocks: torch.Tensor,
                                   occurrence_positions: torch.Tensor, *, group_count: int):
    """Per-group log-sum-exp and best occurrence (runtime backend
    ``segmented_logsumexp_occurrence``, src/gfst_hmb_mpuc/csrc/sm120_stub.cu:42-111,
    174-208).  With m the group max: score m + log(max(sum exp(s - m), 1e-8)) and
    the (block, position) of the group's lowest-index element scoring m when m is
    finite; m + log(1e-8) and (-1, -1) otherwise.  Returns (grouped_scores f32,
    grouped_blocks int64, grouped_positions int64), each [group_count]."""
    nat.require_cuda(scores, inverse, occurrence_blocks, occurrence_positions, what="segmented_logsumexp_occurrence")
    n = _rank1("segmented_logsumexp_occurrence", scores, inverse, occurrence_blocks, occurrence_positions)
    scores = scores.float().contiguous()
    inverse, blocks, positions = (t.to(torch.int64).contiguous()
                                  for t in (inverse, occurrence_blocks, occurrence_positions))
    g = int(group_count)
    out = (torch.empty((g,), dtype=torch.float32, device=scores.device),
           torch.empty((g,), dtype=torch.int64, device=scores.device),
           torch.empty((g,), dtype=torch.int64, device=scores.device))
    with torch.cuda.device(scores.device):
        nat.call("gfst_segmented_logsumexp_occurrence", nat.ptr(scores), nat.ptr(inverse), nat.ptr(blocks),
                 nat.ptr(positions), n, g, *(nat.ptr(t) for t in out), nat.stream_of(scores))
    return out


def collapse_max_scores_by_group(scores: torch.Tensor, group_ids: torch.Tensor):
    """perf.collapse_max_scores_by_group (src/gfst_hmb_mpuc/perf.py:136-161) on the
    segmented kernel: returns (unique_ids int64 sorted, grouped max f32)."""
    n = _rank1("collapse_max_scores_by_group", scores, group_ids)
    if n == 0:
        return group_ids.new_empty((0,), dtype=torch.long), scores.new_empty((0,), dtype=torch.float32)
    unique_ids, inverse = torch.unique(group_ids.to(torch.long), sorted=True, return_inverse=True)
    return unique_ids, segmented_max_by_group(scores, inverse, int(unique_ids.numel()))


def collapse_logsumexp_scores_and_occurrence(scores: torch.Tensor, group_ids: torch.Tensor,
                                             occurrence_blocks: torch.Tensor, occurrence_positions: torch.Tensor):
    """perf.collapse_logsumexp_scores_and_occurrence (src/gfst_hmb_mpuc/perf.py:164-229)
    on the segmented kernel: returns (unique_ids, grouped_scores, grouped_blocks,
    grouped_positions)."""
    n = _rank1("collapse_logsumexp_scores_and_occurrence", scores, group_ids, occurrence_blocks,
               occurrence_positions)
    if n == 0:
        empty_long = group_ids.new_empty((0,), dtype=torch.long)
        return empty_long, scores.new_empty((0,), dtype=torch.float32), empty_long, empty_long
    unique_ids, inverse = torch.unique(group_ids.to(torch.long), sorted=True, return_inverse=True)
    grouped = segmented_logsumexp_occurrence(scores, inverse, occurrence_blocks, occurrence_positions,
                                             group_count=int(unique_ids.numel()))
    return (unique_ids, *grouped)


def exact_block_score(query: torch.Tensor, token_features: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Scores of a block's tokens through the within-block projection (runtime
    backend ``exact_block_score``; projection exact_block_project_forward,
    src/gfst_hmb_mpuc/csrc/sm120_cutlass_exact_block_score.cu:42-129, dotted with
    the query as modeling.py:640-651 does): query [n]; token_features [m, k];
    weight [n, k] (the bias-free Linear weight).  Returns float32 [m] =
    (token_features @ weight.T) @ query, with bf16 roundings of the keys and the
    score for bfloat16 inputs."""
    nat.require_cuda(query, token_features, weight, what="exact_block_score")
    if query.ndim != 1 or token_features.ndim != 2 or weight.ndim != 2:
        raise ValueError("exact_block_score expects query [n], token_features [m, k], weight [n, k]")
    m, k = token_features.shape
    n, kw = weight.shape
    if kw != k or query.shape[0] != n:
        raise ValueError("exact_block_score: dimension mismatch")
    if not (query.dtype == token_features.dtype == weight.dtype):
        raise RuntimeError("exact_block_score: query, token_features and weight must share a dtype")
    query, token_features, weight = query.contiguous(), token_features.contiguous(), weight.contiguous()
    scores = torch.empty((m,), dtype=torch.float32, device=query.device)
    with torch.cuda.device(query.device):
        nat.call("gfst_exact_block_score", nat.ptr(query), nat.ptr(token_features), nat.ptr(weight), m, n, k,
                 nat.dtype_code(query.dtype, "exact_block_score"), nat.ptr(scores), nat.stream_of(query))
    return scores
