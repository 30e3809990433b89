"""Exact-token readout inside the selected blocks, on the sm_100a kernel.

Reference (pkhairkh/gfst-hmb-public): ExactRecallReadout._score_block_tokens
(src/gfst_hmb_mpuc/modeling.py:599-657) scores every token of each retrieved
block against the query, and the best-scoring token is the copy target
(modeling.py:1151-1169).  Token ids here are positions (block * L + p), so the
reference's log-sum-exp collapse by token id is the identity.
"""
from __future__ import annotations

import torch

from . import _native as nat


def exact_readout(Q: torch.Tensor, pool_K: torch.Tensor, pool_V: torch.Tensor | None, top_idx: torch.Tensor):
    """Q [S, Nq, d]; pool_K [S, n_slots, L, d]; pool_V [S, n_slots, L, dv] or None;
    top_idx [S, Nq, k] int32 (entries < 0 skipped).
    Returns (best_tok int32 [S,Nq] (-1 if nothing valid), best_score f32 [S,Nq],
    out_V [S,Nq,dv] or None)."""
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
    with torch.cuda.device(Q.device):
        nat.call("gfst_exact_readout", nat.ptr(Q), nat.ptr(pool_K), nat.ptr(pool_V), nat.ptr(top_idx), S, Nq,
                 n_slots, L, d, dv, k, nat.dtype_code(Q.dtype, "exact_readout"), nat.ptr(best_tok),
                 nat.ptr(best_score), nat.ptr(out_V), nat.stream_of(Q))
    return best_tok, best_score, out_V


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
