"""Centroid path of the exact-token memory on the GPU.

Drop-in for the reference's centroid cell write and centroid readout
(pkhairkh/gfst-hmb-public):

* ``centroid_cell_commit`` -- what GfstDecodeState.append_exact_token
  (cuda_packed backend, src/gfst_hmb_mpuc/state.py:315-470) stores for the L
  tokens of a block plus _finalise_block_cells (state.py:501-551), for many
  blocks at once, on the kernel ``gfst_centroid_cell_commit``;
* ``centroid_readout`` -- ExactRecallReadout._build_centroid_candidates
  (src/gfst_hmb_mpuc/modeling.py:659-982) with the token-id collapse and the
  best group (perf.py:164-229, modeling.py:1151-1169), on
  ``gfst_centroid_readout``.

The learned projections stay with the caller, as linear maps applied once per
query (``centroid_query_proj``) and once per stored token (``within_block_proj``
-> token keys, ``centroid_token_proj`` -> token features).  There is no CPU
path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as nat


class _Params(ctypes.Structure):
    _fields_ = [("block_score_lambda", ctypes.c_float), ("background_subtract", ctypes.c_int),
                ("count_penalty", ctypes.c_float), ("self_field_weight", ctypes.c_float),
                ("top_cells_per_head", ctypes.c_int), ("fdr_q", ctypes.c_float), ("min_selected", ctypes.c_int),
                ("temperature", ctypes.c_float), ("entropy_low", ctypes.c_float), ("entropy_high", ctypes.c_float),
                ("gamma_m", ctypes.c_float), ("gamma_r", ctypes.c_float)]


@dataclass
class CentroidParams:
    """ExactRecallReadout's centroid attributes (modeling.py:371-448; the
    defaults are GfstHmbConfig's, config.py:35-63, and the module's own
    block-score lambda and gains)."""
    block_score_lambda: float = 0.10
    background_subtract: bool = True
    count_penalty: float = 0.5
    self_field_weight: float = 0.15
    top_cells_per_head: int = 8
    fdr_q: float = 0.10
    min_selected: int = 2
    temperature: float = 1.0
    entropy_low: float = 0.35
    entropy_high: float = 0.75
    gamma_m: float = 1.0
    gamma_r: float = 1.0

    def to_c(self) -> _Params:
        return _Params(float(self.block_score_lambda), int(bool(self.background_subtract)), float(self.count_penalty),
                       float(self.self_field_weight), int(self.top_cells_per_head), float(self.fdr_q),
                       int(self.min_selected), float(self.temperature), float(self.entropy_low),
                       float(self.entropy_high), float(self.gamma_m), float(self.gamma_r))


def centroid_cell_commit(cell_ids: torch.Tensor, cell_weights: torch.Tensor, cell_keys: torch.Tensor,
                         cell_values: torch.Tensor, cells_per_block: int):
    """cell_ids int32 [B, L, W], cell_weights float32 [B, L, W], cell_keys float32
    [B, L, dk], cell_values float32 [B, L, dv] (B blocks, any leading shape
    flattened).  Returns (token_cell_ids u8 [B, L, W], token_cell_weights_q u8
    [B, L, W], cell_keys fp16 [B, C, dk], cell_values_q int8 [B, C, dv],
    cell_counts int16 [B, C])."""
    nat.require_cuda(cell_ids, cell_weights, cell_keys, cell_values, what="centroid_cell_commit")
    if cell_ids.dtype != torch.int32 or cell_weights.dtype != torch.float32 or cell_keys.dtype != torch.float32 \
            or cell_values.dtype != torch.float32:
        raise RuntimeError("centroid_cell_commit: int32 ids and float32 weights / keys / values expected")
    *lead, L, W = cell_ids.shape
    dk, dv = int(cell_keys.shape[-1]), int(cell_values.shape[-1])
    if tuple(cell_weights.shape) != tuple(cell_ids.shape) or tuple(cell_keys.shape[:-1]) != (*lead, L) \
            or tuple(cell_values.shape[:-1]) != (*lead, L):
        raise ValueError("centroid_cell_commit: shape mismatch")
    B = 1
    for v in lead:
        B *= int(v)
    C = int(cells_per_block)
    dev = cell_ids.device
    ids_u8 = torch.empty((*lead, L, W), device=dev, dtype=torch.uint8)
    wq_u8 = torch.empty((*lead, L, W), device=dev, dtype=torch.uint8)
    keys = torch.empty((*lead, C, dk), device=dev, dtype=torch.float16)
    vals = torch.empty((*lead, C, dv), device=dev, dtype=torch.int8)
    counts = torch.empty((*lead, C), device=dev, dtype=torch.int16)
    ci, cw, ck, cv = (t.contiguous() for t in (cell_ids, cell_weights, cell_keys, cell_values))
    with torch.cuda.device(dev):
        nat.call("gfst_centroid_cell_commit", nat.ptr(ci), nat.ptr(cw), nat.ptr(ck), nat.ptr(cv), B, L, W, C, dk, dv,
                 nat.ptr(ids_u8), nat.ptr(wq_u8), nat.ptr(keys), nat.ptr(vals), nat.ptr(counts), nat.stream_of(ci))
    return ids_u8, wq_u8, keys, vals, counts


@dataclass
class CentroidReadout:
    best_id: torch.Tensor        # [S, Nq] int32, -1 when no candidate
    best_score: torch.Tensor     # [S, Nq] float32
    best_block: torch.Tensor     # [S, Nq] int32 (memory slot)
    best_pos: torch.Tensor       # [S, Nq] int32
    candidate_scores: torch.Tensor | None = None  # [S, Nq, K, L]
    selected_block: torch.Tensor | None = None    # [S, Nq, H, width] entry index (selection order of valid blocks)
    selected_cell: torch.Tensor | None = None     # [S, Nq, H, width]
    selected_alpha: torch.Tensor | None = None    # [S, Nq, H, width]
    head_stats: torch.Tensor | None = None        # [S, Nq, H, 3]: entropy, margin, selected count
    confidence: torch.Tensor | None = None        # [S, Nq], -1 where the centroid terms were off


def centroid_readout(Q: torch.Tensor, query_heads: torch.Tensor, sel_idx: torch.Tensor, sel_scores: torch.Tensor, *,
                     token_keys: torch.Tensor, token_features: torch.Tensor, token_ids: torch.Tensor,
                     token_cell_ids: torch.Tensor, token_cell_weights_q: torch.Tensor, cell_keys: torch.Tensor,
                     cell_values_q: torch.Tensor, cell_counts: torch.Tensor, prefix_len: torch.Tensor | None = None,
                     params: CentroidParams | None = None, return_candidates: bool = False,
                     return_diagnostics: bool = False) -> CentroidReadout:
    """Q [S, Nq, dq], query_heads [S, Nq, H, dk] float32; sel_idx int32 / sel_scores
    float32 [S, Nq, K] (and prefix_len int32 [S, Nq, K] or None); the store:
    token_keys [S, NB, L, dq], token_features [S, NB, L, H, dv] float32,
    token_ids int32 [S, NB, L], token_cell_ids / token_cell_weights_q u8
    [S, NB, L, W], cell_keys fp16 [S, NB, C, dk], cell_values_q int8
    [S, NB, C, dv], cell_counts int16 [S, NB, C]."""
    prm = params or CentroidParams()
    nat.require_cuda(Q, query_heads, sel_idx, sel_scores, token_keys, token_features, token_ids, token_cell_ids,
                     token_cell_weights_q, cell_keys, cell_values_q, cell_counts, prefix_len, what="centroid_readout")
    S, Nq, dq = Q.shape
    H, dk = int(query_heads.shape[-2]), int(query_heads.shape[-1])
    K = int(sel_idx.shape[-1])
    NB, L = int(token_ids.shape[1]), int(token_ids.shape[2])
    W = int(token_cell_ids.shape[-1])
    C, dv = int(cell_counts.shape[-1]), int(cell_values_q.shape[-1])
    expect = {"query_heads": (query_heads, (S, Nq, H, dk), torch.float32),
              "sel_idx": (sel_idx, (S, Nq, K), torch.int32), "sel_scores": (sel_scores, (S, Nq, K), torch.float32),
              "token_keys": (token_keys, (S, NB, L, dq), torch.float32),
              "token_features": (token_features, (S, NB, L, H, dv), torch.float32),
              "token_ids": (token_ids, (S, NB, L), torch.int32),
              "token_cell_ids": (token_cell_ids, (S, NB, L, W), torch.uint8),
              "token_cell_weights_q": (token_cell_weights_q, (S, NB, L, W), torch.uint8),
              "cell_keys": (cell_keys, (S, NB, C, dk), torch.float16),
              "cell_values_q": (cell_values_q, (S, NB, C, dv), torch.int8),
              "cell_counts": (cell_counts, (S, NB, C), torch.int16)}
    if prefix_len is not None:
        expect["prefix_len"] = (prefix_len, (S, Nq, K), torch.int32)
    if Q.dtype != torch.float32:
        raise RuntimeError("centroid_readout: Q must be float32")
    for name, (t, shape, dt) in expect.items():
        if tuple(t.shape) != shape:
            raise ValueError(f"centroid_readout: {name} {tuple(t.shape)} != {shape}")
        if t.dtype != dt:
            raise RuntimeError(f"centroid_readout: {name} must be {dt}")
    dev = Q.device
    width = int(prm.top_cells_per_head)
    out = CentroidReadout(best_id=torch.empty((S, Nq), device=dev, dtype=torch.int32),
                          best_score=torch.empty((S, Nq), device=dev, dtype=torch.float32),
                          best_block=torch.empty((S, Nq), device=dev, dtype=torch.int32),
                          best_pos=torch.empty((S, Nq), device=dev, dtype=torch.int32))
    if return_candidates:
        out.candidate_scores = torch.empty((S, Nq, K, L), device=dev, dtype=torch.float32)
    if return_diagnostics:
        out.selected_block = torch.empty((S, Nq, H, width), device=dev, dtype=torch.int32)
        out.selected_cell = torch.empty((S, Nq, H, width), device=dev, dtype=torch.int32)
        out.selected_alpha = torch.empty((S, Nq, H, width), device=dev, dtype=torch.float32)
        out.head_stats = torch.empty((S, Nq, H, 3), device=dev, dtype=torch.float32)
        out.confidence = torch.empty((S, Nq), device=dev, dtype=torch.float32)
    ts = [t.contiguous() for t in (Q, query_heads, sel_idx, sel_scores)]
    pl = prefix_len.contiguous() if prefix_len is not None else None
    st = [t.contiguous() for t in (token_keys, token_features, token_ids, token_cell_ids, token_cell_weights_q,
                                   cell_keys, cell_values_q, cell_counts)]
    cprm = prm.to_c()
    with torch.cuda.device(dev):
        nat.call("gfst_centroid_readout", *(nat.ptr(t) for t in ts), nat.ptr(pl), *(nat.ptr(t) for t in st),
                 S, Nq, NB, L, dq, H, dk, dv, C, W, K, ctypes.cast(ctypes.pointer(cprm), ctypes.c_void_p),
                 nat.ptr(out.candidate_scores), nat.ptr(out.best_id), nat.ptr(out.best_score), nat.ptr(out.best_block),
                 nat.ptr(out.best_pos), nat.ptr(out.selected_block), nat.ptr(out.selected_cell),
                 nat.ptr(out.selected_alpha), nat.ptr(out.head_stats), nat.ptr(out.confidence), nat.stream_of(Q))
    return out
