"""CPU restatement of the reference's centroid path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/ (and the golden-vector script's checks), never by the
product package.  Restates, with the same torch operations in the same order
(pkhairkh/gfst-hmb-public):

* the centroid cell write of a block: GfstDecodeState._append_exact_token_cuda_packed
  (src/gfst_hmb_mpuc/state.py:315-470: u8 cell ids and x255-quantised weights
  per token, weighted key / value / count sums per cell) and
  _finalise_block_cells (state.py:501-551: mean keys in fp16, x32-quantised int8
  mean values, x32-quantised int16 counts);
* the significance-gated centroid readout: ExactRecallReadout._build_centroid_candidates
  (src/gfst_hmb_mpuc/modeling.py:659-982): cell scores per centroid head, robust
  z-scores (median / MAD), count penalty and self field, BH-FDR selection per
  head with a minimum-selection fallback, softmax weights, activation mass per
  (block, cell), token mass and centroid-recall log-sum-exp, final token scores.

The learned projections of the reference (centroid_query_proj,
centroid_token_proj, within_block_proj) are linear maps that the caller applies
(to the query, and to every stored token once); these functions take their
outputs: query heads [H, dk], token features [P, H, dv] and base token scores [P].
"""
from __future__ import annotations

import math

import numpy as np
import torch

VALUE_QUANT_SCALE = 32.0   # state.py:12
WEIGHT_QUANT_SCALE = 255.0  # state.py:13
COUNT_QUANT_SCALE = 32.0   # state.py:14


def cell_commit(cell_ids, cell_weights, cell_keys, cell_values, cells_per_block: int):
    """One block of L tokens written through state.py:315-470 and closed by
    state.py:501-551.  cell_ids int [L, W], cell_weights float32 [L, W],
    cell_keys float32 [L, dk], cell_values float32 [L, dv].  Returns
    (ids u8 [L, W], weights_q u8 [L, W], keys f16 [C, dk], values_q i8 [C, dv],
    counts_q i16 [C])."""
    ids_in = torch.as_tensor(np.asarray(cell_ids), dtype=torch.long)
    w_in = torch.as_tensor(np.asarray(cell_weights, np.float32))
    k_in = torch.as_tensor(np.asarray(cell_keys, np.float32))
    v_in = torch.as_tensor(np.asarray(cell_values, np.float32))
    L, W = ids_in.shape
    C, dk, dv = int(cells_per_block), k_in.shape[1], v_in.shape[1]
    ids_u8 = torch.zeros((L, W), dtype=torch.uint8)
    wq_u8 = torch.zeros((L, W), dtype=torch.uint8)
    key_sum = torch.zeros((C, dk), dtype=torch.float32)
    val_sum = torch.zeros((C, dv), dtype=torch.float32)
    counts = torch.zeros((C,), dtype=torch.float32)
    for t in range(L):
        ids_t = ids_in[t].clamp(min=0, max=max(0, C - 1))                        # state.py:366-367
        q = torch.clamp(torch.round(w_in[t] * WEIGHT_QUANT_SCALE), min=0.0,
                        max=WEIGHT_QUANT_SCALE).to(torch.uint8)                   # state.py:377-381
        ids_u8[t] = ids_t.to(torch.uint8)
        wq_u8[t] = q
        w = q.to(torch.float32) / WEIGHT_QUANT_SCALE                              # state.py:406
        pos = w.gt(0.0)
        if bool(pos.any()):
            ii, ww = ids_t[pos], w[pos]
            key_sum.index_add_(0, ii, ww.unsqueeze(-1) * k_in[t].unsqueeze(0))    # state.py:411-413
            val_sum.index_add_(0, ii, ww.unsqueeze(-1) * v_in[t].unsqueeze(0))
            counts.index_add_(0, ii, ww)
    safe = counts.clamp_min(1.0).unsqueeze(-1)                                    # state.py:528-537
    mean_k = torch.where(counts.unsqueeze(-1).gt(0), key_sum / safe, torch.zeros_like(key_sum))
    mean_v = torch.where(counts.unsqueeze(-1).gt(0), val_sum / safe, torch.zeros_like(val_sum))
    vals_q = torch.clamp(torch.round(mean_v * VALUE_QUANT_SCALE), min=-127.0, max=127.0).to(torch.int8)
    counts_q = torch.clamp(torch.round(counts * COUNT_QUANT_SCALE), min=0.0, max=32767.0).to(torch.int16)
    return (ids_u8.numpy(), wq_u8.numpy(), mean_k.to(torch.float16).numpy(), vals_q.numpy(), counts_q.numpy())


def _median_lower(x: torch.Tensor) -> torch.Tensor:
    """torch.median over the last dim (the lower of the two middle values)."""
    return x.median(dim=-1, keepdim=True).values


def centroid_candidates(query_heads, blocks, *, block_score_lambda=0.10, background_subtract=True,
                        count_penalty=0.5, self_field_weight=0.15, top_cells_per_head=8, fdr_q=0.10,
                        min_selected=2, temperature=1.0, entropy_low=0.35, entropy_high=0.75, gamma_m=1.0,
                        gamma_r=1.0, cells_per_block=16, recall_chunk_size=256):
    """modeling.py:659-982 on precomputed projections.

    query_heads: float32 [H, dk] (centroid_query_proj(query) reshaped).
    blocks: list (retrieval order) of dicts with keys token_ids [P], cell_ids [P, W],
      weights_q [P, W], cell_keys f16 [C, dk], cell_values_q i8 [C, dv],
      cell_counts i16 [C], base_scores float32 [P] (within_block_proj(e) @ query),
      features float32 [P, H, dv] (centroid_token_proj(e) reshaped), block_score.
    Returns None where the reference does, else (scores per block, diag dict)."""
    qh = torch.as_tensor(np.asarray(query_heads, np.float32))
    H, dk = qh.shape
    width = int(top_cells_per_head)
    flat_keys, flat_values, flat_bi, flat_ci, flat_bias, flat_counts, flat_self = [], [], [], [], [], [], []
    for bi, blk in enumerate(blocks):                                             # modeling.py:690-727
        counts_i = torch.as_tensor(np.asarray(blk["cell_counts"])).to(torch.long)
        valid = counts_i.gt(0)
        if not bool(valid.any()):
            continue
        vid = torch.nonzero(valid, as_tuple=False).reshape(-1)
        keys = torch.as_tensor(np.asarray(blk["cell_keys"])).to(torch.float32)
        vals = torch.as_tensor(np.asarray(blk["cell_values_q"])).to(torch.float32)
        cnt = torch.as_tensor(np.asarray(blk["cell_counts"])).to(torch.float32)
        flat_keys.append(keys.index_select(0, vid))
        flat_values.append(vals.index_select(0, vid) / VALUE_QUANT_SCALE)
        flat_counts.append(cnt.index_select(0, vid) / COUNT_QUANT_SCALE)
        local = torch.log1p(cnt.index_select(0, vid).clamp_min(0.0))
        flat_self.append(local - local.mean())
        flat_bi.append(torch.full((int(vid.numel()),), bi, dtype=torch.long))
        flat_ci.append(vid)
        flat_bias.append(torch.full((int(vid.numel()),), float(blk["block_score"]), dtype=torch.float32))
    if not flat_keys:
        return None
    all_keys, all_values = torch.cat(flat_keys), torch.cat(flat_values)
    all_bi, all_ci = torch.cat(flat_bi), torch.cat(flat_ci)
    all_bias, all_counts, all_self = torch.cat(flat_bias), torch.cat(flat_counts), torch.cat(flat_self)
    raw = (qh @ all_keys.transpose(0, 1)) / math.sqrt(float(dk))                  # modeling.py:744-745
    raw = raw + float(block_score_lambda) * all_bias.unsqueeze(0)
    centered = raw - _median_lower(raw) if background_subtract else raw          # modeling.py:747-756
    mad = _median_lower(centered.abs())
    sigma = torch.clamp(1.4826 * mad, min=1e-4)
    z = centered / sigma
    z = z - float(count_penalty) * torch.log1p(all_counts.clamp_min(0.0)).unsqueeze(0)
    z = z + float(self_field_weight) * all_self.unsqueeze(0)
    topk = min(width, int(all_keys.shape[0]))
    if width <= 0 or topk <= 0:
        return None
    nb = len(blocks)
    dv = int(all_values.shape[1])
    mass = torch.zeros((nb, int(cells_per_block)), dtype=torch.float32)
    sel_values = torch.zeros((H, width, dv), dtype=torch.float32)
    log_alpha = torch.full((H, width), float("-inf"), dtype=torch.float32)
    sel_blocks = torch.full((H, width), -1, dtype=torch.long)
    sel_cells = torch.full((H, width), -1, dtype=torch.long)
    sel_alphas = torch.zeros((H, width), dtype=torch.float32)
    entropy = torch.zeros((H,), dtype=torch.float32)
    margin = torch.zeros((H,), dtype=torch.float32)
    signif = torch.zeros((H,), dtype=torch.float32)
    counts_sel = torch.zeros((H,), dtype=torch.float32)
    for h in range(H):                                                            # modeling.py:802-865
        hs = z[h]
        ranked_scores, ranked_idx = torch.topk(hs, k=topk, dim=-1)
        pv = 0.5 * torch.erfc(hs / math.sqrt(2.0))
        sp, si = torch.sort(pv, dim=-1)
        ranks = torch.arange(1, int(sp.shape[0]) + 1, dtype=torch.float32)
        thr = float(fdr_q) * (ranks / float(max(1, int(sp.shape[0]))))
        sig = sp.le(thr)
        if bool(sig.any()):
            upto = int(torch.nonzero(sig, as_tuple=False).reshape(-1)[-1]) + 1
            kept = si[:upto]
            ks, kp = hs.index_select(0, kept), pv.index_select(0, kept)
            order = torch.argsort(ks, descending=True)
            kept, ks, kp = kept.index_select(0, order), ks.index_select(0, order), kp.index_select(0, order)
        else:
            ks, kept, kp = ranked_scores.new_empty((0,)), ranked_idx.new_empty((0,)), ranked_scores.new_empty((0,))
        if int(kept.numel()) < int(min_selected):
            kc = min(int(min_selected), int(ranked_idx.numel()))
            ks, kept = ranked_scores[:kc], ranked_idx[:kc]
            kp = pv.index_select(0, kept)
        if int(kept.numel()) == 0:
            continue
        kc = int(min(width, int(kept.numel())))
        ks, kept, kp = ks[:kc], kept[:kc], kp[:kc]
        alpha = torch.softmax(ks / float(temperature), dim=-1)[:kc]
        sel_values[h, :kc] = all_values.index_select(0, kept)
        sel_blocks[h, :kc] = all_bi.index_select(0, kept)
        sel_cells[h, :kc] = all_ci.index_select(0, kept)
        sel_alphas[h, :kc] = alpha
        log_alpha[h, :kc] = torch.log(alpha.clamp_min(1e-8))
        counts_sel[h] = float(kc)
        if kc > 1:
            ac = alpha.clamp_min(1e-8)
            entropy[h] = -(ac * ac.log()).sum() / math.log(float(kc))
            margin[h] = ks[0] - ks[1]
        signif[h] = (-torch.log10(kp.clamp_min(1e-12))).mean()
        mass.index_put_((sel_blocks[h, :kc], sel_cells[h, :kc]), alpha, accumulate=True)
    used = counts_sel.gt(0)
    if not bool(used.any()):
        return None
    mean_ent, mean_sig = entropy[used].mean(), signif[used].mean()              # modeling.py:870-895
    ent_conf = torch.clamp((float(entropy_high) - mean_ent) / max(1e-6, float(entropy_high - entropy_low)),
                           min=0.0, max=1.0)
    sig_conf = torch.clamp(mean_sig / 3.0, min=0.0, max=1.0)
    conf = ent_conf * sig_conf
    gm = torch.tensor(float(gamma_m), dtype=torch.float32)
    gr = torch.tensor(float(gamma_r), dtype=torch.float32)
    scale = math.sqrt(float(dv))
    out_scores = []
    for bi, blk in enumerate(blocks):                                             # modeling.py:904-962
        cid = torch.as_tensor(np.asarray(blk["cell_ids"])).to(torch.long)
        if int(cid.numel()) == 0:
            out_scores.append(None)
            continue
        safe = cid.clamp(0, max(0, int(cells_per_block) - 1))
        gathered = mass[bi].index_select(0, safe.reshape(-1)).reshape_as(safe)
        wq = torch.as_tensor(np.asarray(blk["weights_q"])).to(torch.float32)
        token_mass = (gathered.to(torch.float32) * (wq / WEIGHT_QUANT_SCALE)).sum(dim=-1)
        base = torch.as_tensor(np.asarray(blk["base_scores"], np.float32))
        feats = torch.as_tensor(np.asarray(blk["features"], np.float32))
        chunks = []
        for c0 in range(0, int(feats.shape[0]), int(recall_chunk_size)):
            seed = torch.einsum("thd,hkd->thk", feats[c0:c0 + recall_chunk_size], sel_values) / float(scale)
            chunks.append(torch.logsumexp(seed + log_alpha.unsqueeze(0), dim=(1, 2)))
        recall = torch.cat(chunks)
        out_scores.append((base + (gm * conf) * token_mass + (gr * conf) * recall).numpy())
    diag = {"selected_block_slots": sel_blocks.numpy(), "selected_cell_ids": sel_cells.numpy(),
            "selected_alphas": sel_alphas.numpy(), "selection_entropy": entropy.numpy(),
            "selection_margin": margin.numpy(), "confidence": float(conf), "selected_cells_per_head": counts_sel.numpy()}
    return out_scores, diag
