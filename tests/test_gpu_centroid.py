"""Centroid path kernels (cell write, significance-gated readout) against the
golden vectors of the reference's own state / readout code and the oracle.

Bar: the cell write is bit-exact (integer quantisation and fp16 means of IEEE
fp32 sums in the reference's order).  The readout's float work (dot products,
medians of those, erf / exp / log) rounds differently from torch's CPU kernels,
so final token scores match to 1e-4 absolute, softmax weights and confidence to
1e-5, and the selected cells and the best token exactly wherever the decision
margin exceeds 1e-3.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import centroid
from oracle import centroid_oracle as co
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
SCORE_TOL = 1e-4


def _golden():
    return np.load(GOLDEN / "centroid_path.npz")


def test_cell_commit_matches_reference_golden(cuda_device):
    z = _golden()
    C = int(z["dims"][3])
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device, dt)  # noqa: E731
    ids, wq, keys, vals, cnt = centroid.centroid_cell_commit(t(z["cell_ids_in"], torch.int32), t(z["cell_weights_in"]),
                                                             t(z["cell_keys_in"]), t(z["cell_values_in"]), C)
    assert np.array_equal(ids.cpu().numpy(), z["token_cell_ids"])
    assert np.array_equal(wq.cpu().numpy(), z["token_cell_weights_q"])
    assert np.array_equal(keys.cpu().numpy().view(np.uint16), z["cell_keys"].view(np.uint16))
    assert np.array_equal(vals.cpu().numpy(), z["cell_values_q"])
    assert np.array_equal(cnt.cpu().numpy(), z["cell_counts"])


def test_cell_commit_random_blocks_bit_exact(cuda_device):
    g = np.random.default_rng(3)
    B, L, W, C, dk, dv = 37, 24, 3, 12, 10, 7
    ids = g.integers(-2, C + 3, (B, L, W)).astype(np.int32)
    ids[:, :, 2] = ids[:, :, 0]                      # the same cell twice in one token
    w = g.random((B, L, W)).astype(np.float32)
    w[g.random((B, L, W)) < 0.2] = 0.0
    w[0, 0, 0] = 1.7                                 # clamps to 255
    w[1, 3, 1] = 0.5 / 255.0                         # round half to even
    keys = (g.standard_normal((B, L, dk)) * 3).astype(np.float32)
    vals = (g.standard_normal((B, L, dv)) * 3).astype(np.float32)
    out = centroid.centroid_cell_commit(*(torch.from_numpy(a).to(cuda_device) for a in (ids, w, keys, vals)), C)
    for b in range(B):
        ref = co.cell_commit(ids[b], w[b], keys[b], vals[b], C)
        for got, want in zip(out, ref):
            got = got[b].cpu().numpy()
            if want.dtype == np.float16:
                got, want = got.view(np.uint16), want.view(np.uint16)
            assert np.array_equal(got, want), b


def _golden_store(z, dev):
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).unsqueeze(0).to(dev, dt)  # noqa: E731
    return dict(token_keys=t(z["token_keys"]), token_features=t(z["token_features"]),
                token_ids=t(z["token_ids"], torch.int32), token_cell_ids=t(z["token_cell_ids"]),
                token_cell_weights_q=t(z["token_cell_weights_q"]), cell_keys=t(z["cell_keys"]),
                cell_values_q=t(z["cell_values_q"]), cell_counts=t(z["cell_counts"]))


def test_centroid_readout_matches_reference_golden(cuda_device):
    z = _golden()
    n = int(z["n_cases"])
    K = max(len(z[f"q{ci}_blocks"]) for ci in range(n)) + 1   # one padding selection per row
    L = int(z["dims"][4])
    sel = np.full((1, n, K), -1, np.int32)
    scores = np.zeros((1, n, K), np.float32)
    prefix = np.zeros((1, n, K), np.int32)
    qh = np.stack([z[f"q{ci}_query_heads"] for ci in range(n)])[None]
    for ci in range(n):
        b = z[f"q{ci}_blocks"]
        sel[0, ci, :len(b)] = b
        scores[0, ci, :len(b)] = z[f"q{ci}_block_scores"]
        prefix[0, ci, :len(b)] = z[f"q{ci}_prefixes"]
    dev = cuda_device
    out = centroid.centroid_readout(
        torch.from_numpy(z["queries"][None]).to(dev), torch.from_numpy(qh).to(dev), torch.from_numpy(sel).to(dev),
        torch.from_numpy(scores).to(dev), prefix_len=torch.from_numpy(prefix).to(dev),
        params=centroid.CentroidParams(top_cells_per_head=5, min_selected=2), return_candidates=True,
        return_diagnostics=True, **_golden_store(z, dev))
    cand = out.candidate_scores.cpu().numpy()[0]
    for ci in range(n):
        nb = len(z[f"q{ci}_blocks"])
        got = np.concatenate([cand[ci, k, :z[f"q{ci}_prefixes"][k]] for k in range(nb)])
        want = z[f"q{ci}_scores"]
        assert np.abs(got - want).max() <= SCORE_TOL, ci
        assert np.array_equal(out.selected_block.cpu().numpy()[0, ci], z[f"q{ci}_selected_block_slots"]), ci
        assert np.array_equal(out.selected_cell.cpu().numpy()[0, ci], z[f"q{ci}_selected_cell_ids"]), ci
        assert np.abs(out.selected_alpha.cpu().numpy()[0, ci] - z[f"q{ci}_selected_alphas"]).max() <= 1e-5, ci
        hs = out.head_stats.cpu().numpy()[0, ci]
        assert np.abs(hs[:, 0] - z[f"q{ci}_selection_entropy"]).max() <= 1e-5, ci
        assert np.array_equal(hs[:, 2], z[f"q{ci}_selected_cells_per_head"]), ci
        assert abs(float(out.confidence[0, ci]) - float(z[f"q{ci}_confidence"])) <= 1e-5, ci
        assert np.all(cand[ci, nb:] == -np.inf)
        # best token: the reference's collapse + best group on its own scores
        uid, gs, gb, gp = go.collapse_logsumexp(want, z[f"q{ci}_token_ids"], np.repeat(
            z[f"q{ci}_blocks"], z[f"q{ci}_prefixes"]), z[f"q{ci}_positions"])
        order = np.lexsort((uid, -gs))
        w = order[0]
        if len(order) == 1 or gs[order[0]] - gs[order[1]] > 1e-3:
            assert int(out.best_id[0, ci]) == int(uid[w]), ci
            assert int(out.best_block[0, ci]) == int(gb[w]) and int(out.best_pos[0, ci]) == int(gp[w]), ci
        assert abs(float(out.best_score[0, ci]) - float(gs[w])) <= SCORE_TOL, ci


def _random_store(g, S, NB, L, W, C, dq, H, dk, dv, vocab, dev):
    ids = g.integers(0, C, (S, NB, L, W)).astype(np.int32)
    w = g.random((S, NB, L, W)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    ck = g.standard_normal((S, NB, L, dk)).astype(np.float32)
    dirs = g.standard_normal((C, dk)).astype(np.float32)
    ck += 2.0 * dirs[ids[..., 0]]
    cv = (g.standard_normal((S, NB, L, dv)) * 2).astype(np.float32)
    tid, twq, keys, vals, cnt = centroid.centroid_cell_commit(*(torch.from_numpy(a).to(dev) for a in (ids, w, ck, cv)),
                                                              C)
    store = dict(token_keys=torch.from_numpy(g.standard_normal((S, NB, L, dq)).astype(np.float32)).to(dev),
                 token_features=torch.from_numpy(g.standard_normal((S, NB, L, H, dv)).astype(np.float32)).to(dev),
                 token_ids=torch.from_numpy(g.integers(0, vocab, (S, NB, L)).astype(np.int32)).to(dev),
                 token_cell_ids=tid, token_cell_weights_q=twq, cell_keys=keys, cell_values_q=vals, cell_counts=cnt)
    return store, dirs


def _oracle_query(store, s, qv, qh, sel, scores, prefix, prm, C):
    np_ = {k: v[s].cpu().numpy() for k, v in store.items()}
    ents = []
    for b, sc, p in zip(sel, scores, prefix):
        if b < 0 or p <= 0:
            continue
        ents.append(dict(token_ids=np_["token_ids"][b][:p], cell_ids=np_["token_cell_ids"][b][:p],
                         weights_q=np_["token_cell_weights_q"][b][:p], cell_keys=np_["cell_keys"][b],
                         cell_values_q=np_["cell_values_q"][b], cell_counts=np_["cell_counts"][b],
                         base_scores=(np_["token_keys"][b][:p].astype(np.float64) @ qv).astype(np.float32),
                         features=np_["token_features"][b][:p], block_score=float(sc), block=b))
    res = co.centroid_candidates(qh, ents, top_cells_per_head=prm.top_cells_per_head, min_selected=prm.min_selected,
                                 cells_per_block=C, fdr_q=prm.fdr_q, block_score_lambda=prm.block_score_lambda,
                                 background_subtract=prm.background_subtract, count_penalty=prm.count_penalty,
                                 self_field_weight=prm.self_field_weight, temperature=prm.temperature,
                                 entropy_low=prm.entropy_low, entropy_high=prm.entropy_high, gamma_m=prm.gamma_m,
                                 gamma_r=prm.gamma_r)
    return ents, res


ALT_PARAMS = centroid.CentroidParams(top_cells_per_head=6, min_selected=3, fdr_q=0.3, background_subtract=False,
                                     count_penalty=0.3, self_field_weight=0.0, temperature=0.7, block_score_lambda=0.5,
                                     entropy_low=0.2, entropy_high=0.9, gamma_m=0.5, gamma_r=2.0)


@pytest.mark.parametrize("dq,H,dv,alt", [(24, 4, 6, False), (32, 4, 16, False), (128, 2, 16, False),
                                         (32, 4, 16, True)])
def test_centroid_readout_random_against_oracle(cuda_device, dq, H, dv, alt):
    # (32, 4, 16): the two-threads-per-token path for the reference's default
    # 4 heads x 16 value dims; the others the warp-per-token path; alt: no
    # background subtraction and other weights / gains
    g = np.random.default_rng(11 + dq + H)
    S, Nq, NB, L, W, C, dk, K = 2, 12, 20, 16, 2, 8, 8, 6
    dev = cuda_device
    store, dirs = _random_store(g, S, NB, L, W, C, dq, H, dk, dv, 60, dev)
    Q = g.standard_normal((S, Nq, dq)).astype(np.float32)
    qh = g.standard_normal((S, Nq, H, dk)).astype(np.float32)
    qh[:, ::2, 0] = 2.0 * dirs[g.integers(0, C, (S, Nq // 2))]   # some heads point at a cell direction
    sel = np.stack([np.stack([g.permutation(NB)[:K] for _ in range(Nq)]) for _ in range(S)]).astype(np.int32)
    sel[0, 3, 2] = -1
    scores = g.standard_normal((S, Nq, K)).astype(np.float32)
    prefix = np.full((S, Nq, K), L, np.int32)
    prefix[1, 5, 0] = 9
    prm = ALT_PARAMS if alt else centroid.CentroidParams(top_cells_per_head=6, min_selected=2, fdr_q=0.2)
    out = centroid.centroid_readout(torch.from_numpy(Q).to(dev), torch.from_numpy(qh).to(dev),
                                    torch.from_numpy(sel).to(dev), torch.from_numpy(scores).to(dev),
                                    prefix_len=torch.from_numpy(prefix).to(dev), params=prm,
                                    return_candidates=True, return_diagnostics=True, **store)
    cand = out.candidate_scores.cpu().numpy()
    conf = out.confidence.cpu().numpy()
    n_on = 0
    for s in range(S):
        for q in range(Nq):
            ents, res = _oracle_query(store, s, Q[s, q].astype(np.float64), qh[s, q], sel[s, q], scores[s, q],
                                      prefix[s, q], prm, C)
            ks = [k for k in range(K) if sel[s, q, k] >= 0 and prefix[s, q, k] > 0]
            got = np.concatenate([cand[s, q, k, :prefix[s, q, k]] for k in ks])
            if res is None:
                want = np.concatenate([e["base_scores"] for e in ents])
                assert conf[s, q] == -1.0
            else:
                sc, diag = res
                want = np.concatenate(sc)
                n_on += 1
                assert abs(conf[s, q] - diag["confidence"]) <= 1e-5
                assert np.array_equal(out.selected_cell.cpu().numpy()[s, q], diag["selected_cell_ids"])
            assert np.abs(got - want).max() <= SCORE_TOL, (s, q)
    assert n_on >= Nq


def test_centroid_readout_edges(cuda_device):
    g = np.random.default_rng(5)
    S, Nq, NB, L, W, C, dq, H, dk, dv, K = 1, 3, 6, 8, 2, 8, 16, 2, 8, 4, 3
    dev = cuda_device
    store, _ = _random_store(g, S, NB, L, W, C, dq, H, dk, dv, 30, dev)
    store["cell_counts"][0, 2].zero_()                      # block 2 has no cells
    Q = torch.randn((S, Nq, dq), device=dev)
    qh = torch.randn((S, Nq, H, dk), device=dev)
    sel = torch.tensor([[[-1, -1, -1], [2, -1, 2], [1, 40, 3]]], dtype=torch.int32, device=dev)
    sc = torch.zeros((S, Nq, K), device=dev)
    out = centroid.centroid_readout(Q, qh, sel, sc, return_candidates=True, return_diagnostics=True, **store)
    assert int(out.best_id[0, 0]) == -1 and float(out.best_score[0, 0]) == float("-inf")
    assert torch.all(out.candidate_scores[0, 0] == float("-inf"))
    # only the cell-less block: centroid terms off, base scores
    assert float(out.confidence[0, 1]) == -1.0
    base = (store["token_keys"][0, 2] @ Q[0, 1]).cpu().numpy()
    assert np.abs(out.candidate_scores[0, 1, 0].cpu().numpy() - base).max() <= SCORE_TOL
    assert torch.all(out.candidate_scores[0, 1, 1] == float("-inf"))
    # a slot outside the memory is skipped like an unused selection
    assert torch.all(out.candidate_scores[0, 2, 1] == float("-inf"))
    assert int(out.best_block[0, 2]) in (1, 3)


def test_centroid_rejects(cuda_device):
    dev = cuda_device
    S, Nq, NB, L, W, C, dq, H, dk, dv = 1, 1, 2, 4, 1, 4, 8, 2, 4, 4
    store = dict(token_keys=torch.zeros((S, NB, L, dq), device=dev),
                 token_features=torch.zeros((S, NB, L, H, dv), device=dev),
                 token_ids=torch.zeros((S, NB, L), dtype=torch.int32, device=dev),
                 token_cell_ids=torch.zeros((S, NB, L, W), dtype=torch.uint8, device=dev),
                 token_cell_weights_q=torch.zeros((S, NB, L, W), dtype=torch.uint8, device=dev),
                 cell_keys=torch.zeros((S, NB, C, dk), dtype=torch.float16, device=dev),
                 cell_values_q=torch.zeros((S, NB, C, dv), dtype=torch.int8, device=dev),
                 cell_counts=torch.zeros((S, NB, C), dtype=torch.int16, device=dev))
    Q, qh = torch.zeros((S, Nq, dq), device=dev), torch.zeros((S, Nq, H, dk), device=dev)
    sel, sc = torch.zeros((S, Nq, 33), dtype=torch.int32, device=dev), torch.zeros((S, Nq, 33), device=dev)
    with pytest.raises(RuntimeError, match="K=33"):
        centroid.centroid_readout(Q, qh, sel, sc, **store)
    with pytest.raises(RuntimeError, match="temperature"):
        centroid.centroid_readout(Q, qh, sel[..., :2], sc[..., :2], params=centroid.CentroidParams(temperature=0.0),
                                  **store)
    with pytest.raises(RuntimeError):
        centroid.centroid_readout(Q.cpu(), qh, sel[..., :2], sc[..., :2], **store)
