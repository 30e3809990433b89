"""Parity of block commit, coarse top-k and exact readout kernels against the
CPU oracle, through the C ABI.

Bar: commit summaries bit-exact (same fp32 token-order sum and rounding);
selected block indices and exact-token argmax bit-exact wherever the oracle's
margin to the runner-up exceeds 1e-3 relative; readout values exact copies;
scores within 1e-5 relative (fp32 accumulation order only).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import _native, memory, readout, retrieval, workloads as wl
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16]


def _np(t):
    return t.detach().to("cpu", torch.float32).numpy()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("L,d,dv", [(16, 64, 64), (64, 128, 128), (7, 24, 40), (128, 128, 64)])
def test_block_commit_mean_bit_exact(cuda_device, dtype, L, d, dv):
    S, n_slots = 9, 5
    g = torch.Generator().manual_seed(L * d)
    K = torch.randn((S, L, d), generator=g).to(dtype)
    V = torch.randn((S, L, dv), generator=g).to(dtype)
    mem = memory.BlockMemory(S, n_slots, L, d, dv, dtype=dtype, device=cuda_device)
    for _ in range(3):
        mem.commit(K.to(cuda_device), V.to(cuda_device))
    slot = 2
    assert torch.equal(mem.pool_K[:, slot].cpu(), K)
    assert torch.equal(mem.pool_V[:, slot].cpu(), V)
    ref = go.block_commit_mean(_np(K), bf16=dtype == torch.bfloat16)
    assert np.array_equal(_np(mem.summary[:, slot]), ref)
    assert mem.state_version == 3 and mem.next_slot() == 3
    # untouched slots stay zero
    assert torch.count_nonzero(mem.pool_K[:, 4]).item() == 0


def test_block_commit_ring_wraps(cuda_device):
    mem = memory.BlockMemory(2, 3, 4, 8, dtype=torch.float32, device=cuda_device)
    for b in range(5):
        K = torch.full((2, 4, 8), float(b), device=cuda_device)
        mem.commit(K, K)
    assert mem.slot_block_index().tolist() == [3, 4, 2]
    assert mem.summary[:, 0, 0].tolist() == [3.0, 3.0]


def _check_topk(scores, idx, Q, Ksum, k):
    ref_s, ref_i, ok = go.block_topk(_np(Q), _np(Ksum), k)
    got_i = idx.cpu().numpy()
    got_s = scores.cpu().numpy()
    assert ok.mean() > 0.5 or ref_i.shape[-1] >= Ksum.shape[1]  # the cases are not degenerate
    assert np.array_equal(got_i[ok], ref_i[ok])
    fin = np.isfinite(ref_s)
    np.testing.assert_allclose(got_s[fin & ok[..., None]], ref_s[fin & ok[..., None]], rtol=1e-5, atol=1e-5)
    assert np.array_equal(fin, np.isfinite(got_s))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("S,Nq,NB,d,k", [(4, 64, 16, 64, 2), (3, 200, 64, 128, 4), (2, 130, 512, 128, 16),
                                          (1, 1, 5, 32, 8), (2, 17, 33, 96, 32)])
def test_block_topk_matches_oracle(cuda_device, dtype, S, Nq, NB, d, k):
    g = torch.Generator().manual_seed(S * Nq + NB)
    Q = torch.randn((S, Nq, d), generator=g).to(dtype)
    Ksum = torch.randn((S, NB, d), generator=g).to(dtype)
    scores, idx = retrieval.block_topk(Q.to(cuda_device), Ksum.to(cuda_device), k)
    _check_topk(scores, idx, Q, Ksum, k)


@pytest.mark.parametrize("S,Nq,NB,d,k", [(2, 300, 1000, 128, 8), (3, 64, 512, 128, 16), (1, 129, 257, 64, 4),
                                          (2, 40, 130, 256, 32), (2, 77, 300, 96, 8), (1, 5, 3, 200, 4),
                                          (2, 128, 0, 128, 2), (1, 200, 2100, 128, 8), (2, 64, 4096, 64, 32),
                                          (1, 130, 3000, 256, 16)])
def test_block_topk_tensor_core_tiles(cuda_device, S, Nq, NB, d, k):
    # bf16 memories run the tcgen05 pipeline: partial query and block tiles,
    # K boxes padded by the tensor map, more than two accumulator rounds
    g = torch.Generator().manual_seed(NB * 7 + d)
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    Ksum = torch.randn((S, max(NB, 1), d), generator=g).to(torch.bfloat16)
    scores, idx = retrieval.block_topk(Q.to(cuda_device), Ksum.to(cuda_device), k, n_blocks=NB)
    if NB == 0:
        assert (idx == -1).all() and torch.isinf(scores).all()
    else:
        _check_topk(scores, idx, Q, Ksum[:, :NB], k)
    from gfst_hmb_public_b200 import _native
    assert _native.load().gfst_check_device_errors(1) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_block_topk_ties_pick_lowest_index(cuda_device, dtype):
    Ksum = torch.zeros((1, 300, 8))
    Ksum[0, [200, 5, 130], 0] = 1.0  # three equal best scores, across tiles
    Q = torch.zeros((1, 1, 8))
    Q[0, 0, 0] = 1.0
    scores, idx = retrieval.block_topk(Q.to(dtype).to(cuda_device), Ksum.to(dtype).to(cuda_device), 4)
    assert idx.cpu().tolist() == [[[5, 130, 200, 0]]]


def test_block_topk_ties_across_column_parts(cuda_device):
    # long rows split each tile's columns over two epilogue warps: equal best
    # scores in both parts and in far-apart tiles still come out lowest index first
    Ksum = torch.zeros((1, 2500, 64))
    Ksum[0, [2300, 1000, 64, 30], 0] = 1.0
    Ksum[0, 1500, 0] = 0.5
    Q = torch.zeros((1, 3, 64))
    Q[0, :, 0] = 1.0
    scores, idx = retrieval.block_topk(Q.to(torch.bfloat16).to(cuda_device), Ksum.to(torch.bfloat16).to(cuda_device), 6)
    assert idx.cpu().tolist() == [[[30, 64, 1000, 2300, 1500, 0]] * 3]
    assert scores.cpu()[0, 0, :5].tolist() == [1.0, 1.0, 1.0, 1.0, 0.5]


def test_block_topk_partial_bank(cuda_device):
    Q = torch.randn((2, 3, 16), device=cuda_device)
    Ksum = torch.randn((2, 8, 16), device=cuda_device)
    scores, idx = retrieval.block_topk(Q, Ksum, 6, n_blocks=4)
    assert (idx[..., 4:] == -1).all() and torch.isinf(scores[..., 4:]).all()
    assert (idx[..., :4] >= 0).all() and (idx[..., :4] < 4).all()


def test_retriever_matches_exact_oracle_on_small_bank(cuda_device):
    # the small bank of tests/test_retrieval.py:14-52 in the reference
    keys = torch.tensor([[1.0, 0.0, 0.0, 0.0], [0.0, 1.0, 0.0, 0.0], [0.5, 0.5, 0.0, 0.0],
                         [0.0, 0.0, 1.0, 0.0], [0.0, 0.0, 0.0, 1.0], [0.8, 0.2, 0.0, 0.0]], device=cuda_device)
    query = torch.tensor([1.0, 0.0, 0.0, 0.0], device=cuda_device)

    class State:
        state_version = 0

    state = State()
    r = retrieval.BlockRetriever()
    indices, scores = r.search(state=state, layer_idx=0, batch_idx=0, keys_tensor=keys, query_tensor=query, top_k=3)
    assert indices.tolist() == [0, 5, 2]
    assert torch.allclose(scores.cpu(), torch.tensor([1.0, 0.8, 0.5]), atol=1e-5)
    assert r._index_cache[(id(state), 0, 0)].device_index == 0
    before = r._index_cache[(id(state), 0, 0)].state_version
    state.state_version += 1
    r.search(state=state, layer_idx=0, batch_idx=0, keys_tensor=keys, query_tensor=query, top_k=2)
    assert r._index_cache[(id(state), 0, 0)].state_version > before
    empty_i, empty_s = r.search(state=state, layer_idx=0, batch_idx=0, keys_tensor=keys[:0], query_tensor=query,
                                top_k=2)
    assert empty_i.numel() == 0 and empty_s.numel() == 0


def test_retriever_rejects_cpu_and_wrong_device(cuda_device):
    r = retrieval.BlockRetriever()

    class State:
        state_version = 0

    with pytest.raises(RuntimeError):
        r.search(state=State(), layer_idx=0, batch_idx=0, keys_tensor=torch.eye(4), query_tensor=torch.ones(4),
                 top_k=2)
    if torch.cuda.device_count() > 1:
        with pytest.raises(RuntimeError):
            r.search(state=State(), layer_idx=0, batch_idx=0, keys_tensor=torch.eye(4, device="cuda:1"),
                     query_tensor=torch.ones(4, device="cuda:1"), top_k=2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("S,Nq,NS,L,d,dv,k", [(3, 40, 16, 16, 64, 64, 2), (2, 33, 64, 64, 128, 128, 4),
                                               (2, 9, 9, 128, 128, 64, 8), (1, 5, 4, 5, 16, 24, 3),
                                               (2, 70, 12, 32, 256, 64, 5), (1, 12, 7, 24, 128, 32, 3)])
def test_exact_readout_matches_oracle(cuda_device, dtype, S, Nq, NS, L, d, dv, k):
    g = torch.Generator().manual_seed(S * 100 + Nq)
    pool_K = torch.randn((S, NS, L, d), generator=g).to(dtype)
    pool_V = torch.randn((S, NS, L, dv), generator=g).to(dtype)
    Q = torch.randn((S, Nq, d), generator=g).to(dtype)
    sel = torch.stack([torch.stack([torch.randperm(NS, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    sel = sel.to(torch.int32)
    sel[0, 0, -1] = -1  # a skipped entry
    best_tok, best_score, out_V = readout.exact_readout(Q.to(cuda_device), pool_K.to(cuda_device),
                                                        pool_V.to(cuda_device), sel.to(cuda_device))
    ref_tok, ref_score, ref_V, ok = go.exact_readout(_np(Q), _np(pool_K), _np(pool_V), sel.numpy())
    got_tok = best_tok.cpu().numpy()
    assert ok.mean() > 0.5
    assert np.array_equal(got_tok[ok], ref_tok[ok])
    np.testing.assert_allclose(best_score.cpu().numpy()[ok], ref_score[ok], rtol=1e-5, atol=1e-5)
    assert np.array_equal(_np(out_V)[ok], ref_V[ok])


@pytest.mark.parametrize("dtype", DTYPES)
def test_exact_readout_grouped_chunks_and_duplicates(cuda_device, dtype):
    # 150 queries per stream -> three query chunks (the last partial); some
    # queries list the same block twice, some list out-of-range slots
    S, Nq, NS, L, d, k = 3, 150, 40, 64, 128, 6
    g = torch.Generator().manual_seed(21)
    pool_K = torch.randn((S, NS, L, d), generator=g).to(dtype)
    pool_V = torch.randn((S, NS, L, d), generator=g).to(dtype)
    Q = torch.randn((S, Nq, d), generator=g).to(dtype)
    sel = torch.randint(0, NS, (S, Nq, k), generator=g, dtype=torch.int32)
    sel[:, ::7, 1] = sel[:, ::7, 0]
    sel[:, ::11, 2] = NS + 3
    sel[1, 5, :] = -1
    tok, score, val = readout.exact_readout(Q.to(cuda_device), pool_K.to(cuda_device), pool_V.to(cuda_device),
                                            sel.to(cuda_device))
    ref_tok, ref_score, ref_V, ok = go.exact_readout(_np(Q), _np(pool_K), _np(pool_V),
                                                     np.where(sel.numpy() < NS, sel.numpy(), -1))
    got = tok.cpu().numpy()
    assert got[1, 5] == -1 and ref_tok[1, 5] == -1
    assert np.array_equal(got[ok], ref_tok[ok])
    np.testing.assert_allclose(score.cpu().numpy()[ok], ref_score[ok], rtol=1e-5, atol=1e-5)
    assert np.array_equal(_np(val)[ok], ref_V[ok])


@pytest.mark.parametrize("pattern", ["spread", "shared"])
def test_exact_readout_stage_ring_wraps(cuda_device, pattern):
    # 64 queries x k=32 selections per chunk: with 8 KB blocks the staging ring
    # (8 stages) wraps dozens of times ("spread": ~280 distinct blocks), or
    # every query of the chunk reads the same 32 blocks ("shared": 64 queries
    # per staged block)
    S, Nq, NS, L, d, k = 2, 64, 300, 32, 128, 32
    g = torch.Generator().manual_seed(5)
    pool_K = torch.randn((S, NS, L, d), generator=g).to(torch.bfloat16)
    pool_V = torch.randn((S, NS, L, d), generator=g).to(torch.bfloat16)
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    if pattern == "spread":
        sel = torch.stack([torch.stack([torch.randperm(NS, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    else:
        sel = torch.randperm(NS, generator=g)[:k].expand(S, Nq, k).clone()
    sel = sel.to(torch.int32)
    tok, score, val = readout.exact_readout(Q.to(cuda_device), pool_K.to(cuda_device), pool_V.to(cuda_device),
                                            sel.to(cuda_device))
    ref_tok, ref_score, ref_V, ok = go.exact_readout(_np(Q), _np(pool_K), _np(pool_V), sel.numpy())
    assert ok.mean() > 0.9
    assert np.array_equal(tok.cpu().numpy()[ok], ref_tok[ok])
    np.testing.assert_allclose(score.cpu().numpy()[ok], ref_score[ok], rtol=1e-5, atol=1e-5)
    assert np.array_equal(_np(val)[ok], ref_V[ok])
    assert _native.load().gfst_check_device_errors(1) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_exact_readout_ties_pick_lowest_token(cuda_device, dtype):
    # the same key at tokens 67 (block 4), 32 (block 2) and 25 (block 1)
    S, NS, L, d = 1, 6, 16, 64
    g = torch.Generator().manual_seed(9)
    pool = (0.1 * torch.randn((S, NS, L, d), generator=g)).to(dtype)
    v = torch.randn(d, generator=g).to(dtype)
    for b, p in ((4, 3), (2, 0), (1, 9)):
        pool[0, b, p] = v
    Q = v.reshape(1, 1, d).clone()
    sel = torch.tensor([[[4, 2, 1, 5]]], dtype=torch.int32)
    tok, score, val = readout.exact_readout(Q.to(cuda_device), pool.to(cuda_device), pool.to(cuda_device),
                                            sel.to(cuda_device))
    assert tok.item() == 25
    assert torch.equal(val.cpu()[0, 0], v)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("d", [64, 24])
def test_exact_readout_nan_scores_never_win(cuda_device, dtype, d):
    # block 1: every token scores NaN; block 2: one NaN token.  A query that
    # selected only NaN tokens has no winner (-1, -inf, zero value row).
    S, NS, L = 1, 4, 16
    g = torch.Generator().manual_seed(13)
    pool = torch.randn((S, NS, L, d), generator=g)
    pool[0, 1, :, 0] = float("nan")
    pool[0, 2, 5, 3] = float("nan")
    pool = pool.to(dtype)
    Q = torch.randn((S, 3, d), generator=g).to(dtype)
    sel = torch.tensor([[[1, 1], [1, 2], [2, 3]]], dtype=torch.int32)
    tok, score, val = readout.exact_readout(Q.to(cuda_device), pool.to(cuda_device), pool.to(cuda_device),
                                            sel.to(cuda_device))
    ref_tok, ref_score, ref_V, ok = go.exact_readout(_np(Q), _np(pool), _np(pool), sel.numpy())
    assert ref_tok[0, 0] == -1 and tok[0, 0].item() == -1
    assert torch.isinf(score[0, 0]).item() and (val[0, 0] == 0).all().item()
    assert np.array_equal(tok.cpu().numpy()[ok], ref_tok[ok])
    assert not np.isnan(score.cpu().numpy()).any()


def test_exact_readout_no_valid_block(cuda_device):
    pool = torch.randn((1, 4, 8, 16), device=cuda_device)
    sel = torch.full((1, 2, 3), -1, dtype=torch.int32, device=cuda_device)
    tok, score, v = readout.exact_readout(torch.randn(1, 2, 16, device=cuda_device), pool, pool, sel)
    assert tok.tolist() == [[-1, -1]] and torch.isinf(score).all() and (v == 0).all()


def test_needle_queries_recover_the_needle(cuda_device):
    # long-memory readout in miniature: query = key[needle] + N(0, 0.1^2)
    S, NB, L, d, Nq, k = 4, 256, 128, 128, 64, 8
    g = torch.Generator().manual_seed(77)
    pool_K = torch.randn((S, NB, L, d), generator=g).to(torch.bfloat16)
    needles = torch.randint(0, NB * L, (S, Nq), generator=g)
    keys_flat = pool_K.reshape(S, NB * L, d).float()
    Q = (keys_flat[torch.arange(S)[:, None], needles] + 0.1 * torch.randn((S, Nq, d), generator=g)).to(torch.bfloat16)
    mem_summary = torch.from_numpy(go.block_commit_mean(_np(pool_K), bf16=True)).to(torch.bfloat16)
    scores, idx = retrieval.block_topk(Q.to(cuda_device), mem_summary.to(cuda_device), k)
    tok, _, _ = readout.exact_readout(Q.to(cuda_device), pool_K.to(cuda_device), None, idx)
    ref_s, ref_i, ok = go.block_topk(_np(Q), _np(mem_summary), k)
    got_i = idx.cpu().numpy()
    assert np.array_equal(got_i[ok], ref_i[ok])
    ref_tok, _, _, ok2 = go.exact_readout(_np(Q), _np(pool_K), None, got_i)
    assert np.array_equal(tok.cpu().numpy()[ok2], ref_tok[ok2])


def _collapse_margin_ok(Q, pool_K, ids, sel, tol=1e-4):
    """Queries whose best two token-id groups differ by more than tol (relative)."""
    S, Nq = sel.shape[:2]
    ok = np.ones((S, Nq), bool)
    L = pool_K.shape[2]
    for s in range(S):
        for q in range(Nq):
            blocks = []
            for b in sel[s, q]:
                if 0 <= int(b) < pool_K.shape[1] and int(b) not in blocks:
                    blocks.append(int(b))
            if not blocks:
                continue
            keys = np.concatenate([pool_K[s, b] for b in blocks]).astype(np.float64)
            sc = keys @ Q[s, q].astype(np.float64)
            tid = np.concatenate([ids[s, b] for b in blocks])
            keep = (tid >= 0) & ~np.isnan(sc)
            groups = {}
            for t, v in zip(tid[keep], sc[keep]):
                groups.setdefault(int(t), []).append(v)
            g = sorted((np.log(np.sum(np.exp(np.array(v) - max(v)))) + max(v) for v in groups.values()), reverse=True)
            if len(g) > 1:
                ok[s, q] = abs(g[0] - g[1]) > tol * max(abs(g[0]), 1.0)
    return ok


@pytest.mark.parametrize("dtype", DTYPES)
def test_readout_collapse_matches_reference(cuda_device, dtype):
    z = np.load(Path(__file__).resolve().parent / "golden" / "readout_collapse_e2e.npz")
    Q = torch.from_numpy(z["Q"]).to(dtype)
    pool = torch.from_numpy(z["pool_K"]).to(dtype)
    got = readout.exact_readout_collapse(Q.to(cuda_device), pool.to(cuda_device),
                                         torch.from_numpy(z["token_ids"]).to(cuda_device),
                                         torch.from_numpy(z["top_idx"]).to(cuda_device))
    if dtype == torch.float32:
        ref = [z[k] for k in ("best_id", "best_score", "best_block", "best_pos")]
    else:  # the reference on the bf16-rounded inputs
        ref = go.exact_readout_collapse(_np(Q), _np(pool), z["token_ids"], z["top_idx"])
    ok = _collapse_margin_ok(_np(Q), _np(pool), z["token_ids"], z["top_idx"])
    assert ok.mean() > 0.8
    for g_t, r_t in zip((got[0], got[2], got[3]), (ref[0], ref[2], ref[3])):
        assert np.array_equal(g_t.cpu().numpy()[ok], r_t[ok])
    np.testing.assert_allclose(got[1].cpu().numpy(), ref[1], rtol=1e-5, atol=1e-5)


def test_readout_collapse_edge_cases(cuda_device):
    # duplicate ids within and across blocks, padding ids, a NaN key, a block
    # listed twice, an out-of-range selection, and a query with nothing valid
    g = torch.Generator().manual_seed(6)
    S, NS, L, d, Nq, k = 2, 12, 8, 16, 5, 4
    pool = torch.randn((S, NS, L, d), generator=g)
    ids = torch.randint(0, 6, (S, NS, L), generator=g, dtype=torch.int32)
    ids[0, 3, :4] = -1
    pool[1, 2, 5, 0] = float("nan")
    Q = torch.randn((S, Nq, d), generator=g)
    sel = torch.randint(0, NS, (S, Nq, k), generator=g, dtype=torch.int32)
    sel[0, 1, 2] = sel[0, 1, 0]
    sel[1, 3, 1] = NS + 4
    sel[0, 4, :] = -1
    got = readout.exact_readout_collapse(Q.to(cuda_device), pool.to(cuda_device), ids.to(cuda_device),
                                         sel.to(cuda_device))
    ref = go.exact_readout_collapse(Q.numpy(), pool.numpy(), ids.numpy(), sel.numpy())
    ok = _collapse_margin_ok(Q.numpy(), pool.numpy(), ids.numpy(), sel.numpy())
    for g_t, r_t in zip((got[0], got[2], got[3]), (ref[0], ref[2], ref[3])):
        assert np.array_equal(g_t.cpu().numpy()[ok], r_t[ok])
    assert got[0][0, 4].item() == -1 and got[2][0, 4].item() == -1
    assert torch.isinf(got[1][0, 4]).item()


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64, torch.uint8, torch.bfloat16])
def test_exact_block_materialize_slices(cuda_device, dtype):
    g = torch.Generator().manual_seed(11)
    packed = torch.randint(0, 120, (1000,), generator=g).to(dtype)
    dev = packed.to(cuda_device)
    for start, end in [(0, 1000), (0, 0), (7, 7), (3, 250), (128, 512), (999, 1000), (1, 998)]:
        got = memory.exact_block_materialize(dev, start, end)
        assert got.dtype == dtype and torch.equal(got.cpu(), packed[start:end])
    for start, end in [(-1, 3), (5, 4), (0, 1001)]:
        with pytest.raises(RuntimeError):
            memory.exact_block_materialize(dev, start, end)
    with pytest.raises(RuntimeError):
        memory.exact_block_materialize(dev.view(10, 100), 0, 5)
