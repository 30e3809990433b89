"""Pin the CPU oracle against golden vectors produced by the reference's own
code (tests/golden/make_golden.py) and the reference tests' known answers."""
from pathlib import Path

import numpy as np
import torch

from oracle import build as oracle_build
from oracle import centroid_oracle as co
from oracle import gfst_oracle as go

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name)


def test_known_answer_candidate():
    z = load("qr_known_answer.npz")
    q = go.qr_reference(z["candidate"][None])[0]
    assert np.array_equal(q, z["canonical_q"])  # same LAPACK call, same sign rule
    # the reference's stepwise Householder and MGS agree with it (to fp32)
    assert np.abs(q - z["householder_signfixed_q"]).max() < 1e-6
    assert np.abs(q - z["mgs_q"]).max() < 1e-6
    assert go.orthogonality_error(q).max() < 1e-5  # tests/...householder_vs_mgs_dataset.py:69-70


def test_sign_problem_families():
    z = load("qr_sign_problem_cases.npz")
    q = go.qr_reference(z["matrices"])
    assert np.array_equal(q, z["canonical_q"])
    c = oracle_build.qr_fixed_order(z["matrices"])
    fam = z["families"]
    # the fixed-order C restatement: leading prefixes are well determined on the
    # benign families; rank-deficient families only pin the leading columns
    benign = np.isin(fam, ["gaussian", "column_scaled"])
    assert go.max_prefix_subspace_distance(c[benign], q[benign]).max() < 1e-4
    assert go.orthogonality_error(c).max() < 1e-5


def test_batched_qr_sample():
    z = load("qr_batched_sample.npz")
    q = go.qr_reference(z["matrices"])
    assert np.array_equal(q, z["canonical_q"])
    c = oracle_build.qr_fixed_order(z["matrices"])
    assert np.abs(c - q).max() < 1e-4
    assert go.max_prefix_subspace_distance(c, q).max() < 1e-4


def test_r_diag_rule_matches_its_definition():
    z = load("qr_batched_sample.npz")
    q = go.qr_reference(z["matrices"], sign_mode=go.SIGN_R_DIAG_POSITIVE)
    r = np.matmul(np.swapaxes(q, -1, -2).astype(np.float64), z["matrices"].astype(np.float64))
    assert (np.diagonal(r, axis1=-2, axis2=-1) > 0).all()
    c = oracle_build.qr_fixed_order(z["matrices"], sign_mode=1)
    assert np.abs(c - q).max() < 1e-4


def test_update_rule_trajectory():
    z = load("update_rule_trajectory.npz")
    U = z["U0"]
    for t in range(z["values"].shape[0]):
        cand = go.residual_rank_one_candidate(U, z["values"][t], float(z["alpha"]))
        assert np.array_equal(cand, z["candidates"][t])
        U = go.qr_reference(cand)
        assert np.array_equal(U, z["frames"][t])


def test_retrieval_exact_topk():
    z = load("retrieval_exact_topk.npz")
    Q = z["queries"][None]
    K = z["keys"][None]
    s, i, ok = go.block_topk(Q, K, 5)
    assert np.array_equal(i[0][ok[0]], z["top_idx"][ok[0]])
    np.testing.assert_allclose(s[0], z["top_scores"], rtol=1e-5, atol=1e-5)
    s2, i2, _ = go.block_topk(z["small_query"][None, None], z["small_keys"][None], 3)
    assert i2[0, 0].tolist() == z["small_idx"].tolist() == [0, 5, 2]


def test_block_commit_mean_definition():
    g = np.random.default_rng(0)
    K = g.standard_normal((3, 16, 8)).astype(np.float32)
    m = go.block_commit_mean(K, bf16=False)
    np.testing.assert_allclose(m, K.mean(axis=1), rtol=1e-6, atol=1e-6)
    mb = go.block_commit_mean(go.to_bf16_f32(K), bf16=True)
    assert np.array_equal(mb, go.to_bf16_f32(mb))


def test_readout_collapse_identity_for_unique_positions():
    z = load("readout_collapse.npz")
    # the reference's selected copy token is the max-score group
    uid, gs = z["unique_ids"], z["grouped_scores"]
    assert int(uid[np.argmax(gs)]) == int(z["selected_token"])
    # with unique token ids the collapse is the identity, so the readout's
    # argmax over positions is the reference's selection
    Q = np.zeros((1, 1, 4), np.float32)
    Q[0, 0, 0] = 1.0
    pool = np.zeros((1, 2, 3, 4), np.float32)
    pool[0, 1, 2, 0] = 2.0
    pool[0, 0, 1, 0] = 2.0  # tie: lower token index (0*3+1) wins
    tok, sc, _, _ = go.exact_readout(Q, pool, None, np.array([[[1, 0]]]))
    assert tok[0, 0] == 1 and sc[0, 0] == 2.0


def _tracker_golden(name):
    z = load(name)
    xs = z["values"]
    fd = [int(v) for v in z["flag_dims"]]
    S, T, d = xs.shape
    r = fd[-1]
    U0 = np.broadcast_to(np.eye(d, r, dtype=np.float32), (S, d, r))
    V0 = [np.broadcast_to(np.eye(r, k, dtype=np.float32), (S, r, k)) for k in fd[:-1]]
    return z, fd, U0, V0


def test_local_tracker_matches_reference_methods():
    # golden: GfstHmbSublayer._update_local_bases + _local_alignment_features
    # (modeling.py:2299-2437) called on the reference's own tracker state
    for name in ("local_tracker_d64.npz", "local_tracker_d128.npz"):
        z, fd, U0, V0 = _tracker_golden(name)
        U, V, feats, snaps = go.local_tracker_stream(U0, V0, z["values"], fd, z["forgetting_rates"],
                                                     float(z["eps"]), float(z["eps_update"]),
                                                     float(z["eps_sign"]), out_every=8)
        assert np.array_equal(U, z["largest_basis"])
        assert np.array_equal(feats, z["features"])
        assert np.array_equal(np.swapaxes(snaps, 0, 1), z["frames_every8"])
        for lvl, dim in enumerate(fd[:-1]):
            assert np.array_equal(V[lvl], z["nested_bases"][:, lvl, :, :dim])
        bases = np.concatenate([U @ V[lvl] for lvl in range(len(fd) - 1)] + [U], axis=-1)
        np.testing.assert_allclose(bases, z["local_bases"], atol=1e-6)


def test_block_commit_eig_matches_reference_replays():
    # golden: replay_block_commit_bundle(..., "native") of the reference on
    # projector sums of real block-tracker passes and on degenerate spectra
    z = load("block_commit_eig_cases.npz")
    for c in range(int(z["n_cases"])):
        meta = z[f"c{c}_meta"]
        b, m, t, a = go.block_commit_eig(z[f"c{c}_projector_sum"], z[f"c{c}_reduced_sum"], int(meta[0]),
                                         int(meta[1]), [int(v) for v in meta[2:]])
        assert np.array_equal(b, z[f"c{c}_summary_basis"])
        assert np.array_equal(m, z[f"c{c}_reduced_mean"])
        assert np.array_equal(t, z[f"c{c}_top_vector"])
        assert np.array_equal(a, z[f"c{c}_average_projector"])
    z = load("block_commit_replay.npz")
    b, m, t, a = go.block_commit_eig(z["projector_sum"], z["reduced_sum"], int(z["token_count"]), 4,
                                     [int(v) for v in z["flag_dims"]])
    assert np.array_equal(b, z["summary_basis"]) and np.array_equal(t, z["top_vector"])


def test_global_features_match_reference_branch():
    # golden: softmax + einsum + top_eig_summary + alignment_components, the
    # torch branch of _resolve_single_global_request (modeling.py:2996-3108)
    z = load("global_features.npz")
    f, b = go.global_features(z["bank"], z["sel"], z["scores"], z["x"], 1.0, [int(v) for v in z["flag_dims"]], 32)
    assert np.array_equal(f, z["features"])
    assert np.array_equal(b, z["basis"])


def test_readout_collapse_matches_reference():
    z = load("readout_collapse.npz")
    uid, gs, gb, gp = go.collapse_logsumexp(z["scores"], z["token_ids"], z["blocks"], z["positions"])
    assert np.array_equal(uid, z["unique_ids"]) and np.array_equal(gs, z["grouped_scores"])
    assert np.array_equal(gb, z["grouped_blocks"]) and np.array_equal(gp, z["grouped_positions"])
    z = load("readout_collapse_e2e.npz")
    out = go.exact_readout_collapse(z["Q"], z["pool_K"], z["token_ids"], z["top_idx"])
    for got, key in zip(out, ("best_id", "best_score", "best_block", "best_pos")):
        assert np.array_equal(got, z[key])


def test_segmented_oracle_matches_reference():
    """The restatement of the CUDA segmented kernels agrees with the reference's
    native collapse on its golden list, and with the max collapse."""
    z = load("readout_collapse.npz")
    uid, inv = np.unique(z["token_ids"], return_inverse=True)
    assert np.array_equal(uid, z["unique_ids"])
    gs, gb, gp = go.segmented_logsumexp_occurrence(z["scores"], inv, z["blocks"], z["positions"], uid.size)
    assert np.array_equal(gs, z["grouped_scores"])
    assert np.array_equal(gb, z["grouped_blocks"]) and np.array_equal(gp, z["grouped_positions"])
    mx = go.segmented_max(z["scores"], inv, uid.size)
    want = np.full(uid.size, -np.inf, np.float32)
    np.maximum.at(want, inv, z["scores"])
    assert np.array_equal(mx, want)
    # non-finite maxima take the stub's branch: no occurrence, score m + log(1e-8)
    gs, gb, gp = go.segmented_logsumexp_occurrence(np.array([-np.inf, np.inf, 1.0, np.nan], np.float32),
                                                   np.array([0, 1, 1, 2]), np.arange(4), np.arange(4) + 10, 4)
    assert gs[0] == -np.inf and gs[1] == np.inf and gs[2] == -np.inf and gs[3] == -np.inf
    assert list(gb) == [-1, -1, -1, -1] and list(gp) == [-1, -1, -1, -1]


def centroid_case_blocks(z, ci):
    """Block entries of golden centroid case ci, in the layout centroid_candidates takes."""
    ents, off = [], 0
    base = z[f"q{ci}_base_scores"]
    for b, p, s in zip(z[f"q{ci}_blocks"], z[f"q{ci}_prefixes"], z[f"q{ci}_block_scores"]):
        ents.append(dict(token_ids=z["token_ids"][b][:p], cell_ids=z["token_cell_ids"][b][:p],
                         weights_q=z["token_cell_weights_q"][b][:p], cell_keys=z["cell_keys"][b],
                         cell_values_q=z["cell_values_q"][b], cell_counts=z["cell_counts"][b],
                         base_scores=base[off:off + p], features=z["token_features"][b][:p], block_score=float(s)))
        off += int(p)
    return ents


def test_centroid_cell_write_matches_reference():
    # golden: GfstDecodeState.append_exact_token (cuda_packed, state.py:315-470)
    # + _finalise_block_cells (state.py:501-551), one block at a time; the
    # x255 weight rounding of tests/test_state.py:85-99 ([0.75, 0.25] -> [191, 64])
    z = load("centroid_path.npz")
    C = int(z["dims"][3])
    for b in range(int(z["dims"][5])):
        ids, wq, keys, vals, cnt = co.cell_commit(z["cell_ids_in"][b], z["cell_weights_in"][b], z["cell_keys_in"][b],
                                                  z["cell_values_in"][b], C)
        assert np.array_equal(ids, z["token_cell_ids"][b])
        assert np.array_equal(wq, z["token_cell_weights_q"][b])
        assert np.array_equal(keys.view(np.uint16), z["cell_keys"][b].view(np.uint16))
        assert np.array_equal(vals, z["cell_values_q"][b])
        assert np.array_equal(cnt, z["cell_counts"][b])
    _, wq, _, _, _ = co.cell_commit([[2, 5]], [[0.75, 0.25]], [[0.1, 0.2, 0.3]], [[0.4, 0.5]], 8)
    assert wq.tolist() == [[191, 64]]


def test_centroid_candidates_match_reference():
    # golden: ExactRecallReadout._build_centroid_candidates (modeling.py:659-982)
    # on 9 query / selection cases (BH-FDR sets of 3-5 cells, minimum-count
    # fallbacks, confidence 0 to 1, a partial block, a block without cells)
    z = load("centroid_path.npz")
    for ci in range(int(z["n_cases"])):
        res = co.centroid_candidates(z[f"q{ci}_query_heads"], centroid_case_blocks(z, ci), top_cells_per_head=5,
                                     min_selected=2, cells_per_block=int(z["dims"][3]))
        assert res is not None
        scores, diag = res
        assert np.array_equal(np.concatenate([s for s in scores if s is not None]), z[f"q{ci}_scores"])
        for key in ("selected_block_slots", "selected_cell_ids", "selected_alphas", "selection_entropy",
                    "selection_margin", "selected_cells_per_head"):
            assert np.array_equal(diag[key], z[f"q{ci}_{key}"]), key
        assert np.float32(diag["confidence"]) == z[f"q{ci}_confidence"]


def test_open_block_rule_matches_reference_exact_store():
    """The open-block prefix a query sees is what the reference's own exact
    store reports after the token's append (current_exact_block_length,
    state.py:817-825): p + 1 while p < L - 1, none at the block's last token."""
    z = load("exact_store_open_block.npz")
    for L in (16, 64):
        prefix = z[f"L{L}_prefix"]
        T = prefix.shape[0]
        rule = np.array([go.streaming_open_len(L, L)[t % L] for t in range(T)])
        assert np.array_equal(rule, prefix)
        # the block id is the current block while it is open, and blocks are
        # completed at their last token (before that token's retrieval)
        t = np.arange(T)
        assert np.array_equal(z[f"L{L}_block_id"], np.where(prefix > 0, t // L, -1))
        assert np.array_equal(z[f"L{L}_completed"], (t + 1) // L)


def test_streaming_pass_composition():
    """The token-by-token oracle step: its frames are the per-token stream, its
    memory is the committed blocks with mean-key summaries, and a query sees the
    committed blocks plus its open prefix."""
    g = torch.Generator().manual_seed(3)
    S, T, d, r, m, L, n_slots, k = 2, 48, 16, 4, 1, 8, 3, 2
    U0 = go.qr_reference(torch.randn((S, d, r), generator=g).numpy(), sign_mode=go.SIGN_R_DIAG_POSITIVE)
    A = (torch.randn((S, T, d, m), generator=g) / 4).numpy()
    B = (torch.randn((S, T, r, m), generator=g) / 4).numpy()
    K, V, Q = (torch.randn((S, T, d), generator=g).numpy() for _ in range(3))
    out = go.streaming_pass(U0, A, B, K, V, Q, block_len=L, n_slots=n_slots, k=k, memory_bf16=False)
    Uf, _ = go.stream_frames(U0, A, B, 1.0, 1e-8, go.SIGN_R_DIAG_POSITIVE)
    assert np.array_equal(out["frames"][:, -1], Uf)
    # first block: no committed memory, the open prefix only
    assert (out["top_idx"][:, :L] == -1).all()
    for p in range(L - 1):
        keys = K[:, :p + 1]
        best = np.argmax(np.einsum("spd,sd->sp", keys.astype(np.float64), Q[:, p].astype(np.float64)), axis=1)
        ok = out["read_ok"][:, p]
        assert np.array_equal(out["best_tok"][ok, p], (n_slots * L + best)[ok])
    assert (out["best_tok"][:, L - 1] == -1).all()  # closed block, nothing committed yet
    # tokens of block 4 (blocks 0..3 committed, slot of block 3 = 0 after the wrap)
    t = 4 * L + 2
    summ = np.stack([go.block_commit_mean(K[:, b * L:(b + 1) * L], False) for b in (3, 1, 2)], axis=1)
    _, ref_i, ok = go.block_topk(Q[:, t:t + 1], summ, k)
    ok = ok[:, 0]
    slot_of = np.array([0, 1, 2])  # summ columns are slots 0, 1, 2
    assert np.array_equal(out["top_idx"][ok, t], slot_of[ref_i[ok, 0]])


def test_exact_topk_bf16_matches_reference():
    """exact_topk on bf16 banks (the reference ranks the bf16 result of
    keys @ q): the oracle's rounded scores equal the reference's, and the
    chosen keys agree up to the order of equal scores."""
    z = load("retrieval_exact_topk_bf16.npz")
    for c in range(4):
        keys = torch.from_numpy(z[f"c{c}_keys"]).view(torch.bfloat16).float().numpy()
        q = torch.from_numpy(z[f"c{c}_query"]).view(torch.bfloat16).float().numpy()
        k = int(z[f"c{c}_k"])
        idx, sc = go.exact_topk(keys, q, k, round_bf16=True)
        assert go.same_topk_up_to_ties(idx, sc, z[f"c{c}_idx"], z[f"c{c}_scores"], z[f"c{c}_all_scores"])
        # ties are resolved toward the lower index
        for j in range(1, k):
            if sc[j] == sc[j - 1]:
                assert idx[j] > idx[j - 1]


def mpuc_case(z, tag):
    from oracle import mpuc_oracle as mo

    w = {k: z[f"{tag}_{k}"] for k in mo.WEIGHT_NAMES}
    return w, z[f"{tag}_normalised"], z[f"{tag}_fast_in"], z[f"{tag}_mid_in"], z[f"{tag}_slow_in"]


def test_mpuc_scan_oracle_matches_reference():
    # the reference's own _forward_sequence_tensors (modeling.py:4449-4476) on
    # two cell sizes; float32 matmuls sum in a different order -> 1e-5
    from oracle import mpuc_oracle as mo

    z = load("mpuc_scan.npz")
    for tag in z["tags"]:
        w, x, fin, mid, sin = mpuc_case(z, str(tag))
        got = mo.forward_sequence_tensors(w, x, fin, mid, sin)
        for name, v in zip(("outputs", "boundary_logits", "fast", "mid", "slow"), got):
            ref = z[f"{tag}_{name}"]
            assert v.shape == ref.shape, name
            assert np.abs(v - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), (tag, name)
