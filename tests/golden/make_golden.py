"""Generate the golden vectors in tests/golden/*.npz from the reference's own code.

Run where a copy of the reference exists: its offline install under
``baseline/_ref`` (found by default) or a source checkout named with
``--reference <checkout root>`` or ``$GFST_REFERENCE_SRC``:

    python tests/golden/make_golden.py [--reference <checkout root>]

The reference package cannot be imported as shipped (its __init__ pulls in
modules that were left out of the public release), so
``oracle.reference_import`` registers namespace modules pointing into the
reference's tree, plus a stub for the missing sm120 runtime loader whose
accelerated ops report "unavailable", which sends the reference down its own
torch code paths.  Nothing is copied.

Every fixture stores the inputs and the reference outputs.  The CPU tests pin
the oracle against them; the GPU tests pin the kernels against the oracle.
"""
from __future__ import annotations

import argparse
import importlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
REPO = OUT.parents[1]


def install_reference(pkg_dir: Path):
    """Register the reference package found at ``pkg_dir`` with the
    "unavailable" sm120 stub (oracle.reference_import)."""
    sys.path.insert(0, str(REPO))
    from oracle import reference_import

    return reference_import.install(pkg_dir)


def batched_qr_inputs(n, d, r, seed):
    sys.path.insert(0, str(REPO))
    from gfst_hmb_public_b200 import workloads as wl

    return wl.batched_qr_inputs(n, d, r, seed=seed)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=None,
                        help="root of a reference source checkout (default: baseline/_ref or $GFST_REFERENCE_SRC)")
    parser.add_argument("--only", choices=["mpuc"], default=None, help="write one fixture only")
    args = parser.parse_args()
    sys.path.insert(0, str(REPO))
    from oracle import reference_import

    pkg_dir = (Path(args.reference) / "src" / "gfst_hmb_mpuc") if args.reference else reference_import.find_reference()
    if pkg_dir is None or not (pkg_dir / "gfst.py").is_file():
        raise SystemExit("no copy of the reference: pass --reference <checkout root> or install it under baseline/_ref")
    if args.only == "mpuc":
        install_reference(pkg_dir)
        make_mpuc_fixture(importlib.import_module("gfst_hmb_mpuc.modeling"))
        return
    install_reference(pkg_dir)
    gfst = importlib.import_module("gfst_hmb_mpuc.gfst")
    retrieval = importlib.import_module("gfst_hmb_mpuc.retrieval")
    hh = importlib.import_module("gfst_hmb_mpuc.diagnostics.temp_local_qr_householder_vs_mgs_dataset")
    sign = importlib.import_module("gfst_hmb_mpuc.diagnostics.temp_local_qr_sign_problem_analysis")
    bcr = importlib.import_module("gfst_hmb_mpuc.diagnostics.block_commit_replay")
    perf = importlib.import_module("gfst_hmb_mpuc.perf")
    torch.manual_seed(0)

    # 1. the 4 x 2 known-answer candidate of the reference's QR tests
    #    (tests/test_temp_local_qr_householder_vs_mgs_dataset.py:54-70)
    cand = torch.tensor([[1.0, 0.2], [0.1, 0.95], [0.3, 0.1], [0.2, -0.05]], dtype=torch.float32)
    traced = hh.householder_reduced_q_with_trace(cand, eps_sign=1e-8)
    np.savez(OUT / "qr_known_answer.npz",
             candidate=cand.numpy(),
             canonical_q=gfst.canonical_qr(cand, eps_sign=1e-8).numpy(),
             householder_signfixed_q=traced["signfixed_q"].detach().numpy(),
             mgs_q=hh.modified_gram_schmidt_q(cand, eps_sign=1e-8, reorthogonalize=True).numpy())

    # 2. seeded sign-problem families of the reference's QR diagnostics
    #    (diagnostics/temp_local_qr_sign_problem_analysis.py:249-301)
    cases = sign.generate_random_sign_problem_cases(num_cases=20, seed=1234, rows=64, cols=32)
    mats = torch.stack([c["matrix"] for c in cases])
    np.savez(OUT / "qr_sign_problem_cases.npz",
             matrices=mats.numpy(),
             families=np.array([c["family"] for c in cases]),
             canonical_q=gfst.canonical_qr_batched(mats, eps_sign=1e-8).numpy())

    # 3. batched-QR workload sample through canonical_qr_batched (gfst.py:26-32)
    x = batched_qr_inputs(512, 64, 8, seed=20261201 + 1)
    np.savez(OUT / "qr_batched_sample.npz", matrices=x.numpy(),
             canonical_q=gfst.canonical_qr_batched(x, eps_sign=1e-8).numpy())

    # 4. reference update rule residual_rank_one_v1 over 16 tokens (gfst.py:73-140)
    g = torch.Generator().manual_seed(5)
    U = gfst.canonical_qr_batched(torch.randn((4, 64, 32), generator=g), eps_sign=1e-8)
    xs = torch.randn((16, 4, 64), generator=g)
    traj = []
    cands = []
    Ut = U
    for t in range(16):
        cands.append(gfst.update_basis_candidate_batched(Ut, xs[t], 0.2, eps_update=1e-6))
        Ut = gfst.update_basis_batched(Ut, xs[t], 0.2, eps_update=1e-6, eps_sign=1e-8)
        traj.append(Ut)
    np.savez(OUT / "update_rule_trajectory.npz", U0=U.numpy(), values=xs.numpy(), alpha=np.float32(0.2),
             candidates=torch.stack(cands).numpy(), frames=torch.stack(traj).numpy())

    # 5. retrieval: exact_topk (retrieval.py:165-172) on seeded banks, and the
    #    small bank of tests/test_retrieval.py:14-52
    g = torch.Generator().manual_seed(9)
    keys = torch.randn((64, 32), generator=g)
    queries = torch.randn((8, 32), generator=g)
    idx, vals = zip(*[retrieval.FaissGpuRetriever.exact_topk(keys, q, 5) for q in queries])
    small = torch.tensor([[1.0, 0.0, 0.0, 0.0], [0.0, 1.0, 0.0, 0.0], [0.5, 0.5, 0.0, 0.0],
                          [0.0, 0.0, 1.0, 0.0], [0.0, 0.0, 0.0, 1.0], [0.8, 0.2, 0.0, 0.0]])
    sq = torch.tensor([1.0, 0.0, 0.0, 0.0])
    si, sv = retrieval.FaissGpuRetriever.exact_topk(small, sq, 3)
    np.savez(OUT / "retrieval_exact_topk.npz", keys=keys.numpy(), queries=queries.numpy(),
             top_idx=torch.stack(idx).numpy(), top_scores=torch.stack(vals).numpy(),
             small_keys=small.numpy(), small_query=sq.numpy(), small_idx=si.numpy(), small_scores=sv.numpy())

    # 6. reference block commit replay, native path (block_commit_replay.py:97-139)
    g = torch.Generator().manual_seed(13)
    frames = gfst.canonical_qr_batched(torch.randn((16, 8, 4), generator=g), eps_sign=1e-8)
    proj_sum = sum(gfst.basis_projector(f) for f in frames)
    red_sum = torch.randn((8,), generator=g) * 3.0
    weight = torch.randn((6, 16), generator=g)
    bundle = {"projector_sum": proj_sum, "reduced_sum": red_sum, "token_count": 16, "max_flag_dim": 4,
              "flag_dims": (2, 4), "eps": 1e-6, "eps_sign": 1e-8, "block_key_proj_weight": weight,
              "prefix_dims": (2, 4)}
    rep = bcr.replay_block_commit_bundle(bundle, implementation="native")
    np.savez(OUT / "block_commit_replay.npz", projector_sum=proj_sum.numpy(), reduced_sum=red_sum.numpy(),
             token_count=16, flag_dims=np.array([2, 4]), weight=weight.numpy(),
             average_projector=rep["average_projector"].numpy(), summary_basis=rep["summary_basis"].numpy(),
             reduced_mean=rep["reduced_mean"].numpy(), top_vector=rep["top_vector"].numpy(),
             block_key=rep["block_key"].numpy())

    # 7. exact-token collapse + select (perf.py:164-229, modeling.py:1151-1169)
    g = torch.Generator().manual_seed(17)
    scores = torch.randn((48,), generator=g)
    token_ids = torch.randint(0, 20, (48,), generator=g)
    blocks = torch.arange(48) // 16
    positions = torch.arange(48) % 16
    uid, gsc, gbl, gpo = perf.collapse_logsumexp_scores_and_occurrence(scores, token_ids, blocks, positions)
    order = torch.argsort(gsc, descending=True)
    np.savez(OUT / "readout_collapse.npz", scores=scores.numpy(), token_ids=token_ids.numpy(),
             blocks=blocks.numpy(), positions=positions.numpy(), unique_ids=uid.numpy(),
             grouped_scores=gsc.numpy(), grouped_blocks=gbl.numpy(), grouped_positions=gpo.numpy(),
             selected_token=int(uid[order[0]]))
    # 8. the per-token local tracker: GfstHmbSublayer._update_local_bases
    #    (modeling.py:2299-2423: largest-level update + QR, projection, nested
    #    flag levels in r-space) and _local_alignment_features (2425-2437),
    #    called unbound on a minimal host object that carries the config and
    #    switches every capture hook off
    modeling = importlib.import_module("gfst_hmb_mpuc.modeling")
    config = importlib.import_module("gfst_hmb_mpuc.config")
    state_mod = importlib.import_module("gfst_hmb_mpuc.state")
    sub = modeling.GfstHmbSublayer
    for name, d, flag_dims, n_streams, T, seed in (("local_tracker_d64", 64, (8, 16, 32), 4, 48, 21),
                                                   ("local_tracker_d128", 128, (4, 8, 16), 3, 32, 22)):
        cfg = config.GfstHmbConfig(reduced_dim=d, flag_dims=flag_dims, key_dim=2 * d)
        host = types.SimpleNamespace(gfst_config=cfg, layer_idx=0, _active_transition_probe_capture=None,
                                     _current_transition_token_context=None)
        host._should_capture_transition_probe = lambda **kw: False
        host._should_capture_local_qr = lambda **kw: False
        host._should_record_local_qr_pool = lambda: False
        host._initialise_local_tracker = types.MethodType(sub._initialise_local_tracker, host)
        g = torch.Generator().manual_seed(seed)
        xs = torch.randn((n_streams, T, d), generator=g)
        r = max(flag_dims)
        nl = len(flag_dims) - 1
        feats = np.zeros((n_streams, T, 2 * (nl + 1)), np.float32)
        snaps = np.zeros((n_streams, T // 8, d, r), np.float32)
        U_out = np.zeros((n_streams, d, r), np.float32)
        V_out = np.zeros((n_streams, nl, r, r), np.float32)
        bases_out = []
        for s in range(n_streams):
            st = state_mod._GfstTrackerState()
            for t in range(T):
                local = sub._update_local_bases(host, st, xs[s, t])
                feats[s, t] = sub._local_alignment_features(host, st, xs[s, t]).numpy()
                if (t + 1) % 8 == 0:
                    snaps[s, (t + 1) // 8 - 1] = st.largest_basis.numpy()
            U_out[s] = st.largest_basis.numpy()
            for lvl, vb in enumerate(st.nested_bases):
                V_out[s, lvl, :, : vb.shape[1]] = vb.numpy()
            bases_out.append(np.concatenate([b.numpy() for b in local], axis=1))
        np.savez(OUT / f"{name}.npz", values=xs.numpy(), flag_dims=np.array(flag_dims),
                 forgetting_rates=np.array(cfg.forgetting_rates, np.float64), eps=np.float64(cfg.eps),
                 eps_update=np.float64(cfg.eps_update), eps_sign=np.float64(cfg.eps_sign), features=feats,
                 frames_every8=snaps, largest_basis=U_out, nested_bases=V_out, local_bases=np.stack(bases_out))
    # 9. reference block commits (replay_block_commit_bundle, native path:
    #    block_commit_replay.py:97-139 -> top_eig_summary, gfst.py:389-430) on
    #    projector sums of real block-tracker passes (modeling.py:3460-3479:
    #    rule update, canonical QR, projector_sum += U U^T, reduced_sum += x)
    #    and on degenerate spectra (repeated eigenvalues -> cluster bases)
    cases = []
    for s_idx, (d, fds, T) in enumerate(((64, (8, 16, 32), 64), (64, (8, 16, 32), 64), (64, (4, 8, 16), 48),
                                         (32, (2, 4, 8), 16), (16, (2, 4), 40))):
        g = torch.Generator().manual_seed(100 + s_idx)
        r = max(fds)
        U = torch.eye(d, r)
        ps = torch.zeros((d, d))
        rs = torch.zeros((d,))
        for _ in range(T):
            x = torch.randn((d,), generator=g)
            U = gfst.canonical_qr_batched(gfst.update_basis_candidate(U, x, 0.20, eps_update=1e-6).unsqueeze(0),
                                          eps_sign=1e-8).squeeze(0)
            ps = ps + gfst.basis_projector(U[:, :r])
            rs = rs + x
        cases.append((ps, rs, T, r, fds))
    # degenerate: one projector repeated (eigenvalue 1 with multiplicity r, 0 otherwise)
    g = torch.Generator().manual_seed(200)
    Uq = gfst.canonical_qr(torch.randn((16, 4), generator=g))
    cases.append((8.0 * gfst.basis_projector(Uq), torch.randn((16,), generator=g), 8, 4, (2, 4)))
    # the reference test's capture: diag(0, 0, 1, 1) summed twice
    cases.append((2.0 * torch.diag(torch.tensor([0.0, 0.0, 1.0, 1.0])), 2.0 * torch.tensor([1.0, -0.5, 0.25, 0.75]),
                  2, 2, (1, 2)))
    # two repeated projectors of different weights: clusters {1/3 x2}, {2/3 x2} inside d=12
    Ua = gfst.canonical_qr(torch.randn((12, 4), generator=g))
    cases.append((gfst.basis_projector(Ua[:, :2]) + 2.0 * gfst.basis_projector(Ua[:, 2:]),
                  torch.randn((12,), generator=g), 3, 4, (2, 4)))
    # a full block of the block tracker with its tokens kept: x, then the
    # commit of its sums (modeling.py:3460-3507)
    g = torch.Generator().manual_seed(300)
    d, fds, T = 64, (8, 16, 32), 64
    xs = torch.randn((3, T, d), generator=g)
    trk = {"values": xs.numpy(), "flag_dims": np.array(fds)}
    Us, Ps, Rs, bases, tops = [], [], [], [], []
    for s in range(3):
        U = torch.eye(d, 32)
        ps = torch.zeros((d, d))
        rs = torch.zeros((d,))
        for t in range(T):
            U = gfst.canonical_qr_batched(gfst.update_basis_candidate(U, xs[s, t], 0.20, eps_update=1e-6)
                                          .unsqueeze(0), eps_sign=1e-8).squeeze(0)
            ps = ps + gfst.basis_projector(U[:, :32])
            rs = rs + xs[s, t]
        rep = bcr.replay_block_commit_bundle(
            {"projector_sum": ps, "reduced_sum": rs, "token_count": T, "max_flag_dim": 32, "flag_dims": fds,
             "eps": 1e-6, "eps_sign": 1e-8, "block_key_proj_weight": None, "prefix_dims": fds},
            implementation="native")
        Us.append(U.numpy()); Ps.append(ps.numpy()); Rs.append(rs.numpy())
        bases.append(rep["summary_basis"].numpy()); tops.append(rep["top_vector"].numpy())
    np.savez(OUT / "block_tracker_pass.npz", **trk, largest_basis=np.stack(Us), projector_sum=np.stack(Ps),
             reduced_sum=np.stack(Rs), summary_basis=np.stack(bases), top_vector=np.stack(tops))

    # 10. global sketch features, the non-accelerated branch of
    #     _resolve_single_global_request (modeling.py:2996-3108): softmax of the
    #     final scores, einsum of the selected summary projectors, top_eig_summary,
    #     alignment_components over the flag dims (gfst.py:389-430, 580-588)
    g = torch.Generator().manual_seed(400)
    S, NB, d, K, NQ, fds = 2, 40, 64, 8, 6, (8, 16, 32)
    bank = torch.stack([torch.stack([gfst.basis_projector(torch.linalg.qr(torch.randn((d, 32), generator=g))[0])
                                     for _ in range(NB)]) for _ in range(S)])
    sel = torch.stack([torch.stack([torch.randperm(NB, generator=g)[:K] for _ in range(NQ)]) for _ in range(S)])
    scores = 2.0 * torch.randn((S, NQ, K), generator=g)
    xg = torch.randn((S, NQ, d), generator=g)
    feats = torch.zeros((S, NQ, 2 * len(fds)))
    bases = torch.zeros((S, NQ, d, 32))
    for s_i in range(S):
        for q in range(NQ):
            w = torch.softmax(scores[s_i, q] * float(1.0), dim=0)
            sketch = torch.einsum("k,kij->ij", w, bank[s_i, sel[s_i, q]])
            summ = gfst.top_eig_summary(sketch, rank=32, rank_boundaries=fds)
            pp = {int(k): v for k, v in dict(summ["prefix_projectors"]).items()}
            feats[s_i, q] = gfst.alignment_components(
                xg[s_i, q], [pp.get(int(m), gfst.basis_projector(summ["basis"][:, :m])) for m in fds], 1e-6)
            bases[s_i, q] = summ["basis"]
    np.savez(OUT / "global_features.npz", bank=bank.numpy(), sel=sel.numpy().astype(np.int32), scores=scores.numpy(),
             x=xg.numpy(), flag_dims=np.array(fds), features=feats.numpy(), basis=bases.numpy())

    # 11. readout with the token-id collapse end to end: float32 token scores of
    #     the selected blocks (modeling.py:599-657, k . q), the reference's
    #     collapse_logsumexp_scores_and_occurrence (perf.py:164-229), best group
    g = torch.Generator().manual_seed(500)
    S, NS, L, d, Nq, K = 2, 20, 16, 32, 10, 4
    poolc = torch.randn((S, NS, L, d), generator=g)
    ids = torch.randint(0, 50, (S, NS, L), generator=g, dtype=torch.int32)
    Qc = torch.randn((S, Nq, d), generator=g)
    selc = torch.stack([torch.stack([torch.randperm(NS, generator=g)[:K] for _ in range(Nq)]) for _ in range(S)])
    res = np.zeros((4, S, Nq), np.float64)
    for s_i in range(S):
        for q in range(Nq):
            blocks = [int(b) for b in selc[s_i, q]]
            keys = torch.cat([poolc[s_i, b] for b in blocks])
            scs = keys @ Qc[s_i, q]
            tid = torch.cat([ids[s_i, b] for b in blocks])
            blk = torch.tensor(blocks).repeat_interleave(L)
            pos = torch.arange(L).repeat(len(blocks))
            uid, gsc, gbl, gpo = perf.collapse_logsumexp_scores_and_occurrence(scs, tid, blk, pos)
            w = int(np.lexsort((uid.numpy(), -gsc.numpy()))[0])
            res[:, s_i, q] = [int(uid[w]), float(gsc[w]), int(gbl[w]), int(gpo[w])]
    np.savez(OUT / "readout_collapse_e2e.npz", pool_K=poolc.numpy(), token_ids=ids.numpy(), Q=Qc.numpy(),
             top_idx=selc.numpy().astype(np.int32), best_id=res[0].astype(np.int32),
             best_score=res[1].astype(np.float32), best_block=res[2].astype(np.int32),
             best_pos=res[3].astype(np.int32))

    out = {}
    for ci, (ps, rs, T, r, fds) in enumerate(cases):
        bundle = {"projector_sum": ps, "reduced_sum": rs, "token_count": T, "max_flag_dim": r, "flag_dims": fds,
                  "eps": 1e-6, "eps_sign": 1e-8, "block_key_proj_weight": None, "prefix_dims": fds}
        rep = bcr.replay_block_commit_bundle(bundle, implementation="native")
        out[f"c{ci}_projector_sum"] = ps.numpy()
        out[f"c{ci}_reduced_sum"] = rs.numpy()
        out[f"c{ci}_meta"] = np.array([T, r] + list(fds))
        for key in ("average_projector", "summary_basis", "reduced_mean", "top_vector"):
            out[f"c{ci}_{key}"] = rep[key].numpy()
    out["n_cases"] = np.array(len(cases))
    np.savez(OUT / "block_commit_eig_cases.npz", **out)
    make_centroid_fixture(modeling, state_mod)
    make_store_and_topk_fixtures()
    make_mpuc_fixture(modeling)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


def make_centroid_fixture(modeling, state_mod) -> None:
    """12. The centroid path: tokens written with cell ids / weights / keys /
    values through GfstDecodeState.append_exact_token (cuda_packed backend,
    state.py:315-551), blocks read back with load_exact_block, and
    ExactRecallReadout._build_centroid_candidates (modeling.py:659-982) on
    several queries and block selections (a partial block, a block without
    cells, selections that take the BH-FDR set and ones that fall back to
    the minimum count)."""
    torch.manual_seed(77)
    g = torch.Generator().manual_seed(77)
    hidden, key_dim, H, dk, dv, C, L, NB, W, vocab = 24, 16, 4, 8, 6, 8, 12, 6, 2, 40
    rd = modeling.ExactRecallReadout(hidden_size=hidden, key_dim=key_dim, centroid_heads=H, centroid_key_dim=dk,
                                     centroid_value_dim=dv, cells_per_block=C, centroid_top_cells_per_head=5,
                                     centroid_min_selected_cells_per_head=2)
    emb = torch.nn.Embedding(vocab, hidden)
    with torch.no_grad():  # query heads 0, 2 read query[0:8], heads 1, 3 read query[8:16]
        sel = torch.zeros((H * dk, key_dim))
        for h in range(H):
            for j in range(dk):
                sel[h * dk + j, (h * dk + j) % key_dim] = 1.0
        rd.centroid_query_proj.weight.copy_(sel)
    state = state_mod.GfstDecodeState(num_layers=1, batch_size=1, state_pack_backend="cuda_packed")
    tok = torch.randint(0, vocab, (NB, L), generator=g)
    cids = torch.randint(0, C + 2, (NB, L, W), generator=g)            # out-of-range ids are clamped
    cw = torch.rand((NB, L, W), generator=g)
    cw = cw / cw.sum(-1, keepdim=True)
    cw[:, ::5, 1] = 0.0                                                 # single-cell tokens
    cw[3] = 0.0                                                         # block 3 writes no cell
    ckey = torch.randn((NB, L, dk), generator=g)
    cval = torch.randn((NB, L, dv), generator=g) * 2.0
    # blocks 0 and 4: single-cell tokens whose keys follow a per-cell direction,
    # so a query head along one direction singles out that cell
    cell_dirs = torch.randn((C, dk), generator=g)
    for b in (0, 4):
        cw[b, :, 0], cw[b, :, 1] = 1.0, 0.0
        first = cids[b, :, 0].clamp(0, C - 1)
        ckey[b] = 2.5 * cell_dirs[first] + 0.2 * torch.randn((L, dk), generator=g)
    for b in range(NB):
        for t in range(L):
            state.append_exact_token(batch_idx=0, absolute_position=b * L + t, token_id=int(tok[b, t]), block_len=L,
                                     cells_per_block=C, centroid_key_dim=dk, centroid_value_dim=dv,
                                     cell_ids=cids[b, t], cell_weights=cw[b, t], cell_key=ckey[b, t],
                                     cell_value=cval[b, t])
    recs = [state.load_exact_block(batch_idx=0, block_id=b, block_len=L, cache_capacity=NB) for b in range(NB)]
    store = {
        "token_ids": np.stack([r.token_id_tensor.numpy() for r in recs]).astype(np.int32),
        "token_cell_ids": np.stack([r.token_cell_id_tensor.numpy() for r in recs]).astype(np.uint8),
        "token_cell_weights_q": np.stack([r.token_cell_weight_q_tensor.numpy() for r in recs]).astype(np.uint8),
        "cell_keys": np.stack([r.cell_keys.numpy() for r in recs]),
        "cell_values_q": np.stack([r.cell_values_q.numpy() for r in recs]),
        "cell_counts": np.stack([r.cell_counts.numpy() for r in recs]),
    }
    with torch.no_grad():
        feats_all = emb(tok.reshape(-1))
        token_keys = rd.within_block_proj(feats_all).reshape(NB, L, key_dim)
        token_feats = rd.centroid_token_proj(feats_all).reshape(NB, L, H, dv)
    # (query, [(block, prefix, score)]) cases
    cases = [([0, 1, 2], [L, L, L], [0.9, 0.4, -0.2]),
             ([4, 3, 5, 0], [L, L, 7, L], [1.5, 1.0, 0.2, -0.3]),
             ([5], [L], [0.0]),
             ([2, 4], [5, L], [0.3, 0.1]),
             ([1, 0, 5, 2, 4], [L, L, L, L, L], [0.2, 0.2, 0.1, 0.0, -0.1])]
    queries = torch.randn((len(cases), key_dim), generator=g) * 2.0
    # aligned queries: heads 0 / 2 point at one cell's mean key, heads 1 / 3 at
    # another's, so their robust z-scores pass the BH-FDR test
    present = [sorted(set(int(c) for c in cids[b, :, 0].clamp(0, C - 1))) for b in range(NB)]
    aligned = [(([0, 1, 2, 4, 5], [L] * 5, [0.5, 0.1, 0.3, 0.0, -0.2]), present[0][0], present[4][1], 1.5),
               (([5, 4, 2, 1], [L, L, L, 9], [0.2, 0.2, 0.2, 0.2]), present[4][2], present[4][2], 3.0),
               (([2, 0, 3], [L, L, L], [0.0, 0.4, 0.8]), present[0][1], present[0][2], 0.8),
               (([4, 0], [L, 6], [0.0, 0.0]), present[4][0], present[0][-1], 1.0)]
    extra = []
    for case, c0, c1, amp in aligned:
        cases.append(case)
        extra.append(torch.cat([amp * cell_dirs[c0], amp * cell_dirs[c1]]))
    queries = torch.cat([queries, torch.stack(extra)])
    out = {k: v for k, v in store.items()}
    out.update(cell_ids_in=cids.numpy().astype(np.int32), cell_weights_in=cw.numpy(), cell_keys_in=ckey.numpy(),
               cell_values_in=cval.numpy(), token_keys=token_keys.numpy(), token_features=token_feats.numpy(),
               queries=queries.numpy(), dims=np.array([H, dk, dv, C, L, NB, W]), n_cases=np.array(len(cases)))
    for ci, (blocks, prefixes, bscores) in enumerate(cases):
        q = queries[ci]
        entries = [(recs[b], p, s) for b, p, s in zip(blocks, prefixes, bscores)]
        with torch.no_grad():
            res = rd._build_centroid_candidates(query=q, embedding_layer=emb, block_entries=entries)
            qh = rd.centroid_query_proj(q).reshape(H, dk).float()
            base = [rd._score_block_tokens(query=q, embedding_layer=emb, record=recs[b], prefix_length=p,
                                           block_score=s)[0] for b, p, s in zip(blocks, prefixes, bscores)]
        out[f"q{ci}_blocks"] = np.array(blocks, np.int32)
        out[f"q{ci}_prefixes"] = np.array(prefixes, np.int32)
        out[f"q{ci}_block_scores"] = np.array(bscores, np.float32)
        out[f"q{ci}_query_heads"] = qh.numpy()
        out[f"q{ci}_base_scores"] = np.concatenate([b.numpy() for b in base])
        out[f"q{ci}_none"] = np.array(res is None)
        if res is not None:
            scores, tids, blks, poss, diag = res
            out[f"q{ci}_scores"] = torch.cat(scores).numpy()
            out[f"q{ci}_token_ids"] = torch.cat(tids).numpy().astype(np.int32)
            out[f"q{ci}_positions"] = torch.cat(poss).numpy().astype(np.int32)
            for key in ("selected_block_slots", "selected_cell_ids", "selected_alphas", "selection_entropy",
                        "selection_margin", "selected_cells_per_head"):
                out[f"q{ci}_{key}"] = diag[key].numpy()
            out[f"q{ci}_confidence"] = np.float32(diag["confidence"])
    np.savez(OUT / "centroid_path.npz", **out)



def make_store_and_topk_fixtures() -> None:
    """The exact store's open block and exact_topk on bf16 banks."""
    retrieval = importlib.import_module("gfst_hmb_mpuc.retrieval")
    # 13. the exact store's open block as the readout sees it: after each
    #     append_exact_token (state.py:651-815), the current block id and its
    #     prefix length (current_exact_block_id / current_exact_block_length,
    #     state.py:817-825), which modeling.py:2948-2963 appends to the
    #     retrieved blocks, and how many blocks the store has completed
    st_mod = importlib.import_module("gfst_hmb_mpuc.state")
    store_out = {}
    for L_open in (16, 64):
        state = st_mod.GfstDecodeState(num_layers=1, batch_size=1)
        ids, prefixes, completed = [], [], []
        for t in range(3 * L_open + 5):
            state.append_exact_token(batch_idx=0, absolute_position=t, token_id=1000 + t, block_len=L_open)
            bid = state.current_exact_block_id(0, L_open)
            ids.append(-1 if bid is None else int(bid))
            prefixes.append(int(state.current_exact_block_length(0)))
            completed.append(len(state.samples[0].exact_store.completed_blocks))
        store_out[f"L{L_open}_block_id"] = np.array(ids, np.int32)
        store_out[f"L{L_open}_prefix"] = np.array(prefixes, np.int32)
        store_out[f"L{L_open}_completed"] = np.array(completed, np.int32)
    np.savez(OUT / "exact_store_open_block.npz", **store_out)

    # 14. exact_topk (retrieval.py:165-172) on bf16 banks: the reference ranks
    #     the bf16 result of keys @ q, so equal scores are common; and any k
    g = torch.Generator().manual_seed(14)
    topk_out = {}
    for ci, (count, d, k) in enumerate(((300, 64, 50), (4000, 64, 40), (17000, 32, 64), (77, 32, 77))):
        # multiples of 1/8 in [-2, 2): every partial sum is exact in float32,
        # so the bf16 rounding of a score does not depend on the summation order
        keys = (torch.randint(-16, 16, (count, d), generator=g) / 8.0).to(torch.bfloat16)
        q = (torch.randint(-16, 16, (d,), generator=g) / 8.0).to(torch.bfloat16)
        idx, sc = retrieval.FaissGpuRetriever.exact_topk(keys, q, k)
        topk_out[f"c{ci}_keys"] = keys.view(torch.int16).numpy()
        topk_out[f"c{ci}_query"] = q.view(torch.int16).numpy()
        topk_out[f"c{ci}_k"] = np.array(k)
        topk_out[f"c{ci}_idx"] = idx.numpy()
        topk_out[f"c{ci}_scores"] = sc.numpy()
        topk_out[f"c{ci}_all_scores"] = (keys @ q).float().numpy()
    np.savez(OUT / "retrieval_exact_topk_bf16.npz", **topk_out)



def make_mpuc_fixture(modeling) -> None:
    """13. The MPUC recurrent cell: MpucGfstHmbBlock._forward_sequence_tensors
    (modeling.py:4449-4476) with _token_step / _update_band /
    _semantic_residual (4343-4411), called on a block that holds only the
    cell (oracle.reference_import.reference_mpuc_cell: the reference's own
    constructors and sizes, nn.Linear's default initialisation under a fixed
    seed).  Stored: the branch outputs the scan consumes, the normalised
    tokens, every weight, and the reference's five outputs."""
    sys.path.insert(0, str(REPO))
    from oracle import mpuc_oracle, reference_import

    cls = modeling.MpucGfstHmbBlock
    out = {}
    for tag, H, B, T, seed in (("h64", 64, 3, 40, 901), ("h128", 128, 2, 24, 902)):
        blk = reference_import.reference_mpuc_cell(modeling, H, seed)
        g = torch.Generator().manual_seed(seed + 1)
        normalised = torch.randn((B, T, H), generator=g)
        with torch.no_grad():
            fin = blk.fast_branch.forward_sequence(normalised)
            mid_in = blk.mid_branch.forward_sequence(normalised)
            sin = blk.slow_branch.forward_sequence(normalised)
            outs = cls._forward_sequence_tensors(blk, normalised)
        params = dict(blk.named_parameters())
        for short, full in mpuc_oracle.WEIGHT_NAMES.items():
            out[f"{tag}_{short}"] = params[full].detach().numpy()
        out[f"{tag}_normalised"] = normalised.numpy()
        out[f"{tag}_fast_in"], out[f"{tag}_mid_in"], out[f"{tag}_slow_in"] = fin.numpy(), mid_in.numpy(), sin.numpy()
        for name, v in zip(("outputs", "boundary_logits", "fast", "mid", "slow"), outs):
            out[f"{tag}_{name}"] = v.detach().numpy()
    np.savez(OUT / "mpuc_scan.npz", tags=np.array(["h64", "h128"]), **out)

if __name__ == "__main__":
    main()
