"""The reference's own callers, run through the B200 binding.

``gfst_hmb_public_b200.sm120_binding`` is installed as the reference's
``runtime_backends.sm120`` (oracle.reference_import registers the reference
package from its offline install, baseline/_ref), and the reference's own
code drives the kernels:

* retrieval -- the drop-in BlockRetriever, built from the reference's own
  FaissGpuRetrievalConfig and queried with its GfstDecodeState, returns what
  the reference's exact_topk returns (the equality its FAISS test asserts,
  tests/test_retrieval.py:14-52), and rebuilds its record when the state
  version changes;
* local QR -- reconstruct_local_qr_capture / analyze_local_qr_divergence
  (diagnostics/local_qr_divergence.py:171-190, 365-420) replay a capture
  through the B200 QR operator and agree with the reference's own QR;
* block commit -- compare_block_commit_bundle (block_commit_replay.py:184-238)
  runs its "candidate" path through the binding's gfst_block_commit and
  classifies the reference's own replays as clean commits.

Skipped when no copy of the reference is present.
"""
import importlib
import math

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import retrieval, sm120_binding
from oracle import reference_import

pytestmark = pytest.mark.gpu

REF = reference_import.find_reference()
if REF is None:
    pytest.skip("no copy of the reference (baseline/_ref)", allow_module_level=True)


@pytest.fixture
def ref():
    reference_import.install(REF, backend=sm120_binding)
    yield importlib
    reference_import.install(REF, backend=None)


def test_retriever_matches_reference_exact_topk(cuda_device, ref):
    config = ref.import_module("gfst_hmb_mpuc.config")
    state_mod = ref.import_module("gfst_hmb_mpuc.state")
    ref_retrieval = ref.import_module("gfst_hmb_mpuc.retrieval")
    retriever = retrieval.BlockRetriever(config.FaissGpuRetrievalConfig(
        gpu_device=0, index_type="ivfflatip", nlist=4, nprobe=2, flat_fallback_threshold=64))
    state = state_mod.GfstDecodeState(num_layers=1, batch_size=1)
    g = torch.Generator().manual_seed(21)
    keys = torch.randn((300, 32), generator=g).to(cuda_device)
    for qi in range(8):
        query = torch.randn((32,), generator=g).to(cuda_device)
        indices, scores = retriever.search(state=state, layer_idx=0, batch_idx=0, keys_tensor=keys,
                                           query_tensor=query, top_k=11)
        exact_indices, exact_scores = ref_retrieval.FaissGpuRetriever.exact_topk(keys, query, 11)
        assert indices.tolist() == exact_indices.tolist()
        assert torch.allclose(scores, exact_scores, atol=1e-5)
    record = retriever._index_cache[(id(state), 0, 0)]
    assert record.device_index == 0
    before = record.state_version
    state.mark_mutated()
    retriever.search(state=state, layer_idx=0, batch_idx=0, keys_tensor=keys, query_tensor=query, top_k=3)
    assert retriever._index_cache[(id(state), 0, 0)].state_version != before


def _capture(gfst, seed):
    """A local-QR capture in the layout the reference's tracker records
    (modeling.py:2330-2423): the largest basis, its candidate under the
    reference rule, and the nested steps in r-space."""
    g = torch.Generator().manual_seed(seed)
    d, dims, rates = 64, (8, 16, 32), (0.05, 0.10, 0.20)
    r = dims[-1]
    basis = gfst.canonical_qr(torch.randn((d, r), generator=g))
    x = torch.randn((d,), generator=g)
    cand = gfst.update_basis_candidate(basis, x, rates[-1])
    p = gfst.canonical_qr(cand).transpose(0, 1) @ x
    steps = []
    for i, dim in enumerate(dims[:-1]):
        nb = gfst.canonical_qr(torch.randn((r, dim), generator=g))
        nc = gfst.update_basis_candidate(nb, p, rates[i])
        steps.append({"nested_index": i, "dim": dim, "nested_basis_in": nb, "nested_candidate": nc})
    return {"metadata": {"layer_idx": 0, "batch_idx": 0, "token_idx": 5, "absolute_position": 5,
                         "flag_dims": list(dims), "max_flag_dim": r, "eps": 1e-6, "eps_sign": 1e-8},
            "reduced_token": x, "largest_basis_in": basis, "largest_candidate": cand, "nested_steps": steps}


def test_local_qr_replay_through_binding(cuda_device, ref):
    gfst = ref.import_module("gfst_hmb_mpuc.gfst")
    lqd = ref.import_module("gfst_hmb_mpuc.diagnostics.local_qr_divergence")

    def native_qr(candidate, eps_sign):
        return gfst.canonical_qr_batched(candidate.unsqueeze(0), eps_sign=float(eps_sign)).squeeze(0)

    for seed in range(4):
        payload = _capture(gfst, seed)
        want = lqd.reconstruct_local_qr_capture(payload, qr_operator=native_qr)
        got = lqd.reconstruct_local_qr_capture(payload, qr_operator=sm120_binding.tensor_qr_operator)
        assert (got["largest_basis_out"] - want["largest_basis_out"]).abs().max() <= 1e-5
        assert (got["projected"] - want["projected"]).abs().max() <= 1e-5
        assert (got["local_features"] - want["local_features"]).abs().max() <= 1e-5
        # the divergence analysis of a rollout through each operator finds no
        # local-feature divergence to attribute
        native_payload = dict(payload, largest_basis_out=want["largest_basis_out"], projected=want["projected"],
                              local_features=want["local_features"])
        b200_payload = dict(payload, largest_basis_out=got["largest_basis_out"], projected=got["projected"],
                            local_features=got["local_features"])
        analysis = lqd.analyze_local_qr_divergence(native_payload, b200_payload, native_qr_operator=native_qr,
                                                   kernel_qr_operator=sm120_binding.tensor_qr_operator)
        assert analysis["rollout_local_feature_max_abs"] <= 1e-5


def test_block_commit_replay_candidate_is_clean(cuda_device, ref):
    """compare_block_commit_bundle's candidate path runs the B200 commit.  The
    commit outputs meet the diagnostic's clean tolerance (1e-8).  The
    diagnostic forms each prefix projector with a float32 product on the
    replay's own device (the CPU for "native", cuda:0 for "candidate"), which
    may round an ulp (about 6e-8) apart; formed on the CPU from the B200
    basis they are clean too, and the diagnostic's own deltas stay within its
    projector tolerance (1e-7)."""
    bcr = ref.import_module("gfst_hmb_mpuc.diagnostics.block_commit_replay")
    from pathlib import Path

    z = np.load(Path(__file__).resolve().parent / "golden" / "block_commit_eig_cases.npz")
    clean, proj_tol = 1e-8, 1e-7
    for c in range(int(z["n_cases"])):
        meta = [int(v) for v in z[f"c{c}_meta"]]
        bundle = {"projector_sum": torch.from_numpy(z[f"c{c}_projector_sum"]),
                  "reduced_sum": torch.from_numpy(z[f"c{c}_reduced_sum"]), "token_count": meta[0],
                  "max_flag_dim": meta[1], "flag_dims": tuple(meta[2:]), "eps": 1e-6, "eps_sign": 1e-8,
                  "block_key_proj_weight": None,
                  "prefix_dims": bcr._canonical_prefix_dims(max_flag_dim=meta[1])}
        native = bcr.replay_block_commit_bundle(bundle, implementation="native")
        cand = bcr.replay_block_commit_bundle(bundle, implementation="candidate")
        assert cand["used_accelerated_kernel"] is True
        # cases 5 and 7 repeat projectors: eigenvalue groups a few 1e-7 apart,
        # where the float32 basis may round an ulp apart (6e-8)
        vec_tol = 6e-8 if c in (5, 7) else clean
        for key, tol in (("average_projector", clean), ("reduced_mean", clean), ("top_vector", vec_tol),
                         ("summary_basis", vec_tol)):
            err = float((cand[key] - native[key]).abs().max())
            assert err <= tol, f"case {c} {key}: {err:.3e}"
        cpu_prefix = bcr._prefix_projectors_from_basis(cand["summary_basis"], prefix_dims=bundle["prefix_dims"])
        for dim, want in native["prefix_projectors"].items():
            err = float((cpu_prefix[dim] - want).abs().max())
            assert err <= (proj_tol if c in (5, 7) else clean), f"case {c} prefix {dim}: {err:.3e}"
        summary = bcr.compare_block_commit_bundle(bundle, reference_implementation="native",
                                                  variant_implementation="candidate")
        assert summary["variant_used_accelerated_kernel"] is True
        deltas = summary["prefix_projector_deltas"]
        assert max(deltas.values()) <= proj_tol, f"case {c}: {deltas}"
        assert summary["classification"] in ("clean_commit", "other_commit_mismatch"), summary["classification"]
        if summary["classification"] != "clean_commit":
            # only the device-formed projectors are past 1e-8
            assert max(deltas.values()) > clean
            assert max(summary["average_projector_max_abs"], summary["reduced_mean_max_abs"]) <= clean


def test_reference_mpuc_block_runs_the_scan_kernel(cuda_device, ref):
    # the reference's own MpucGfstHmbBlock._forward_sequence with its
    # "sm120_cutlass" backend calls runtime_backends.mpuc_recurrent_scan
    # (modeling.py:4424-4430); registered with install_mpuc_recurrent_scan,
    # that is the B200 scan, and it gives what the reference's own
    # _forward_sequence_tensors gives on the CPU
    modeling = ref.import_module("gfst_hmb_mpuc.modeling")
    blk = reference_import.reference_mpuc_cell(modeling, 128, 31)
    g = torch.Generator().manual_seed(32)
    normalised = torch.randn((3, 20, 128), generator=g)
    with torch.no_grad():
        want = modeling.MpucGfstHmbBlock._forward_sequence_tensors(blk, normalised)
    blk = blk.to(cuda_device)
    # no block registered: "not available", the caller keeps its own path
    assert sm120_binding.mpuc_recurrent_scan(normalised.to(cuda_device), None, None, None) is None
    sm120_binding.install_mpuc_recurrent_scan(blk)
    assert blk.recurrent_kernel_backend == "sm120_cutlass"
    calls = []
    inner = sm120_binding.mpuc.recurrent_scan

    def counting(*a, **k):
        calls.append(1)
        return inner(*a, **k)

    sm120_binding.mpuc.recurrent_scan = counting
    try:
        with torch.no_grad():
            outputs, logits, cache = blk._forward_sequence(normalised.to(cuda_device))
    finally:
        sm120_binding.mpuc.recurrent_scan = inner
    assert calls, "the reference's call site did not reach the B200 scan"
    for got, exp in ((outputs, want[0]), (logits, want[1]), (cache.fast_state, want[2]), (cache.mid_state, want[3]),
                     (cache.slow_state, want[4])):
        got = got.cpu().numpy()
        exp = exp.numpy()
        assert np.abs(got - exp).max() <= 1e-4 * max(1.0, float(np.abs(exp).max()))
