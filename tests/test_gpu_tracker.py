"""Parity of the per-token local tracker kernel (largest flag basis, nested flag
levels, alignment features) against the reference's own methods (golden
vectors of GfstHmbSublayer._update_local_bases + _local_alignment_features) and
the CPU oracle, through the C ABI.

Bar (fp32, reduction order differs from torch's): frames and nested bases
orthonormal to 1e-5, elementwise within 2e-4 of the reference trajectory after
up to 48 tokens, features within 1e-4 absolute.
"""
import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import tracker
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("name", ["local_tracker_d64", "local_tracker_d128"])
def test_tracker_matches_reference_golden(cuda_device, name):
    z = np.load(GOLDEN / f"{name}.npz")
    fd = tuple(int(v) for v in z["flag_dims"])
    xs = torch.from_numpy(z["values"])
    S, T, d = xs.shape
    tr = tracker.LocalTracker(S, reduced_dim=d, flag_dims=fd, forgetting_rates=tuple(z["forgetting_rates"]),
                              eps=float(z["eps"]), eps_update=float(z["eps_update"]), eps_sign=float(z["eps_sign"]),
                              device=cuda_device)
    feats = []
    for t0 in range(0, T, 8):  # eight tokens per call; state carries over between calls
        feats.append(tr.step(xs[:, t0:t0 + 8].to(cuda_device)))
        snap = _np(tr.largest_basis)
        np.testing.assert_allclose(snap, z["frames_every8"][:, t0 // 8], atol=2e-4)
    feats = _np(torch.cat(feats, dim=1))
    np.testing.assert_allclose(feats, z["features"], atol=1e-4)
    U = _np(tr.largest_basis)
    np.testing.assert_allclose(U, z["largest_basis"], atol=2e-4)
    assert go.orthogonality_error(U).max() < 1e-5
    for lvl, V in enumerate(tr.nested_bases):
        Vn = _np(V)
        np.testing.assert_allclose(Vn, z["nested_bases"][:, lvl, :, : fd[lvl]], atol=2e-4)
        assert go.orthogonality_error(Vn).max() < 1e-5
    bases = np.concatenate([_np(b) for b in tr.local_bases()], axis=-1)
    np.testing.assert_allclose(bases, z["local_bases"], atol=2e-4)


@pytest.mark.parametrize("sign_mode", ["first_significant", "r_diag_positive"])
@pytest.mark.parametrize("d,flag_dims,S,T", [(32, (2, 4, 8), 9, 12), (64, (4, 16), 5, 10), (128, (8, 16, 32), 6, 6),
                                             (256, (4, 8, 16), 3, 6), (16, (8,), 4, 8), (64, (2, 4, 8, 16, 32), 3, 5)])
def test_tracker_matches_oracle(cuda_device, sign_mode, d, flag_dims, S, T):
    g = torch.Generator().manual_seed(d + T)
    xs = torch.randn((S, T, d), generator=g)
    rates = tuple(0.05 * (i + 1) for i in range(len(flag_dims)))
    tr = tracker.LocalTracker(S, reduced_dim=d, flag_dims=flag_dims, forgetting_rates=rates, sign_mode=sign_mode,
                              device=cuda_device)
    feats = _np(tr.step(xs.to(cuda_device)))
    r = flag_dims[-1]
    U0 = np.broadcast_to(np.eye(d, r, dtype=np.float32), (S, d, r))
    V0 = [np.broadcast_to(np.eye(r, k, dtype=np.float32), (S, r, k)) for k in flag_dims[:-1]]
    mode = go.SIGN_FIRST_SIGNIFICANT if sign_mode == "first_significant" else go.SIGN_R_DIAG_POSITIVE
    U, V, ref_feats, _ = go.local_tracker_stream(U0, V0, xs.numpy(), flag_dims, rates, sign_mode=mode)
    np.testing.assert_allclose(_np(tr.largest_basis), U, atol=2e-4)
    for lvl, Vl in enumerate(tr.nested_bases):
        np.testing.assert_allclose(_np(Vl), V[lvl], atol=2e-4)
    np.testing.assert_allclose(feats, ref_feats, atol=1e-4)
    assert feats.shape == (S, T, 2 * len(flag_dims))
    # nested columns past each level's size come back zero
    if len(flag_dims) > 1:
        nested = _np(tr._nested)
        for lvl, dim in enumerate(flag_dims[:-1]):
            assert not nested[:, lvl, :, dim:].any()


def test_tracker_zero_token_and_no_features(cuda_device):
    # an all-zero token: s = 0, the candidate is (1 - a) B, features are 0
    d, fd = 64, (8, 16, 32)
    xs = torch.zeros((2, 3, d))
    xs[1, 1] = torch.randn(d, generator=torch.Generator().manual_seed(1))
    tr = tracker.LocalTracker(2, reduced_dim=d, flag_dims=fd, device=cuda_device)
    feats = _np(tr.step(xs.to(cuda_device)))
    assert np.isfinite(feats).all()
    assert (feats[0] == 0).all()
    U0 = np.broadcast_to(np.eye(d, 32, dtype=np.float32), (2, d, 32))
    V0 = [np.broadcast_to(np.eye(32, k, dtype=np.float32), (2, 32, k)) for k in fd[:-1]]
    U, V, ref, _ = go.local_tracker_stream(U0, V0, xs.numpy(), fd, (0.05, 0.10, 0.20))
    np.testing.assert_allclose(feats, ref, atol=1e-4)
    np.testing.assert_allclose(_np(tr.largest_basis), U, atol=2e-4)
    assert tr.step(xs[:, :1].to(cuda_device), features=False) is None
    assert torch.isfinite(tr.largest_basis).all()


def test_tracker_rejects(cuda_device):
    tr = tracker.LocalTracker(2, reduced_dim=64, device=cuda_device)
    with pytest.raises(ValueError):
        tr.step(torch.randn(2, 3, 32, device=cuda_device))
    with pytest.raises(RuntimeError):
        tr.step(torch.randn(2, 3, 64, device=cuda_device, dtype=torch.float64))
    with pytest.raises(ValueError):
        tracker.LocalTracker(2, reduced_dim=64, flag_dims=(16, 8, 32), device=cuda_device)
    with pytest.raises(RuntimeError):  # d % 4 != 0 is refused by the library
        tracker.LocalTracker(1, reduced_dim=30, flag_dims=(4, 8), forgetting_rates=(0.1, 0.2),
                             device=cuda_device).step(
            torch.randn(1, 2, 30, device=cuda_device))


def test_block_tracker_matches_reference_pass(cuda_device):
    # golden: one 64-token block of the reference's block tracker per stream
    # (update + canonical QR + projector / token sums) and its native commit
    z = np.load(GOLDEN / "block_tracker_pass.npz")
    xs = torch.from_numpy(z["values"])
    S, T, d = xs.shape
    bt = tracker.BlockTracker(S, reduced_dim=d, flag_dims=tuple(int(v) for v in z["flag_dims"]), block_len=T,
                              device=cuda_device)
    bt.step(xs[:, :20].to(cuda_device))  # the block in three calls
    bt.step(xs[:, 20:21].to(cuda_device))
    np.testing.assert_allclose(_np(bt.largest_basis), go.block_tracker_stream(
        np.broadcast_to(np.eye(d, 32, dtype=np.float32), (S, d, 32)), np.zeros((S, d, d), np.float32),
        np.zeros((S, d), np.float32), z["values"][:, :21], 0.2)[0], atol=2e-4)
    U_mid = bt.largest_basis.clone()
    P_mid, R_mid = bt.projector_sum.clone(), bt.reduced_sum.clone()
    commits = bt.step(xs[:, 21:].to(cuda_device))
    assert len(commits) == 1 and bt.current_block_tokens == 0
    # the sums at the end of the block, recomputed without the reset
    U2, P2, R2 = U_mid.clone(), P_mid.clone(), R_mid.clone()
    tracker.block_tracker_stream(U2, P2, R2, xs[:, 21:].to(cuda_device), rate=0.2)
    np.testing.assert_allclose(_np(U2), z["largest_basis"], atol=2e-4)
    np.testing.assert_allclose(_np(P2), z["projector_sum"], atol=1e-4)
    assert np.array_equal(_np(R2), z["reduced_sum"])  # token sums in token order: bit-exact
    basis, mean, top, avg = (_np(t) for t in commits[0])
    assert np.array_equal(mean, z["reduced_sum"] / np.float32(T))
    for s in range(S):  # the commit of slightly different fp32 sums: same subspaces
        for k in (8, 16, 32):
            pg = basis[s][:, :k] @ basis[s][:, :k].T
            pr = z["summary_basis"][s][:, :k] @ z["summary_basis"][s][:, :k].T
            assert np.abs(pg - pr).max() < 1e-3
    # after the reset the tracker starts a fresh block
    assert torch.equal(bt.largest_basis[0], torch.eye(d, 32, device=cuda_device))
    assert bt.projector_sum.abs().max().item() == 0.0


def test_block_tracker_chunking_is_bitwise(cuda_device):
    g = torch.Generator().manual_seed(4)
    S, d, r, T = 5, 32, 8, 24
    xs = torch.randn((S, T, d), generator=g).to(cuda_device)
    states = []
    for cuts in ((T,), (5, 11, 8), (1,) * T):
        U = torch.eye(d, r, device=cuda_device).expand(S, d, r).contiguous()
        P = torch.zeros((S, d, d), device=cuda_device)
        R = torch.zeros((S, d), device=cuda_device)
        t0 = 0
        for c in cuts:
            tracker.block_tracker_stream(U, P, R, xs[:, t0:t0 + c], rate=0.15)
            t0 += c
        states.append((U, P, R))
    for U, P, R in states[1:]:
        assert torch.equal(U, states[0][0]) and torch.equal(P, states[0][1]) and torch.equal(R, states[0][2])
    ref = go.block_tracker_stream(np.broadcast_to(np.eye(d, r, dtype=np.float32), (S, d, r)),
                                  np.zeros((S, d, d), np.float32), np.zeros((S, d), np.float32), _np(xs), 0.15)
    np.testing.assert_allclose(_np(states[0][0]), ref[0], atol=2e-4)
    np.testing.assert_allclose(_np(states[0][1]), ref[1], atol=1e-4)
    assert np.array_equal(_np(states[0][2]), ref[2])
    P = _np(states[0][1])
    assert np.array_equal(P, np.swapaxes(P, 1, 2))  # exactly symmetric


def test_block_tracker_rejects(cuda_device):
    with pytest.raises(RuntimeError):  # d > 64
        tracker.BlockTracker(1, reduced_dim=128, device=cuda_device).step(torch.randn(1, 2, 128, device=cuda_device))
