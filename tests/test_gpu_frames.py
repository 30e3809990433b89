"""Parity of the sm_100a frame kernels (update + Householder thin QR, streaming
pass) against the CPU oracle, through the C ABI.

Tolerances (the parity bar for frames): orthogonality max|Q^T Q - I| <= 1e-5,
principal-angle distance of every leading-column prefix <= 1e-4, and
elementwise |Q - Q_oracle| <= 1e-4 (two correct fp32 Householder codes differ by
up to ~5e-5 on the near-collinear frames).
"""
import math

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import gfst, workloads as wl
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

ORTH_TOL = 1e-5
SUBSPACE_TOL = 1e-4
ELEM_TOL = 1e-4
MODES = [go.SIGN_FIRST_SIGNIFICANT, go.SIGN_R_DIAG_POSITIVE]


def _check_frames(q_dev: torch.Tensor, q_ref: np.ndarray, elem_tol: float = ELEM_TOL):
    q = q_dev.detach().cpu().numpy()
    assert q.shape == q_ref.shape
    assert np.isfinite(q).all()
    assert go.orthogonality_error(q).max() <= ORTH_TOL
    assert go.max_prefix_subspace_distance(q, q_ref).max() <= SUBSPACE_TOL
    assert np.abs(q - q_ref).max() <= elem_tol


def test_reference_golden_candidate(cuda_device):
    # 4 x 2 candidate of tests/test_temp_local_qr_householder_vs_mgs_dataset.py:54-70
    cand = np.array([[1.0, 0.2], [0.1, 0.95], [0.3, 0.1], [0.2, -0.05]], np.float32)
    q = gfst.gfst_local_qr(torch.from_numpy(cand).to(cuda_device), 1e-8)
    _check_frames(q.unsqueeze(0), go.qr_reference(cand[None], 1e-8)[0][None])


@pytest.mark.parametrize("sign_mode", MODES)
def test_batched_qr_workload_sample(cuda_device, sign_mode):
    spec = wl.BATCHED_QR
    x = wl.batched_qr_inputs(8192, spec["d"], spec["r"], seed=spec["seed"])
    q = gfst.frame_update_qr(x.to(cuda_device), sign_mode=sign_mode)
    _check_frames(q, go.qr_reference(x.numpy(), 1e-8, sign_mode))


@pytest.mark.parametrize(
    "d,r",
    [(4, 2), (5, 3), (7, 1), (8, 8), (16, 4), (33, 17), (64, 8), (64, 32), (100, 20), (128, 16), (128, 32),
     (200, 8), (256, 16), (9, 9)],
)
def test_every_shape_class(cuda_device, d, r):
    g = torch.Generator().manual_seed(d * 1000 + r)
    x = torch.randn((37, d, r), generator=g)
    for mode in MODES:
        q = gfst.frame_update_qr(x.to(cuda_device), sign_mode=mode)
        _check_frames(q, go.qr_reference(x.numpy(), 1e-8, mode))


@pytest.mark.parametrize("m,beta", [(1, 1.0), (2, 0.8), (4, 1.0), (8, 0.5)])
def test_rank_m_update_then_qr(cuda_device, m, beta):
    g = torch.Generator().manual_seed(100 + m)
    U = wl.random_orthonormal_frames(64, 128, 32, seed=7)
    A = torch.randn((64, 128, m), generator=g) / 11.3
    B = torch.randn((64, 32, m), generator=g) / 11.3
    q = gfst.frame_update_qr(U.to(cuda_device), A.to(cuda_device), B.to(cuda_device), beta=beta,
                             sign_mode="r_diag_positive")
    ref = go.qr_reference(go.frame_candidate(U.numpy(), A.numpy(), B.numpy(), beta), 1e-8,
                          go.SIGN_R_DIAG_POSITIVE)
    _check_frames(q, ref)


def test_reference_update_rule(cuda_device):
    # residual_rank_one_v1 (gfst.py:115-140) folded into beta*U + A B^T
    g = torch.Generator().manual_seed(3)
    U = wl.random_orthonormal_frames(16, 64, 32, seed=11)
    x = torch.randn((16, 64), generator=g)
    q = gfst.update_basis_batched(U.to(cuda_device), x.to(cuda_device), 0.2)
    ref = go.qr_reference(go.residual_rank_one_candidate(U.numpy(), x.numpy(), 0.2), 1e-8)
    _check_frames(q, ref)


def test_degenerate_frames(cuda_device):
    x = torch.zeros((3, 16, 4))
    x[1, :, 0] = 1.0            # rank one, repeated column
    x[1, :, 1] = 1.0
    x[2] = torch.eye(16, 4) * -2.0  # negative diagonal
    for mode in MODES:
        q = gfst.frame_update_qr(x.to(cuda_device), sign_mode=mode).cpu().numpy()
        ref = go.qr_reference(x.numpy(), 1e-8, mode)
        assert np.isfinite(q).all()
        # zero frame -> identity columns, like LAPACK
        assert np.abs(q[0] - ref[0]).max() <= 1e-6
        assert np.abs(q[2] - ref[2]).max() <= 1e-6
        # rank-deficient frame: the leading column is determined
        assert np.abs(q[1][:, 0] - ref[1][:, 0]).max() <= 1e-6


def test_deterministic(cuda_device):
    x = wl.batched_qr_inputs(4096, 64, 8, seed=5).to(cuda_device)
    a = gfst.frame_update_qr(x)
    b = gfst.frame_update_qr(x)
    assert torch.equal(a, b)


def test_in_place_alias(cuda_device):
    x = wl.batched_qr_inputs(512, 64, 8, seed=6).to(cuda_device)
    ref = gfst.frame_update_qr(x)
    gfst.frame_update_qr(x, out=x)
    assert torch.equal(ref, x)


def test_nan_input_returns(cuda_device):
    x = torch.randn((8, 64, 8))
    x[3, 5, 2] = float("nan")
    q = gfst.frame_update_qr(x.to(cuda_device)).cpu()
    assert torch.isfinite(q[0]).all() and not torch.isfinite(q[3]).all()


@pytest.mark.parametrize("sign_mode", MODES)
def test_stream_small_trajectory(cuda_device, sign_mode):
    spec = wl.STREAM_SMALL
    F = spec.streams
    U0 = wl.random_orthonormal_frames(F, spec.d, spec.r, seed=spec.seed)
    A, B = wl.stream_update_factors(F, spec.tokens, spec.d, spec.r, spec.m, seed=spec.seed + 100)
    U = U0.to(cuda_device).clone()
    snaps = gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), sign_mode=sign_mode, out_every=16)
    ref_final, ref_snaps = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), 1.0, 1e-8, sign_mode, 16)
    _check_frames(U, ref_final)
    assert snaps.shape == ref_snaps.shape
    for i in range(snaps.shape[0]):
        _check_frames(snaps[i], ref_snaps[i])


@pytest.mark.parametrize("qr_method", ["householder", "cholesky2", "cholesky2_split"])
@pytest.mark.parametrize("d,r,m,T", [(128, 16, 2, 256), (128, 32, 4, 96), (64, 32, 4, 64), (64, 16, 4, 64)])
def test_stream_mid_and_full_frames(cuda_device, d, r, m, T, qr_method):
    F = 12
    U0 = wl.random_orthonormal_frames(F, d, r, seed=d + r)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=d * r)
    U = U0.to(cuda_device).clone()
    gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), sign_mode="r_diag_positive", qr_method=qr_method)
    ref, _ = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), 1.0, 1e-8, go.SIGN_R_DIAG_POSITIVE)
    _check_frames(U, ref)


@pytest.mark.parametrize("qr_method", ["cholesky2", "cholesky2_split"])
@pytest.mark.parametrize("sign_mode", MODES)
@pytest.mark.parametrize("d,r,m", [(128, 32, 4), (100, 24, 4), (40, 12, 2)])
def test_stream_cholesky2_sign_modes_and_padding(cuda_device, d, r, m, sign_mode, qr_method):
    # padded rows (d < 64 or 128) and columns (r < 16 or 32) go through the
    # same Gram / Cholesky / solve with unit columns in R
    F, T = 10, 48
    U0 = wl.random_orthonormal_frames(F, d, r, seed=3 * d + r)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=d + 7 * r)
    U = U0.to(cuda_device).clone()
    snaps = gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), sign_mode=sign_mode, out_every=16,
                               qr_method=qr_method)
    ref_final, ref_snaps = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), 1.0, 1e-8, sign_mode, 16)
    _check_frames(U, ref_final)
    for i in range(snaps.shape[0]):
        _check_frames(snaps[i], ref_snaps[i])


@pytest.mark.parametrize("qr_method", ["cholesky2", "cholesky2_split"])
@pytest.mark.parametrize("sign_mode", MODES)
def test_stream_cholesky2_falls_back_on_zero_columns(cuda_device, sign_mode, qr_method):
    # U = 0 and B = [I_m; 0]: the frame is [A, 0, ..., 0], whose zero columns
    # fail the pivot test; Householder then gives LAPACK's answer (trailing
    # columns = the reflectors applied to unit vectors)
    F, d, r, m = 6, 128, 32, 4
    g = torch.Generator().manual_seed(11)
    A = torch.randn((F, 1, d, m), generator=g)
    B = torch.zeros((F, 1, r, m))
    B[:, 0, :m, :] = torch.eye(m)
    U = torch.zeros((F, d, r), device=cuda_device)
    gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), sign_mode=sign_mode, qr_method=qr_method)
    ref, _ = go.stream_frames(np.zeros((F, d, r), np.float32), A.numpy(), B.numpy(), 1.0, 1e-8, sign_mode)
    q = U.cpu().numpy()
    assert np.isfinite(q).all()
    assert go.orthogonality_error(q).max() <= ORTH_TOL
    assert np.abs(q - ref).max() <= 1e-5


@pytest.mark.parametrize("qr_method", ["cholesky2", "cholesky2_split"])
@pytest.mark.parametrize("beta", [0.03, 0.05, 0.1])
def test_stream_cholesky2_mixed_conditioning(cuda_device, beta, qr_method):
    # a shrunken frame plus a rank-4 update: relative pivots around the 1e-2
    # test, so tokens and frames go either way; every token must still match
    F, d, r, m, T = 16, 128, 32, 4, 24
    U0 = wl.random_orthonormal_frames(F, d, r, seed=21)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=22)
    A = A * 2.0
    U = U0.to(cuda_device).clone()
    gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), beta=beta, sign_mode="r_diag_positive",
                       qr_method=qr_method)
    ref, _ = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), beta, 1e-8, go.SIGN_R_DIAG_POSITIVE)
    _check_frames(U, ref)


def test_stream_matches_repeated_single_steps(cuda_device):
    F, d, r, m, T = 40, 128, 16, 2, 24
    U0 = wl.random_orthonormal_frames(F, d, r, seed=1).to(cuda_device)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=2, device="cpu")
    A, B = A.to(cuda_device), B.to(cuda_device)
    U = U0.clone()
    gfst.stream_frames(U, A, B, qr_method="householder")
    V = U0.clone()
    for t in range(T):
        V = gfst.frame_update_qr(V, A[:, t].contiguous(), B[:, t].contiguous())
    # same kernels, same arithmetic order -> bitwise identical
    assert torch.equal(U, V)
    # CholeskyQR2 computes the same factor to fp32 rounding
    W = U0.clone()
    gfst.stream_frames(W, A, B, qr_method="cholesky2")
    assert (W - V).abs().max().item() <= 1e-5
    X = U0.clone()
    gfst.stream_frames(X, A, B, qr_method="cholesky2_split")
    assert (X - V).abs().max().item() <= 1e-5


@pytest.mark.parametrize("d,r,m", [(128, 32, 4), (128, 16, 2)])
def test_split_and_single_warp_cholesky2_agree(cuda_device, d, r, m):
    # the split kernel sums the Gram in four row blocks: the same factor to fp32
    # rounding as the one-warp kernel, over many frames and tokens; and it is
    # deterministic
    F, T = 300, 64
    U0 = wl.random_orthonormal_frames(F, d, r, seed=5).to(cuda_device)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=6, device="cpu")
    A, B = A.to(cuda_device), B.to(cuda_device)
    one, split, again = U0.clone(), U0.clone(), U0.clone()
    gfst.stream_frames(one, A, B, sign_mode="r_diag_positive", qr_method="cholesky2")
    gfst.stream_frames(split, A, B, sign_mode="r_diag_positive", qr_method="cholesky2_split")
    gfst.stream_frames(again, A, B, sign_mode="r_diag_positive", qr_method="cholesky2_split")
    assert torch.equal(split, again)
    assert (split - one).abs().max().item() <= 1e-5
    assert go.orthogonality_error(split.cpu().numpy()).max() <= ORTH_TOL


def test_stream_cholesky2_rejects_other_shapes(cuda_device):
    # CholeskyQR2 covers 8 < d <= 128; the split kernel only 8 < r <= 32
    for d, r, method in ((8, 8, "cholesky2"), (200, 8, "cholesky2"), (64, 8, "cholesky2_split")):
        U = torch.zeros((2, d, r), device=cuda_device)
        A = torch.zeros((2, 1, d, 4), device=cuda_device)
        B = torch.zeros((2, 1, r, 4), device=cuda_device)
        with pytest.raises(RuntimeError):
            gfst.stream_frames(U, A, B, qr_method=method)


@pytest.mark.parametrize("qr_method", ["householder", "cholesky2", "auto"])
@pytest.mark.parametrize("sign_mode", MODES)
@pytest.mark.parametrize("d,r,m", [(64, 8, 1), (40, 5, 4), (128, 8, 2), (20, 4, 1)])
def test_stream_narrow_frames(cuda_device, d, r, m, sign_mode, qr_method):
    # frames of <= 8 columns: CholeskyQR2 in the Householder kernel's lane
    # layout (8 or 16 lanes per frame), padded rows and columns included
    F, T = 19, 64
    U0 = wl.random_orthonormal_frames(F, d, r, seed=5 * d + r)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=d + 11 * r)
    U = U0.to(cuda_device).clone()
    snaps = gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), sign_mode=sign_mode, out_every=16,
                               qr_method=qr_method)
    ref_final, ref_snaps = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), 1.0, 1e-8, sign_mode, 16)
    _check_frames(U, ref_final)
    for i in range(snaps.shape[0]):
        _check_frames(snaps[i], ref_snaps[i])


@pytest.mark.parametrize("beta", [0.03, 0.1])
def test_stream_narrow_frames_mixed_conditioning(cuda_device, beta):
    # shrunken 64 x 8 frames plus rank-4 updates: pivots around the 1e-2 test,
    # so some warps take Householder for a token and others CholeskyQR2
    F, d, r, m, T = 40, 64, 8, 4, 32
    U0 = wl.random_orthonormal_frames(F, d, r, seed=31)
    A, B = wl.stream_update_factors(F, T, d, r, m, seed=32)
    A = A * 2.0
    U = U0.to(cuda_device).clone()
    gfst.stream_frames(U, A.to(cuda_device), B.to(cuda_device), beta=beta, sign_mode="r_diag_positive",
                       qr_method="cholesky2")
    ref, _ = go.stream_frames(U0.numpy(), A.numpy(), B.numpy(), beta, 1e-8, go.SIGN_R_DIAG_POSITIVE)
    _check_frames(U, ref)


@pytest.mark.parametrize("sign_mode", MODES)
def test_batched_narrow_qr_near_collinear_and_scaled(cuda_device, sign_mode):
    # one QR per frame, 64 x 8: columns scaled over 3.5 decades (Cholesky's
    # error is componentwise in the column scaling) and, in every fifth frame,
    # a column at cos 0.9999 to the previous one (pivot test fails -> that
    # warp's frames go through Householder)
    g = torch.Generator().manual_seed(41)
    x = torch.randn((400, 64, 8), generator=g) * torch.pow(10.0, -torch.arange(8) / 2.0)
    for f in range(0, 400, 5):
        c = x[f, :, 2] / x[f, :, 2].norm()
        p = torch.randn(64, generator=g)
        p -= (p @ c) * c
        p /= p.norm()
        x[f, :, 3] = 0.9999 * c + math.sqrt(1 - 0.9999 ** 2) * p
    q = gfst.frame_update_qr(x.to(cuda_device), sign_mode=sign_mode)
    _check_frames(q, go.qr_reference(x.numpy(), 1e-8, sign_mode))


def test_cpu_tensors_rejected():
    with pytest.raises(RuntimeError):
        gfst.canonical_qr_batched(torch.randn(2, 8, 4))


def test_unsupported_shape_rejected(cuda_device):
    with pytest.raises(RuntimeError):
        gfst.frame_update_qr(torch.randn(2, 64, 33, device=cuda_device))
    with pytest.raises(RuntimeError):
        gfst.frame_update_qr(torch.randn(2, 300, 8, device=cuda_device))
