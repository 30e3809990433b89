"""GFST frame operators on B200: batched Householder thin QR with sign fixing,
rank-m frame updates, and the on-chip streaming pass.

Drop-in for the reference's local-QR operator surface (paths relative to
pkhairkh/gfst-hmb-public):

* ``canonical_qr_batched`` / ``canonical_qr``      <- src/gfst_hmb_mpuc/gfst.py:17-32
* ``canonicalize`` rule (first significant entry)  <- src/gfst_hmb_mpuc/gfst.py:35-46
* ``gfst_local_qr(candidate, eps_sign)``            <- runtime_backends.gfst_local_qr
  (src/gfst_hmb_mpuc/runtime_backends/__init__.py:9; native op
  src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:665-671).  It has the
  ``TensorQrOperator`` signature ``(Tensor, float) -> Tensor`` used by
  src/gfst_hmb_mpuc/diagnostics/local_qr_divergence.py:10,171-190.
* ``update_basis_candidate_batched`` / ``update_basis_batched``
                                                    <- src/gfst_hmb_mpuc/gfst.py:73-140

All ops take CUDA float32 tensors and run hand-written sm_100a kernels; CPU
tensors raise ``RuntimeError`` (there is no CPU path).
"""
from __future__ import annotations

import torch

from . import _native as nat

SIGN_FIRST_SIGNIFICANT = nat.SIGN_FIRST_SIGNIFICANT
SIGN_R_DIAG_POSITIVE = nat.SIGN_R_DIAG_POSITIVE
RESIDUAL_RANK_ONE_GFST_UPDATE_RULE = "residual_rank_one_v1"

_SIGN_MODES = {
    "first_significant": SIGN_FIRST_SIGNIFICANT,
    "r_diag_positive": SIGN_R_DIAG_POSITIVE,
    SIGN_FIRST_SIGNIFICANT: SIGN_FIRST_SIGNIFICANT,
    SIGN_R_DIAG_POSITIVE: SIGN_R_DIAG_POSITIVE,
}


def _sign_mode(mode) -> int:
    try:
        return _SIGN_MODES[mode]
    except KeyError:
        raise ValueError(f"unknown sign mode {mode!r}; use 'first_significant' or 'r_diag_positive'") from None


def _frames_view(x: torch.Tensor, what: str) -> tuple[torch.Tensor, tuple[int, ...]]:
    if x.ndim < 2:
        raise ValueError(f"{what}: expected rank >= 2, got shape {tuple(x.shape)}")
    if x.dtype != torch.float32:
        raise RuntimeError(f"{what}: expected float32, got {x.dtype}")
    lead = tuple(x.shape[:-2])
    return x.contiguous().reshape(-1, x.shape[-2], x.shape[-1]), lead


def frame_update_qr(
    U: torch.Tensor,
    A: torch.Tensor | None = None,
    B: torch.Tensor | None = None,
    *,
    beta: float = 1.0,
    eps_sign: float = 1e-8,
    sign_mode="first_significant",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Return the sign-fixed thin Q of ``beta * U + A @ B^T`` for every frame.

    U: [..., d, r]; A: [..., d, m]; B: [..., r, m] (A and B omitted for a plain QR).
    """
    nat.require_cuda(U, A, B, out, what="frame_update_qr")
    U3, lead = _frames_view(U, "frame_update_qr")
    n, d, r = U3.shape
    m = 0
    A3 = B3 = None
    if A is not None or B is not None:
        if A is None or B is None:
            raise ValueError("frame_update_qr: pass both A and B or neither")
        m = int(A.shape[-1])
        A3 = A.contiguous().reshape(n, d, m)
        B3 = B.contiguous().reshape(n, r, m)
        if A3.dtype != torch.float32 or B3.dtype != torch.float32:
            raise RuntimeError("frame_update_qr: A and B must be float32")
    if out is None:
        out = torch.empty_like(U3)
    else:
        if out.shape != U.shape or not out.is_contiguous():
            raise ValueError("frame_update_qr: out must be contiguous with U's shape")
    with torch.cuda.device(U.device):
        nat.call(
            "gfst_frame_update_qr",
            nat.ptr(U3), nat.ptr(A3), nat.ptr(B3), float(beta), nat.ptr(out), n, d, r, m,
            float(eps_sign), _sign_mode(sign_mode), nat.stream_of(U3),
        )
    return out.reshape(*lead, d, r)


def canonical_qr_batched(matrices: torch.Tensor, *, eps_sign: float = 1e-8) -> torch.Tensor:
    """Reduced Q of every matrix with the reference's first-significant-entry sign rule."""
    if matrices.ndim < 3:
        raise ValueError(f"expected rank >= 3 for batched QR, got shape {tuple(matrices.shape)}")
    if matrices.numel() == 0:
        return matrices.new_empty(matrices.shape)
    return frame_update_qr(matrices, eps_sign=eps_sign, sign_mode="first_significant")


def canonical_qr(matrix: torch.Tensor, *, eps_sign: float = 1e-8) -> torch.Tensor:
    if matrix.ndim != 2:
        raise ValueError(f"expected a rank-2 matrix, got shape {tuple(matrix.shape)}")
    if matrix.numel() == 0:
        return matrix.new_empty(matrix.shape)
    return frame_update_qr(matrix.unsqueeze(0), eps_sign=eps_sign).squeeze(0)


def gfst_local_qr(candidate_matrices: torch.Tensor, eps_sign: float) -> torch.Tensor:
    """Reference ``gfst_local_qr(candidate[B,m,n], eps_sign) -> Q[B,m,n]`` (m >= n), sign-fixed.

    Also accepts a single [m, n] candidate (the diagnostics' ``TensorQrOperator``).
    """
    if candidate_matrices.ndim == 2:
        return canonical_qr(candidate_matrices, eps_sign=float(eps_sign))
    if candidate_matrices.ndim != 3:
        raise ValueError(f"expected [B, m, n] candidates, got shape {tuple(candidate_matrices.shape)}")
    if candidate_matrices.shape[-2] < candidate_matrices.shape[-1]:
        raise ValueError("gfst_local_qr requires m >= n")
    return canonical_qr_batched(candidate_matrices, eps_sign=float(eps_sign))


_QR_METHODS = {"auto": 0, "householder": 1, "cholesky2": 2, "cholesky2_split": 3}


def stream_frames(
    U: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    *,
    beta: float = 1.0,
    eps_sign: float = 1e-8,
    sign_mode="first_significant",
    out_every: int = 0,
    qr_method: str = "auto",
) -> torch.Tensor | None:
    """Run T tokens of ``U <- QR(beta*U + A_t B_t^T)`` with every frame held on chip.

    U: [F, d, r] float32, updated in place.  A: [F, T, d, m]; B: [F, T, r, m].
    With ``out_every > 0`` the frames after tokens out_every-1, 2*out_every-1, ...
    are returned as [T // out_every, F, d, r]; otherwise returns None.
    ``qr_method``: "auto" (CholeskyQR2 for 32 < d <= 128 and 8 < r <= 32 --
    up to 2 frames per SM for d = 128 (4 for d <= 64) with each frame split
    over d/32 warps -- and for
    8 < d <= 128 with r <= 8; Householder otherwise), "householder",
    "cholesky2" (one frame per warp; 2 or 4 frames per warp with r <= 8) or
    "cholesky2_split" (one frame per CTA of d/32 warps, 8 < r <= 32); with
    CholeskyQR2 a frame whose Gram pivots fail the conditioning test falls
    back to Householder for that token (with r <= 8, every frame of its warp).
    """
    nat.require_cuda(U, A, B, what="stream_frames")
    if U.ndim != 3 or A.ndim != 4 or B.ndim != 4:
        raise ValueError("stream_frames expects U [F,d,r], A [F,T,d,m], B [F,T,r,m]")
    if not U.is_contiguous():
        raise ValueError("stream_frames: U must be contiguous (it is updated in place)")
    F, d, r = U.shape
    T, m = int(A.shape[1]), int(A.shape[3])
    if tuple(A.shape) != (F, T, d, m) or tuple(B.shape) != (F, T, r, m):
        raise ValueError(f"stream_frames: shape mismatch U{tuple(U.shape)} A{tuple(A.shape)} B{tuple(B.shape)}")
    for name, t in (("U", U), ("A", A), ("B", B)):
        if t.dtype != torch.float32:
            raise RuntimeError(f"stream_frames: {name} must be float32")
    A = A.contiguous()
    B = B.contiguous()
    snaps = None
    if out_every > 0:
        snaps = torch.empty((T // out_every, F, d, r), device=U.device, dtype=torch.float32)
    with torch.cuda.device(U.device):
        nat.call(
            "gfst_frame_stream_ex",
            nat.ptr(U), nat.ptr(A), nat.ptr(B), float(beta), F, T, d, r, m, float(eps_sign),
            _sign_mode(sign_mode), nat.ptr(snaps), int(out_every), _QR_METHODS[qr_method], nat.stream_of(U),
        )
    return snaps


def residual_rank_one_factors(
    basis: torch.Tensor, value: torch.Tensor, alpha: float, *, eps_update: float = 1e-6
) -> tuple[float, torch.Tensor, torch.Tensor]:
    """(beta, A, B) with ``beta*U + A B^T`` equal to the reference rule
    ``residual_rank_one_v1`` (gfst.py:115-140):
    (1-alpha) U + alpha x a^T + alpha s e_r^T,  a = U^T x,
    s = (x - U a) / sqrt(|x|^2 + eps_update^2).
    """
    weights = torch.matmul(basis.transpose(-2, -1), value.unsqueeze(-1)).squeeze(-1)
    projection = torch.matmul(basis, weights.unsqueeze(-1)).squeeze(-1)
    residual = value - projection
    value_norm = torch.linalg.vector_norm(value, dim=-1, keepdim=True)
    scaled_residual = residual / torch.sqrt(value_norm.square() + float(eps_update) ** 2)
    novelty = torch.zeros_like(weights)
    novelty[..., -1] = 1.0
    A = torch.stack((value, scaled_residual), dim=-1)
    B = torch.stack((alpha * weights, alpha * novelty), dim=-1)
    return 1.0 - float(alpha), A, B


def update_basis_batched(
    basis: torch.Tensor,
    value: torch.Tensor,
    alpha: float,
    *,
    update_rule: str = RESIDUAL_RANK_ONE_GFST_UPDATE_RULE,
    eps_update: float = 1e-6,
    eps_sign: float = 1e-8,
) -> torch.Tensor:
    """Reference ``update_basis_batched`` (gfst.py:73-88): rule update then canonical QR,
    with the update folded into the QR kernel as ``beta*U + A B^T``."""
    if str(update_rule) != RESIDUAL_RANK_ONE_GFST_UPDATE_RULE:
        raise ValueError(
            f"unsupported gfst update rule {update_rule!r}; expected {RESIDUAL_RANK_ONE_GFST_UPDATE_RULE!r}"
        )
    if basis.ndim != 3 or value.ndim != 2:
        raise ValueError("update_basis_batched expects basis [B,d,r] and value [B,d]")
    beta, A, B = residual_rank_one_factors(basis, value, alpha, eps_update=eps_update)
    return frame_update_qr(basis, A, B, beta=beta, eps_sign=eps_sign, sign_mode="first_significant")
