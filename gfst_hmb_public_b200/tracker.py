"""Per-token local tracker on the GPU: the largest flag basis, the nested flag
levels and the alignment features of every stream, advanced T tokens per call.

Drop-in for the reference's per-(sample, layer) tracker (pkhairkh/gfst-hmb-public):
``_GfstTrackerState`` (src/gfst_hmb_mpuc/state.py:93-96) advanced by
``GfstHmbSublayer._update_local_bases`` (src/gfst_hmb_mpuc/modeling.py:2299-2423),
initialised by ``_initialise_local_tracker`` (modeling.py:2284-2297, ``init_basis``
= eye, gfst.py:49-50), with ``_local_alignment_features`` (modeling.py:2425-2437)
evaluated after every token.  One call runs the kernel
``gfst_local_tracker_stream`` over all streams and tokens; nothing falls back
to the CPU.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _native as nat
from .gfst import _sign_mode


def local_tracker_stream(
    U: torch.Tensor,
    nested: torch.Tensor | None,
    x: torch.Tensor,
    *,
    flag_dims: Sequence[int],
    forgetting_rates: Sequence[float],
    eps: float = 1e-6,
    eps_update: float = 1e-6,
    eps_sign: float = 1e-8,
    sign_mode="first_significant",
    features: bool = True,
) -> torch.Tensor | None:
    """Advance the trackers over the tokens x [S, T, d] (float32, CUDA).

    U [S, d, r] (r = flag_dims[-1]) and nested [S, L, r, r] (L = len(flag_dims)-1;
    level l in columns [0, flag_dims[l])) are updated in place.  Returns the
    alignment features [S, T, 2 * len(flag_dims)] (cumulative, increment pairs)
    or None with ``features=False``.
    """
    flag_dims = [int(v) for v in flag_dims]
    rates = [float(v) for v in forgetting_rates]
    if len(rates) != len(flag_dims):
        raise ValueError("forgetting_rates must match flag_dims")
    nl = len(flag_dims) - 1
    nat.require_cuda(U, x, what="local_tracker_stream")
    if U.ndim != 3 or x.ndim != 3:
        raise ValueError("local_tracker_stream expects U [S,d,r], x [S,T,d]")
    S, d, r = U.shape
    T = int(x.shape[1])
    if tuple(x.shape) != (S, T, d) or r != flag_dims[-1]:
        raise ValueError(f"local_tracker_stream: shape mismatch U{tuple(U.shape)} x{tuple(x.shape)} "
                         f"flag_dims{tuple(flag_dims)}")
    if nl > 0 and (nested is None or tuple(nested.shape) != (S, nl, r, r)):
        raise ValueError(f"local_tracker_stream: nested must be [S, {nl}, {r}, {r}]")
    for name, t in (("U", U), ("x", x)) + ((("nested", nested),) if nl > 0 else ()):
        if t.dtype != torch.float32:
            raise RuntimeError(f"local_tracker_stream: {name} must be float32")
        if t.device != U.device:
            raise RuntimeError("local_tracker_stream: all tensors must be on one device")
    if not U.is_contiguous() or (nl > 0 and not nested.is_contiguous()):
        raise ValueError("local_tracker_stream: U and nested must be contiguous (updated in place)")
    x = x.contiguous()
    feats = torch.empty((S, T, 2 * (nl + 1)), device=U.device, dtype=torch.float32) if features else None
    dims_arr = (ctypes.c_int32 * max(nl, 1))(*flag_dims[:-1])
    rates_arr = (ctypes.c_double * len(rates))(*rates)
    with torch.cuda.device(U.device):
        nat.call(
            "gfst_local_tracker_stream",
            nat.ptr(U), nat.ptr(nested) if nl > 0 else None, nat.ptr(x), S, T, d, r, nl,
            ctypes.cast(dims_arr, ctypes.c_void_p), ctypes.cast(rates_arr, ctypes.c_void_p), float(eps),
            float(eps_update), float(eps_sign), _sign_mode(sign_mode), nat.ptr(feats), nat.stream_of(U),
        )
    return feats


class LocalTracker:
    """Batched local trackers of ``n_streams`` (sample, layer) pairs.

    ``reduced_dim``, ``flag_dims``, ``forgetting_rates``, ``eps``, ``eps_update``
    and ``eps_sign`` mean what they mean in the reference's GfstHmbConfig
    (config.py:26-74).  ``largest_basis`` [S, d, r] and ``nested_bases`` (list of
    [S, r, dim_l] views) mirror ``_GfstTrackerState``.
    """

    def __init__(self, n_streams: int, *, reduced_dim: int = 64, flag_dims: Sequence[int] = (8, 16, 32),
                 forgetting_rates: Sequence[float] = (0.05, 0.10, 0.20), eps: float = 1e-6,
                 eps_update: float = 1e-6, eps_sign: float = 1e-8, sign_mode="first_significant",
                 device="cuda"):
        self.flag_dims = tuple(int(v) for v in flag_dims)
        self.forgetting_rates = tuple(float(v) for v in forgetting_rates)
        if len(self.flag_dims) != len(self.forgetting_rates):
            raise ValueError("forgetting_rates must match flag_dims")
        if tuple(sorted(set(self.flag_dims))) != self.flag_dims:
            raise ValueError("flag_dims must be strictly increasing")
        self.eps, self.eps_update, self.eps_sign, self.sign_mode = eps, eps_update, eps_sign, sign_mode
        device = torch.device(device)
        d, r = int(reduced_dim), self.flag_dims[-1]
        self.largest_basis = torch.eye(d, r, device=device).expand(n_streams, d, r).contiguous()
        nl = len(self.flag_dims) - 1
        self._nested = torch.zeros((n_streams, nl, r, r), device=device)
        for lvl, dim in enumerate(self.flag_dims[:-1]):
            self._nested[:, lvl, :, :dim] = torch.eye(r, dim, device=device)

    @property
    def nested_bases(self) -> list[torch.Tensor]:
        return [self._nested[:, lvl, :, :dim] for lvl, dim in enumerate(self.flag_dims[:-1])]

    def step(self, x: torch.Tensor, *, features: bool = True) -> torch.Tensor | None:
        """Consume tokens x [S, T, reduced_dim]; returns features [S, T, 2 * len(flag_dims)]."""
        return local_tracker_stream(self.largest_basis, self._nested if len(self.flag_dims) > 1 else None, x,
                                    flag_dims=self.flag_dims, forgetting_rates=self.forgetting_rates, eps=self.eps,
                                    eps_update=self.eps_update, eps_sign=self.eps_sign, sign_mode=self.sign_mode,
                                    features=features)

    def local_bases(self) -> list[torch.Tensor]:
        """U V_l for each nested level, then U (modeling.py:2417-2420)."""
        U = self.largest_basis
        return [torch.matmul(U, V) for V in self.nested_bases] + [U[..., : self.flag_dims[-1]]]


def block_tracker_stream(U: torch.Tensor, projector_sum: torch.Tensor, reduced_sum: torch.Tensor, x: torch.Tensor, *,
                         rate: float, eps_update: float = 1e-6, eps_sign: float = 1e-8,
                         sign_mode="first_significant") -> None:
    """Per-token block tracker over x [S, T, d]: U [S, d, r] takes the rule update
    at ``rate`` and its canonical QR, projector_sum [S, d, d] += U U^T,
    reduced_sum [S, d] += x; all three updated in place (modeling.py:3460-3479)."""
    nat.require_cuda(U, projector_sum, reduced_sum, x, what="block_tracker_stream")
    if U.ndim != 3 or x.ndim != 3:
        raise ValueError("block_tracker_stream expects U [S,d,r], x [S,T,d]")
    S, d, r = U.shape
    T = int(x.shape[1])
    if tuple(x.shape) != (S, T, d) or tuple(projector_sum.shape) != (S, d, d) or tuple(reduced_sum.shape) != (S, d):
        raise ValueError("block_tracker_stream: shape mismatch")
    for name, t in (("U", U), ("projector_sum", projector_sum), ("reduced_sum", reduced_sum), ("x", x)):
        if t.dtype != torch.float32:
            raise RuntimeError(f"block_tracker_stream: {name} must be float32")
        if t.device != U.device:
            raise RuntimeError("block_tracker_stream: all tensors must be on one device")
    for t in (U, projector_sum, reduced_sum):
        if not t.is_contiguous():
            raise ValueError("block_tracker_stream: state tensors must be contiguous (updated in place)")
    x = x.contiguous()
    with torch.cuda.device(U.device):
        nat.call("gfst_block_tracker_stream", nat.ptr(U), nat.ptr(projector_sum), nat.ptr(reduced_sum), nat.ptr(x), S,
                 T, d, r, float(rate), float(eps_update), float(eps_sign), _sign_mode(sign_mode), nat.stream_of(U))


class BlockTracker:
    """Batched block compressors: the reference's ``_GfstBlockCompressorState``
    (state.py:99-107) driven by ``_update_block_memory`` (modeling.py:3401-3571):
    per token the block basis update and the projector / token sums, and at
    every ``block_len`` tokens the reference-faithful eigen commit
    (``block_commit.gfst_block_commit``) followed by the reset of
    ``_reset_block_tracker`` (modeling.py:2464-2484)."""

    def __init__(self, n_streams: int, *, reduced_dim: int = 64, flag_dims: Sequence[int] = (8, 16, 32),
                 forgetting_rates: Sequence[float] = (0.05, 0.10, 0.20), block_len: int = 64,
                 eps_update: float = 1e-6, eps_sign: float = 1e-8, sign_mode="first_significant", device="cuda"):
        self.n_streams, self.d = int(n_streams), int(reduced_dim)
        self.flag_dims = tuple(int(v) for v in flag_dims)
        self.r = self.flag_dims[-1]
        self.rate = float(forgetting_rates[-1])
        self.block_len = int(block_len)
        self.eps_update, self.eps_sign, self.sign_mode = eps_update, eps_sign, sign_mode
        self.device = torch.device(device)
        self.reset()

    def reset(self) -> None:
        S, d, r = self.n_streams, self.d, self.r
        self.largest_basis = torch.eye(d, r, device=self.device).expand(S, d, r).contiguous()
        self.projector_sum = torch.zeros((S, d, d), device=self.device)
        self.reduced_sum = torch.zeros((S, d), device=self.device)
        self.current_block_tokens = 0

    def step(self, x: torch.Tensor) -> list[tuple[torch.Tensor, ...]]:
        """Consume tokens x [S, T, reduced_dim]; returns one (summary_basis,
        reduced_mean, top_vector, average_projector) tuple per block closed."""
        from . import block_commit

        commits = []
        t0, T = 0, int(x.shape[1])
        while t0 < T:
            n = min(T - t0, self.block_len - self.current_block_tokens)
            block_tracker_stream(self.largest_basis, self.projector_sum, self.reduced_sum, x[:, t0:t0 + n],
                                 rate=self.rate, eps_update=self.eps_update, eps_sign=self.eps_sign,
                                 sign_mode=self.sign_mode)
            self.current_block_tokens += n
            t0 += n
            if self.current_block_tokens == self.block_len:
                commits.append(block_commit.gfst_block_commit(
                    projector_sum=self.projector_sum, reduced_sum=self.reduced_sum, token_count=self.block_len,
                    max_flag_dim=self.r, flag_dims=self.flag_dims, eps_sign=self.eps_sign))
                self.reset()
        return commits
