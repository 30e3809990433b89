"""Reference-faithful block commit (the eigen summary of a closed block) on the GPU.

Drop-in for the reference's accelerated commit op
``runtime_backends.gfst_block_commit(projector_sum=, reduced_sum=, token_count=,
max_flag_dim=, flag_dims=) -> (summary_basis, reduced_mean, top_vector,
average_projector)`` (call sites src/gfst_hmb_mpuc/modeling.py:3487-3495 and
src/gfst_hmb_mpuc/diagnostics/block_commit_replay.py:144-154), computing what
its torch path computes (average projector, ``top_eig_summary``,
src/gfst_hmb_mpuc/gfst.py:172-430) with the sm_100a kernel
``gfst_block_commit_eig``.  ``replay_block_commit_bundle`` mirrors the
replay diagnostic's ``implementation="candidate"`` branch
(block_commit_replay.py:141-175) on a bundle of the same layout.  There is no
CPU path: the reference's own ``"native"`` replay is the comparison point.
"""
from __future__ import annotations

import ctypes
from typing import Any, Sequence

import torch

from . import _native as nat


def gfst_block_commit(*, projector_sum: torch.Tensor, reduced_sum: torch.Tensor, token_count: int,
                      max_flag_dim: int, flag_dims: Sequence[int], eps_sign: float = 1e-8):
    """projector_sum [d, d] (or [S, d, d]) and reduced_sum [d] (or [S, d]) float32
    CUDA tensors.  Returns (summary_basis [.., d, max_flag_dim], reduced_mean,
    top_vector, average_projector), float32 on the same device."""
    nat.require_cuda(projector_sum, reduced_sum, what="gfst_block_commit")
    single = projector_sum.ndim == 2
    ps = projector_sum.unsqueeze(0) if single else projector_sum
    rs = reduced_sum.unsqueeze(0) if single else reduced_sum
    if ps.ndim != 3 or ps.shape[1] != ps.shape[2] or rs.shape != ps.shape[:2]:
        raise ValueError(f"gfst_block_commit: projector_sum {tuple(projector_sum.shape)} and reduced_sum "
                         f"{tuple(reduced_sum.shape)} do not match")
    for name, t in (("projector_sum", ps), ("reduced_sum", rs)):
        if t.dtype != torch.float32:
            raise RuntimeError(f"gfst_block_commit: {name} must be float32")
    if rs.device != ps.device:
        raise RuntimeError("gfst_block_commit: tensors on different devices")
    S, d = ps.shape[0], ps.shape[1]
    dims = [int(v) for v in flag_dims]
    ps, rs = ps.contiguous(), rs.contiguous()
    basis = torch.empty((S, d, int(max_flag_dim)), device=ps.device, dtype=torch.float32)
    mean = torch.empty((S, d), device=ps.device, dtype=torch.float32)
    top = torch.empty((S, d), device=ps.device, dtype=torch.float32)
    avg = torch.empty((S, d, d), device=ps.device, dtype=torch.float32)
    dims_arr = (ctypes.c_int32 * max(len(dims), 1))(*dims)
    with torch.cuda.device(ps.device):
        nat.call("gfst_block_commit_eig", nat.ptr(ps), nat.ptr(rs), S, d, int(token_count), int(max_flag_dim),
                 ctypes.cast(dims_arr, ctypes.c_void_p), len(dims), float(eps_sign), nat.ptr(basis), nat.ptr(mean),
                 nat.ptr(top), nat.ptr(avg), nat.stream_of(ps))
    if single:
        return basis[0], mean[0], top[0], avg[0]
    return basis, mean, top, avg


def _prefix_projectors(basis: torch.Tensor, prefix_dims: Sequence[int]) -> dict[int, torch.Tensor]:
    """block_commit_replay.py:35-41: symmetrised B[:, :k] B[:, :k]^T for each prefix width."""
    out = {}
    for k in prefix_dims:
        if int(k) <= basis.shape[-1]:
            b = basis[..., : int(k)]
            p = b @ b.transpose(-1, -2)
            out[int(k)] = 0.5 * (p + p.transpose(-1, -2))
    return out


def replay_block_commit_bundle(bundle: dict[str, Any], *, implementation: str = "candidate",
                               device: str | torch.device = "cuda") -> dict[str, Any]:
    """The replay diagnostic's accelerated branch on this kernel.  Bundle keys as
    block_commit_bundle_from_capture builds them (projector_sum, reduced_sum,
    token_count, max_flag_dim, flag_dims, eps_sign, prefix_dims,
    block_key_proj_weight)."""
    if implementation != "candidate":
        raise ValueError(f"only the 'candidate' (GPU) replay lives here, not {implementation!r}")
    dev = torch.device(device)
    basis, mean, top, avg = gfst_block_commit(
        projector_sum=bundle["projector_sum"].to(dev, torch.float32),
        reduced_sum=bundle["reduced_sum"].to(dev, torch.float32),
        token_count=int(bundle["token_count"]), max_flag_dim=int(bundle["max_flag_dim"]),
        flag_dims=tuple(int(v) for v in bundle["flag_dims"]), eps_sign=float(bundle.get("eps_sign", 1e-8)))
    prefix = _prefix_projectors(basis, tuple(int(v) for v in bundle.get("prefix_dims", ())))
    weight = bundle.get("block_key_proj_weight")
    key = None
    if weight is not None:  # block_commit_replay.py:44-53: W [mean; top_vector]
        key = torch.nn.functional.linear(torch.cat((mean, top)), weight.to(dev, torch.float32))
    cpu = lambda t: t.detach().to("cpu", torch.float32).clone()  # noqa: E731
    return {"implementation": "candidate", "used_accelerated_kernel": True,
            "average_projector": cpu(avg), "summary_basis": cpu(basis),
            "prefix_projectors": {k: cpu(v) for k, v in prefix.items()},
            "reduced_mean": cpu(mean), "top_vector": cpu(top), "block_key": None if key is None else cpu(key)}


def global_features(projector_bank: torch.Tensor, sel_idx: torch.Tensor, sel_scores: torch.Tensor, x: torch.Tensor,
                    *, temperature: float = 1.0, flag_dims: Sequence[int] = (8, 16, 32), max_flag_dim: int | None = None,
                    eps: float = 1e-6, eps_sign: float = 1e-8, return_sketch: bool = False,
                    return_basis: bool = False):
    """Global sketch features of every (stream, query): the torch branch of
    GfstHmbSublayer._resolve_single_global_request (modeling.py:2996-3108) --
    softmax-weighted sum of the selected blocks' summary projectors, its
    canonical top eigen basis, alignment components over the flag dims -- on
    the kernel ``gfst_global_features``.  projector_bank [S, NB, d, d];
    sel_idx int32 / sel_scores float32 [S, Nq, K] (entries outside [0, NB) are
    ignored); x [S, Nq, d].  Returns features [S, Nq, 2 * len(flag_dims)] (and the
    sketch [S, Nq, d, d] / basis [S, Nq, d, max_flag_dim] when asked)."""
    nat.require_cuda(projector_bank, sel_idx, sel_scores, x, what="global_features")
    S, NB, d, _ = projector_bank.shape
    Nq, K = int(sel_idx.shape[1]), int(sel_idx.shape[2])
    if tuple(sel_scores.shape) != (S, Nq, K) or tuple(x.shape) != (S, Nq, d) or tuple(sel_idx.shape) != (S, Nq, K):
        raise ValueError("global_features: shape mismatch")
    if sel_idx.dtype != torch.int32 or projector_bank.dtype != torch.float32 or x.dtype != torch.float32 \
            or sel_scores.dtype != torch.float32:
        raise RuntimeError("global_features: float32 bank / scores / x and int32 indices expected")
    dims = [int(v) for v in flag_dims]
    mfd = int(max_flag_dim if max_flag_dim is not None else max(dims))
    bank, idx, sc, xx = (t.contiguous() for t in (projector_bank, sel_idx, sel_scores, x))
    feats = torch.empty((S, Nq, 2 * len(dims)), device=x.device, dtype=torch.float32)
    sketch = torch.empty((S, Nq, d, d), device=x.device, dtype=torch.float32) if return_sketch else None
    basis = torch.empty((S, Nq, d, mfd), device=x.device, dtype=torch.float32) if return_basis else None
    dims_arr = (ctypes.c_int32 * len(dims))(*dims)
    with torch.cuda.device(x.device):
        nat.call("gfst_global_features", nat.ptr(bank), nat.ptr(idx), nat.ptr(sc), nat.ptr(xx), S, Nq, NB, d, K,
                 float(temperature), mfd, ctypes.cast(dims_arr, ctypes.c_void_p), len(dims), float(eps),
                 float(eps_sign), nat.ptr(feats), nat.ptr(sketch), nat.ptr(basis), nat.stream_of(x))
    out = [feats]
    if return_sketch:
        out.append(sketch)
    if return_basis:
        out.append(basis)
    return out[0] if len(out) == 1 else tuple(out)


def gfst_global_sketch(*, summary_projectors: torch.Tensor, final_indices: torch.Tensor, final_scores: torch.Tensor,
                       reduced_token: torch.Tensor, retrieval_temperature: float, flag_dims: Sequence[int],
                       max_flag_dim: int, eps: float):
    """runtime_backends.gfst_global_sketch with the keywords of its call site
    (modeling.py:3021-3030): one request -- summary_projectors [NB, d, d],
    final_indices [K] (into summary_projectors), final_scores [K], reduced_token
    [d] -- on the kernel ``gfst_global_features``.  Returns (features
    [2 * len(flag_dims)], global_sketch [d, d], eig_basis [d, max_flag_dim])."""
    nat.require_cuda(summary_projectors, final_indices, final_scores, reduced_token, what="gfst_global_sketch")
    if summary_projectors.ndim != 3 or final_indices.ndim != 1 or final_scores.shape != final_indices.shape \
            or reduced_token.ndim != 1:
        raise ValueError("gfst_global_sketch expects projectors [NB, d, d], indices [K], scores [K], token [d]")
    bank = summary_projectors.float()[None]
    idx = final_indices.to(torch.int32)[None, None]
    sc = final_scores.float()[None, None]
    x = reduced_token.float()[None, None]
    feats, sketch, basis = global_features(bank, idx, sc, x, temperature=float(retrieval_temperature),
                                           flag_dims=flag_dims, max_flag_dim=int(max_flag_dim), eps=float(eps),
                                           return_sketch=True, return_basis=True)
    return feats[0, 0], sketch[0, 0], basis[0, 0]


def gfst_heev(matrices: torch.Tensor, *, check: bool = True):
    """runtime_backends.gfst_heev (native gfst_heev_sm120_forward,
    src/gfst_hmb_mpuc/csrc/mathdx/mathdx_runtime.cu:620-650, 750-780; called at
    modeling.py:3181): batched symmetric eigendecomposition of [d, d] or
    [B, d, d] float32 / float64 matrices (lower triangle read, d <= 64),
    computed in float64.  Returns (eigenvalues [..., d] ascending, eigenvectors
    [..., d, d] with column j for eigenvalue j) in the input dtype.  With
    ``check`` a matrix whose iteration did not converge raises RuntimeError, as
    the reference's info check does (this waits for the stream)."""
    nat.require_cuda(matrices, what="gfst_heev")
    if matrices.ndim not in (2, 3) or matrices.shape[-1] != matrices.shape[-2]:
        raise ValueError("gfst_heev expects [d, d] or [B, d, d] matrices")
    if matrices.dtype not in (torch.float32, torch.float64):
        raise RuntimeError(f"gfst_heev: unsupported dtype {matrices.dtype} (float32 or float64)")
    single = matrices.ndim == 2
    a = (matrices[None] if single else matrices).contiguous()
    B, d = int(a.shape[0]), int(a.shape[-1])
    vals = torch.empty((B, d), dtype=a.dtype, device=a.device)
    vecs = torch.empty((B, d, d), dtype=a.dtype, device=a.device)
    info = torch.empty((B,), dtype=torch.int32, device=a.device)
    code = nat.DTYPE_F32 if a.dtype == torch.float32 else nat.DTYPE_F64
    with torch.cuda.device(a.device):
        nat.call("gfst_heev", nat.ptr(a), B, d, code, nat.ptr(vals), nat.ptr(vecs), nat.ptr(info),
                 nat.stream_of(a))
    if check and B > 0 and bool((info != 0).any()):
        raise RuntimeError("gfst_heev: the Jacobi iteration did not converge for "
                           f"{int((info != 0).sum())} of {B} matrices")
    return (vals[0], vecs[0]) if single else (vals, vecs)
