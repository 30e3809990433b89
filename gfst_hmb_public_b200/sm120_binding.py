"""The reference's ``runtime_backends.sm120`` operator surface on the B200 kernels.

pkhairkh/gfst-hmb-public imports its accelerated operators from
``gfst_hmb_mpuc.runtime_backends``, which re-exports every name below from
``runtime_backends/sm120.py`` (src/gfst_hmb_mpuc/runtime_backends/__init__.py:1-53;
the public release omits that module and its sm_120 extensions).  Installed as
``gfst_hmb_mpuc.runtime_backends.sm120``, this module sends the reference's own
callers to the sm_100a kernels of this package:

* ``gfst_local_qr``            the local-QR operator (mathdx_extension.cpp:20-22)
* ``gfst_block_commit``        the block commit (modeling.py:3486-3505)
* ``gfst_heev``                batched symmetric eigenpairs (modeling.py:3181)
* ``gfst_global_sketch``       the global sketch features (modeling.py:3021-3030)
* ``exact_block_score``        within-block token scores (modeling.py:646-651)
* ``exact_block_materialize``  the packed-store slice (state.py:568)
* ``segmented_max_by_group`` / ``segmented_logsumexp_occurrence``
                               the readout collapse reductions (perf.py:153, 189)
* ``mpuc_recurrent_scan``      the MPUC recurrent scan (modeling.py:4424-4430),
                               for blocks registered with
                               ``install_mpuc_recurrent_scan``

The operators without a kernel here (the eigenpair-to-summary helpers, the
extension loaders and reports) return ``None`` or
``False``, which the reference's callers treat as "not available" and answer
with their own torch code, exactly as they do when an sm_120 extension is
missing.  Every operator given CPU tensors raises RuntimeError (there is no
CPU path), as the reference's extension checks do.
"""
from __future__ import annotations

import threading

import torch

from . import block_commit, gfst, memory, mpuc, readout


def _cuda() -> bool:
    return torch.cuda.is_available()


# ---- availability flags (runtime_backends/__init__.py) ----------------------
def sm120_exact_math_kernels_available() -> bool:
    return _cuda()


def exact_readout_score_available() -> bool:
    return _cuda()


def segmented_reduction_available() -> bool:
    return _cuda()


def mathdx_extension_available() -> bool:
    return _cuda()


def experimental_canonical_summary_enabled() -> bool:
    return False


def mpuc_recurrent_scan_available() -> bool:
    return _cuda()


# ---- operators with a B200 kernel -------------------------------------------
def gfst_local_qr(candidate_matrices: torch.Tensor, eps_sign: float) -> torch.Tensor:
    """[B, m, n] float32 CUDA (m >= n) -> the thin Q with the first-significant
    sign rule (gfst.py:35-46); mathdx_extension.cpp:20-22."""
    return gfst.gfst_local_qr(candidate_matrices, eps_sign)


def tensor_qr_operator(candidate: torch.Tensor, eps_sign: float) -> torch.Tensor:
    """The QR diagnostics' TensorQrOperator (diagnostics/local_qr_divergence.py:10),
    e.g. for reconstruct_local_qr_capture(payload, qr_operator=...): one [m, n]
    candidate (or a [B, m, n] batch) on any device; the QR runs on the current
    CUDA device and Q comes back on the candidate's device."""
    x = candidate.to(device=torch.device("cuda", torch.cuda.current_device()), dtype=torch.float32)
    q = gfst.gfst_local_qr(x if x.ndim == 3 else x.unsqueeze(0), eps_sign)
    q = q if x.ndim == 3 else q.squeeze(0)
    return q.to(candidate.device)


def gfst_block_commit(*, projector_sum, reduced_sum, token_count, max_flag_dim, flag_dims):
    """(summary_basis, reduced_mean, top_vector, average_projector) of a closed
    block (modeling.py:3487-3495)."""
    return block_commit.gfst_block_commit(projector_sum=projector_sum, reduced_sum=reduced_sum,
                                          token_count=token_count, max_flag_dim=max_flag_dim, flag_dims=flag_dims)


def gfst_heev(matrices: torch.Tensor):
    """(eigenvalues ascending, eigenvectors) of a batch of symmetric matrices
    (mathdx_runtime.cu:750-780)."""
    return block_commit.gfst_heev(matrices)


def gfst_global_sketch(**kwargs):
    """(features, global_sketch, eig_basis) with the keywords of modeling.py:3021-3030."""
    return block_commit.gfst_global_sketch(**kwargs)


def exact_block_score(query_vector: torch.Tensor, token_features: torch.Tensor,
                      within_block_weight: torch.Tensor) -> torch.Tensor:
    """Scores of a block's tokens through the bias-free within-block projection,
    float32 [m] (modeling.py:646-651)."""
    return readout.exact_block_score(query_vector, token_features, within_block_weight)


def exact_block_materialize(packed: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """packed[start:end] of a 1-D CUDA tensor (sm120_stub.cu:225-245)."""
    return memory.exact_block_materialize(packed, start, end)


def segmented_max_by_group(scores: torch.Tensor, inverse: torch.Tensor, group_count: int) -> torch.Tensor:
    """Per-group maximum (sm120_stub.cu:16-40, caller perf.py:153)."""
    return readout.segmented_max_by_group(scores, inverse, group_count)


def segmented_logsumexp_occurrence(scores, inverse, occurrence_blocks, occurrence_positions, *, group_count):
    """(grouped_scores, grouped_blocks, grouped_positions) (sm120_stub.cu:42-111,
    caller perf.py:189-197)."""
    return readout.segmented_logsumexp_occurrence(scores, inverse, occurrence_blocks, occurrence_positions,
                                                  group_count=group_count)


# ---- operators without a B200 kernel: "not available" -----------------------
def _unavailable(*args, **kwargs):
    return None


gfst_reference_block_average = _unavailable
gfst_reference_global_sketch = _unavailable
gfst_canonical_summary_from_eigpairs = _unavailable
gfst_summary_from_sketch = _unavailable
gfst_summary_from_sketch_batched = _unavailable
load_sm120_extension = _unavailable
load_mathdx_extension = _unavailable
mathdx_extension_dependency_report = _unavailable
mathdx_runtime_dependency_report = _unavailable


# ---- the MPUC recurrent scan -------------------------------------------------
# The reference calls mpuc_recurrent_scan(normalized, fast_inputs, mid_inputs,
# slow_inputs) from MpucGfstHmbBlock._forward_sequence (modeling.py:4424-4430)
# without the cell's weights; install_mpuc_recurrent_scan registers a block so
# that, while its _forward_sequence runs, the op finds that block's weights.
_active = threading.local()


def mpuc_recurrent_scan(normalized, fast_inputs, mid_inputs, slow_inputs):
    """runtime_backends.mpuc_recurrent_scan (csrc/sm120_stub.cu:210-224): the
    outputs, boundary logits and final fast / mid / slow states of
    _forward_sequence_tensors (modeling.py:4449-4476), the recurrence on the
    B200 scan kernel and the output projection batched over all tokens.
    Returns None -- the caller's "not available", after which it runs its own
    compiled path -- when no block registered with install_mpuc_recurrent_scan
    is running on this thread."""
    cell = getattr(_active, "cell", None)
    if cell is None:
        return None
    states, logits, fast, mid, slow = mpuc.recurrent_scan(cell, fast_inputs, mid_inputs, slow_inputs)
    out = mpuc.output_projection(cell, normalized, states)
    dt = normalized.dtype
    return out.to(dt), logits.to(dt), fast.to(dt), mid.to(dt), slow.to(dt)


def install_mpuc_recurrent_scan(block) -> "mpuc.MpucCellWeights":
    """Send ``block``'s recurrent scan (an MpucGfstHmbBlock) through the B200
    kernel: pack its weights on the current CUDA device (once: re-install after
    the parameters change), select the reference's own "sm120_cutlass" backend
    (set_recurrent_kernel_backend, modeling.py:4494-4508) and wrap the block's
    _forward_sequence so that mpuc_recurrent_scan sees these weights while it
    runs."""
    weights = mpuc.MpucCellWeights.from_module(block)
    inner = block._forward_sequence

    def forward_sequence(normalised):
        prev = getattr(_active, "cell", None)
        _active.cell = weights
        try:
            return inner(normalised)
        finally:
            _active.cell = prev

    block._forward_sequence = forward_sequence
    block.set_recurrent_kernel_backend("sm120_cutlass")
    return weights
