"""Parity of the segmented reductions and the block token score against the
CPU oracle (the reference's CUDA-backend semantics) and the reference's golden
collapse, through the C ABI.

Bar: group maxima, occurrences and group counts bit-exact; log-sum-exp scores
within 2e-6 relative + 2e-6 absolute (the device's expf/logf against the
host's); block scores within the rounding the formula allows (bf16: two bf16
roundings; fp32: 1e-5 of the absolute-value product).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import readout
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _lse_close(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    same_inf = np.isinf(want) & (got == want)
    fin = np.isfinite(want)
    assert np.all(same_inf | fin), (got[~fin], want[~fin])
    np.testing.assert_allclose(got[fin], want[fin], rtol=2e-6, atol=2e-6)


def test_collapse_matches_reference_golden(cuda_device):
    z = np.load(GOLDEN / "readout_collapse.npz")
    args = [torch.as_tensor(z[k]).to(cuda_device) for k in ("scores", "token_ids", "blocks", "positions")]
    uid, gs, gb, gp = readout.collapse_logsumexp_scores_and_occurrence(*args)
    assert np.array_equal(uid.cpu().numpy(), z["unique_ids"])
    _lse_close(gs.cpu().numpy(), z["grouped_scores"])
    assert np.array_equal(gb.cpu().numpy(), z["grouped_blocks"])
    assert np.array_equal(gp.cpu().numpy(), z["grouped_positions"])
    assert int(uid[torch.argmax(gs)]) == int(z["selected_token"])
    uid2, mx = readout.collapse_max_scores_by_group(args[0], args[1])
    want = np.full(uid.numel(), -np.inf, np.float32)
    np.maximum.at(want, np.searchsorted(z["unique_ids"], z["token_ids"]), z["scores"])
    assert torch.equal(uid2, uid) and np.array_equal(mx.cpu().numpy(), want)


@pytest.mark.parametrize("n,groups,ties", [(1, 1, False), (37, 5, True), (1024, 700, False), (2048, 64, True),
                                           (16384, 3000, True), (16384, 1, False), (5000, 5000, False)])
def test_segmented_matches_oracle(cuda_device, n, groups, ties):
    rng = np.random.default_rng(n * 7 + groups)
    scores = rng.standard_normal(n).astype(np.float32) * 4
    if ties:  # coarse values: many equal maxima inside a group
        scores = np.round(scores).astype(np.float32)
    inverse = rng.integers(0, groups, n)
    blocks = rng.integers(0, 512, n)
    positions = rng.integers(0, 128, n)
    dev = [torch.as_tensor(a).to(cuda_device) for a in (scores, inverse, blocks, positions)]
    gs, gb, gp = readout.segmented_logsumexp_occurrence(*dev, group_count=groups)
    ws, wb, wp = go.segmented_logsumexp_occurrence(scores, inverse, blocks, positions, groups)
    _lse_close(gs.cpu().numpy(), ws)
    assert np.array_equal(gb.cpu().numpy(), wb) and np.array_equal(gp.cpu().numpy(), wp)
    mx = readout.segmented_max_by_group(dev[0], dev[1], groups)
    assert np.array_equal(mx.cpu().numpy(), go.segmented_max(scores, inverse, groups))


def test_segmented_edge_cases(cuda_device):
    inf, nan = np.float32(np.inf), np.float32(np.nan)
    # group 0: all -inf; 1: +inf max; 2: NaN beside a finite max; 3: only NaN;
    # 4: empty; 5: ties (first index wins); element 9 belongs to no group (out of range)
    scores = np.array([-inf, -inf, inf, 1.0, nan, 2.0, nan, 3.0, 3.0, 9.0, 3.0], np.float32)
    inverse = np.array([0, 0, 1, 1, 2, 2, 3, 5, 5, 7, 5])
    blocks = np.arange(11) + 100
    positions = np.arange(11) + 200
    groups = 6
    dev = [torch.as_tensor(a).to(cuda_device) for a in (scores, inverse, blocks, positions)]
    gs, gb, gp = readout.segmented_logsumexp_occurrence(*dev, group_count=groups)
    ws, wb, wp = go.segmented_logsumexp_occurrence(scores, inverse, blocks, positions, groups)
    _lse_close(gs.cpu().numpy(), ws)
    assert np.array_equal(gb.cpu().numpy(), wb) and np.array_equal(gp.cpu().numpy(), wp)
    assert list(wb) == [-1, -1, 105, -1, -1, 107]
    # the NaN element of group 2 makes the stub's sum NaN, so it is clamped to 1e-8
    assert ws[2] == np.float32(2.0) + np.log(np.float32(1e-8), dtype=np.float32)
    mx = readout.segmented_max_by_group(dev[0], dev[1], groups).cpu().numpy()
    assert np.array_equal(mx, go.segmented_max(scores, inverse, groups))
    assert mx[4] == -inf and mx[3] == -inf
    # an empty list: every group empty
    e = torch.empty(0, device=cuda_device)
    el = torch.empty(0, dtype=torch.long, device=cuda_device)
    gs, gb, gp = readout.segmented_logsumexp_occurrence(e, el, el, el, group_count=3)
    assert torch.all(gs.cpu() == -inf) and torch.all(gb.cpu() == -1) and torch.all(gp.cpu() == -1)
    # no groups at all
    assert readout.segmented_max_by_group(dev[0], dev[1], 0).numel() == 0
    uid, gs, gb, gp = readout.collapse_logsumexp_scores_and_occurrence(e, el, el, el)
    assert uid.numel() == 0 and gs.numel() == 0


def test_segmented_rejects_oversize(cuda_device):
    big = torch.zeros(16385, device=cuda_device)
    with pytest.raises(RuntimeError, match="exceed"):
        readout.segmented_max_by_group(big, big.long(), 4)


def _block_score_ref(q, F, W):
    """modeling.py:651 (the native path): (within_block_proj(F) @ q).float(), in
    the inputs' dtype: fp32 products and sums, bf16 roundings of the
    projection output and of the score."""
    key = F.float() @ W.float().T
    if F.dtype == torch.bfloat16:
        key = key.to(torch.bfloat16).float()
    score = key @ q.float()
    if F.dtype == torch.bfloat16:
        score = score.to(torch.bfloat16).float()
    bound = key.abs() @ q.float().abs()
    chain = (F.float().abs() @ W.float().abs().T) @ q.float().abs()
    return score, bound, chain


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("m,n,k", [
    # tensor-core kernel (bf16, k % 64 == 0, n % 16 == 0): one block, a few tiles, many tiles per CTA,
    # n not a multiple of 32, the largest W that fits, a single token
    (64, 128, 128), (128, 128, 128), (300, 256, 64), (1000, 48, 192), (70001, 128, 128), (129, 16, 256),
    (517, 256, 192), (1, 128, 128),
    # SIMT kernel (other shapes; W too large for shared memory next to two tiles)
    (17, 40, 72), (1, 8, 8), (300, 264, 100), (33, 256, 256)])
def test_exact_block_score(cuda_device, dtype, m, n, k):
    g = torch.Generator().manual_seed(m * 1000 + n + k)
    q = torch.randn(n, generator=g).to(dtype)
    F = torch.randn(m, k, generator=g).to(dtype)
    W = (torch.randn(n, k, generator=g) / k ** 0.5).to(dtype)
    got = readout.exact_block_score(q.to(cuda_device), F.to(cuda_device), W.to(cuda_device)).cpu()
    ref, bound, chain = _block_score_ref(q, F, W)
    assert got.dtype == torch.float32 and got.shape == (m,)
    if dtype == torch.bfloat16:
        # a key may round to the neighbouring bf16 value (one ulp, 2^-7 relative)
        # and the score's own rounding may land one ulp away too
        tol = 2.0 ** -7 * bound + 2.0 ** -6 * ref.abs() + 1e-5 * chain + 1e-6
    else:
        tol = 1e-5 * chain + 1e-6
    assert torch.all((got - ref).abs() <= tol), float(((got - ref).abs() - tol).max())


def test_exact_block_score_identity_weight_matches_readout_scores(cuda_device):
    """W = I (the configuration the readout kernels score): score = bf16(key . q)."""
    g = torch.Generator().manual_seed(5)
    d = 128
    q = torch.randn(d, generator=g).to(torch.bfloat16)
    F = torch.randn(64, d, generator=g).to(torch.bfloat16)
    got = readout.exact_block_score(q.to(cuda_device), F.to(cuda_device),
                                    torch.eye(d, dtype=torch.bfloat16, device=cuda_device)).cpu()
    ref = (F.float() @ q.float()).to(torch.bfloat16).float()
    diff = (got - ref).abs()
    # both round an fp32 sum to bf16: one ulp apart at most, plus the sums' own order
    assert torch.all(diff <= 2.0 ** -7 * ref.abs() + 1e-5 * (F.float().abs() @ q.float().abs()) + 1e-6)
    assert readout.exact_block_score(q.to(cuda_device), F[:0].to(cuda_device),
                                     torch.eye(d, dtype=torch.bfloat16, device=cuda_device)).numel() == 0
