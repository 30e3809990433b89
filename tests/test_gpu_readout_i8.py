"""The exact readout with an int8 first look (gfst_exact_readout_i8,
gfst_block_commit_i8) through the C ABI.

It must return what the exact readout returns: the best token in the total
order (score descending, token ascending; NaN never wins), its score and its
value row.  Checked against the oracle (float64 scores, bit-exact selection
wherever the margin to the runner-up exceeds 1e-3 relative) and against the
bf16 tensor-core readout on the same inputs, including the cases the bound
handles specially: exact ties, queries whose candidate list overflows (scored
in full), keys with a wide dynamic range, non-finite keys, all-zero queries,
d = 256.  The int8 side data must bound what it claims to bound.
"""
import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import memory, readout
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu


def _pools(S, slots, L, d, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    K = (torch.randn((S, slots, L, d), generator=g) * scale).to(torch.bfloat16)
    V = torch.randn((S, slots, L, d), generator=g).to(torch.bfloat16)
    return K, V, g


def _commit_all(K, V, device):
    S, slots, L, d = K.shape
    mem = memory.BlockMemory(S, slots, L, d, dtype=torch.bfloat16, device=device, int8_keys=True)
    for b in range(slots):
        mem.commit(K[:, b].to(device), V[:, b].to(device))
    return mem


def _both(Q, mem, sel):
    a = readout.exact_readout(Q, mem.pool_K, mem.pool_V, sel, k8=mem.k8)
    b = readout.exact_readout(Q, mem.pool_K, mem.pool_V, sel)
    return a, b


def _check_vs_bf16(a, b):
    tok_a, sc_a, v_a = (t.cpu() for t in a)
    tok_b, sc_b, v_b = (t.cpu() for t in b)
    assert torch.equal(tok_a, tok_b)
    fin = torch.isfinite(sc_b)
    assert torch.equal(torch.isfinite(sc_a), fin)
    assert ((sc_a[fin] - sc_b[fin]).abs() <= 1e-5 * sc_b[fin].abs().clamp_min(1.0)).all()
    assert torch.equal(v_a, v_b)


@pytest.mark.parametrize("d", [128, 256])
def test_int8_first_look_matches_exact_readout(cuda_device, d):
    S, slots, L, Nq, k = 12, 40, 64, 100, 16
    K, V, g = _pools(S, slots, L, d, 7 + d)
    mem = _commit_all(K, V, cuda_device)
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.stack([torch.randperm(slots, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    sel = sel.to(torch.int32)
    sel[0, :5, 3] = -1          # skipped selections
    sel[1, 7, :] = -1           # a query with nothing selected
    a, b = _both(Q.to(cuda_device), mem, sel.to(cuda_device))
    _check_vs_bf16(a, b)
    rt, rs, _, ok = go.exact_readout(Q.float().numpy(), K.float().numpy(), None, sel.numpy())
    tok = a[0].cpu().numpy()
    assert np.array_equal(tok[ok], rt[ok])
    assert (tok[1, 7] == -1)


def test_int8_side_data_bounds_the_keys(cuda_device):
    S, slots, L, d = 3, 4, 32, 128
    K, V, g = _pools(S, slots, L, d, 11)
    K[0, 1, 5] = 0.0                       # all-zero key
    K[1, 2, 3, 0] = 3000.0                 # wide range in one key
    mem = _commit_all(K, V, cuda_device)
    k8 = mem.pool_K8.cpu().numpy().astype(np.float64)
    side = mem.k8_scale.cpu().numpy().astype(np.float64)
    scale, E, N = side[..., :L], side[..., L], side[..., L + 1]
    kf = K.float().numpy().astype(np.float64)
    err = np.sqrt(((kf - scale[..., None] * k8) ** 2).sum(-1))
    nrm = np.sqrt((kf ** 2).sum(-1))
    assert (err.max(-1) <= E).all()
    assert (nrm.max(-1) <= N).all()
    assert (np.abs(k8) <= 127).all()
    assert scale[0, 1, 5] == 0.0 and (k8[0, 1, 5] == 0).all()


def test_int8_first_look_ties_and_overflowing_lists(cuda_device):
    # block 3 of every stream: all 64 rows equal (exact ties: every row's
    # bound reaches the query's best, so the candidate list overflows and the
    # query is scored in full); block 5: pairs of equal rows
    S, slots, L, d, Nq, k = 6, 10, 64, 128, 70, 6
    K, V, g = _pools(S, slots, L, d, 21)
    K[:, 3] = K[:, 3, :1].expand(S, L, d)
    K[:, 5, 1::2] = K[:, 5, 0::2]
    mem = _commit_all(K, V, cuda_device)
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.stack([torch.randperm(slots, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    sel = sel.to(torch.int32)
    sel[:, :10, 0] = 3                     # the all-equal block in every chunk
    sel[:, :10, 1:] = torch.where(sel[:, :10, 1:] == 3, torch.full_like(sel[:, :10, 1:], 5), sel[:, :10, 1:])
    a, b = _both(Q.to(cuda_device), mem, sel.to(cuda_device))
    _check_vs_bf16(a, b)


def test_int8_first_look_wide_range_and_non_finite_keys(cuda_device):
    S, slots, L, d, Nq, k = 4, 8, 32, 128, 40, 4
    K, V, g = _pools(S, slots, L, d, 31)
    K[:, 1, :, 0] = 500.0                  # a dominant coordinate: coarse int8 steps elsewhere
    K[0, 2, 7, 9] = float("nan")           # NaN scores never win
    K[1, 4, 3, 2] = float("inf")           # +-inf scores
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    Q[2, 5] = 0.0                          # an all-zero query: scored in full
    mem = _commit_all(K, V, cuda_device)
    sel = torch.stack([torch.stack([torch.randperm(slots, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    a, b = _both(Q.to(cuda_device), mem, sel.to(torch.int32).to(cuda_device))
    _check_vs_bf16(a, b)


def test_int8_first_look_in_the_streaming_step(cuda_device):
    # StreamingStep keeps int8 copies by default (bf16, d = 128): its results
    # equal those of a step without them, step by step, through a ring wrap
    from gfst_hmb_public_b200 import workloads as wl
    from gfst_hmb_public_b200.step import StreamingStep

    S, d, r, m, L, slots, k = 10, 128, 16, 2, 64, 3, 2
    U0 = wl.random_orthonormal_frames(S, d, r, seed=3, device=cuda_device)
    a = StreamingStep(S, d=d, r=r, block_len=L, n_slots=slots, k=k, device=cuda_device)
    b = StreamingStep(S, d=d, r=r, block_len=L, n_slots=slots, k=k, device=cuda_device, int8_keys=False)
    assert a.memory.k8 is not None and b.memory.k8 is None
    a.set_frames(U0)
    b.set_frames(U0)
    g = torch.Generator().manual_seed(4)
    for _ in range(5):
        A = (torch.randn((S, L, d, m), generator=g) / d ** 0.5).to(cuda_device)
        B = (torch.randn((S, L, r, m), generator=g) / d ** 0.5).to(cuda_device)
        Kb, Vb, Qb = (torch.randn((S, L, d), generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
        oa, ob = a.step(A, B, Kb, Vb, Qb), b.step(A, B, Kb, Vb, Qb)
        _check_vs_bf16((oa.best_tok, oa.best_score, oa.value), (ob.best_tok, ob.best_score, ob.value))


@pytest.mark.parametrize("L,slots,d", [(16, 48, 128), (128, 24, 128), (256, 12, 128), (16, 4100, 128),
                                       (128, 10, 256)])
def test_int8_first_look_block_lengths_and_large_rings(cuda_device, L, slots, d):
    # every supported block length (16 | L <= 256: one to four 16-row tile
    # groups per column tile, 2 to 8 ring stages), d = 256 with long blocks,
    # and a ring of more than 4096 slots (selections grouped by the bitonic
    # sort instead of the counting sort)
    S, Nq, k = 2, 70, 6
    g = torch.Generator().manual_seed(40 + L + slots)
    mem = memory.BlockMemory(S, slots, L, d, dtype=torch.bfloat16, device=cuda_device, int8_keys=True)
    K = torch.randn((S, slots, L, d), generator=g).to(torch.bfloat16)
    V = torch.randn((S, slots, L, d), generator=g).to(torch.bfloat16)
    for b in range(slots):
        mem.commit(K[:, b].to(cuda_device), V[:, b].to(cuda_device))
    Q = torch.randn((S, Nq, d), generator=g).to(torch.bfloat16)
    sel = torch.stack([torch.stack([torch.randperm(slots, generator=g)[:k] for _ in range(Nq)]) for _ in range(S)])
    sel = sel.to(torch.int32)
    if slots > 4096:
        sel[:, :, 0] = slots - 1 - torch.arange(Nq, dtype=torch.int32)  # blocks beyond the counting sort's range
    a, b = _both(Q.to(cuda_device), mem, sel.to(cuda_device))
    _check_vs_bf16(a, b)
    rt, rs, _, ok = go.exact_readout(Q.float().numpy(), K.float().numpy(), None, sel.numpy())
    tok = a[0].cpu().numpy()
    assert np.array_equal(tok[ok], rt[ok])
