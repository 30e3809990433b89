"""Parity of the MPUC recurrent scan kernel (gfst_mpuc_recurrent_scan) through
the C ABI: against the reference's own _forward_sequence_tensors
(modeling.py:4449-4476, golden fixture) and against the CPU oracle at a wider
cell, with several launches' worth of sequences and non-zero initial states.

Tolerance: the kernel and the reference both compute in fp32 but sum the
matrix-vector products in different orders; over tens of tokens of a
contracting recurrence the states agree to about 1e-6, checked at 1e-4
(relative to the largest magnitude).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import mpuc
from oracle import mpuc_oracle as mo

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 1e-4


def _close(got, ref, what):
    got = got.detach().cpu().numpy() if isinstance(got, torch.Tensor) else got
    assert got.shape == ref.shape, what
    assert np.isfinite(got).all(), what
    assert np.abs(got - ref).max() <= TOL * max(1.0, float(np.abs(ref).max())), what


def _random_cell(H, seed, C=None):
    """Weights with nn.Linear's default scale (uniform in +-1/sqrt(fan_in))."""
    rng = np.random.default_rng(seed)
    F, M = H // 2, H // 4
    S = H - F - M
    C = C or max(64, H // 16)
    BH = max(8, H // 16)
    SR = max(64, H // 16)

    def lin(o, i):
        return rng.uniform(-1, 1, (o, i)).astype(np.float32) / np.sqrt(i)

    def bias(o, i):
        return rng.uniform(-1, 1, (o,)).astype(np.float32) / np.sqrt(i)

    w = {"fast_gate_w": lin(F, F), "fast_gate_b": bias(F, F), "fast_cand_w": lin(F, F), "fast_cand_b": bias(F, F),
         "mid_gate_w": lin(M, M), "mid_gate_b": bias(M, M), "mid_cand_w": lin(M, M), "mid_cand_b": bias(M, M),
         "slow_gate_w": lin(S, S), "slow_gate_b": bias(S, S), "slow_cand_w": lin(S, S), "slow_cand_b": bias(S, S),
         "fm_down": lin(C, M), "fm_up": lin(F, C), "fs_down": lin(C, S), "fs_up": lin(F, C),
         "mf_down": lin(C, F), "mf_up": lin(M, C), "ms_down": lin(C, S), "ms_up": lin(M, C),
         "sf_down": lin(C, F), "sf_up": lin(S, C), "sm_down": lin(C, M), "sm_up": lin(S, C),
         "bnd_w1": lin(BH, 4), "bnd_b1": bias(BH, 4), "bnd_w2": lin(1, BH), "bnd_b2": bias(1, BH),
         "sem_in": lin(SR, H), "sem_cond": lin(SR, M + S), "sem_out": lin(H, SR), "fusion": lin(H, H)}
    return w, (F, M, S)


@pytest.mark.parametrize("tag", ["h64", "h128"])
def test_scan_matches_reference_forward_sequence(cuda_device, tag):
    z = np.load(GOLDEN / "mpuc_scan.npz")
    cell = mpuc.MpucCellWeights({k: z[f"{tag}_{k}"] for k in mo.WEIGHT_NAMES}, cuda_device)
    ins = [torch.from_numpy(z[f"{tag}_{n}"]).to(cuda_device) for n in ("fast_in", "mid_in", "slow_in")]
    states, logits, fast, mid, slow = mpuc.recurrent_scan(cell, *ins)
    out = mpuc.output_projection(cell, torch.from_numpy(z[f"{tag}_normalised"]).to(cuda_device), states)
    for name, v in zip(("outputs", "boundary_logits", "fast", "mid", "slow"), (out, logits, fast, mid, slow)):
        _close(v, z[f"{tag}_{name}"], f"{tag} {name}")


def test_scan_matches_oracle_wide_cell_many_sequences(cuda_device):
    # H = 256 (fast 128, mid 64, slow 64), bridge rank 64; 11 sequences (a
    # launch of 8 and one of 3), 48 tokens, starting from non-zero states
    H, B, T = 256, 11, 48
    w, (F, M, S) = _random_cell(H, 5)
    rng = np.random.default_rng(6)
    fin = rng.standard_normal((B, T, F)).astype(np.float32)
    mid_in = rng.standard_normal((B, T, M)).astype(np.float32)
    sin = rng.standard_normal((B, T, S)).astype(np.float32)
    init = [0.5 * rng.standard_normal((B, n)).astype(np.float32) for n in (F, M, S)]
    ref = mo.recurrent_scan(w, fin, mid_in, sin, init=init)
    cell = mpuc.MpucCellWeights(w, cuda_device)
    got = mpuc.recurrent_scan(cell, *(torch.from_numpy(x).to(cuda_device) for x in (fin, mid_in, sin)),
                              state=tuple(torch.from_numpy(x).to(cuda_device) for x in init))
    for name, g, r in zip(("states", "boundary_logits", "fast", "mid", "slow"), got, ref):
        _close(g, r, name)
    normalised = rng.standard_normal((B, T, H)).astype(np.float32)
    out = mpuc.output_projection(cell, torch.from_numpy(normalised).to(cuda_device), got[0])
    _close(out, mo.fused_outputs(w, normalised, ref[0]), "outputs")


def test_scan_is_deterministic_and_resumable(cuda_device):
    # the same call twice gives the same bits; T tokens in one call equal
    # T1 + T2 tokens in two calls that carry the states over
    H, B, T, T1 = 128, 3, 30, 13
    w, (F, M, S) = _random_cell(H, 7)
    cell = mpuc.MpucCellWeights(w, cuda_device)
    g = torch.Generator().manual_seed(8)
    ins = [torch.randn((B, T, n), generator=g).to(cuda_device) for n in (F, M, S)]
    a = mpuc.recurrent_scan(cell, *ins)
    b = mpuc.recurrent_scan(cell, *ins)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    first = mpuc.recurrent_scan(cell, *(x[:, :T1].contiguous() for x in ins))
    second = mpuc.recurrent_scan(cell, *(x[:, T1:].contiguous() for x in ins), state=first[2:])
    assert torch.equal(torch.cat([first[0], second[0]], dim=1), a[0])
    assert torch.equal(torch.cat([first[1], second[1]], dim=1), a[1])
    for x, y in zip(second[2:], a[2:]):
        assert torch.equal(x, y)


def test_scan_rejects_bad_shapes(cuda_device):
    w, (F, M, S) = _random_cell(64, 9)
    cell = mpuc.MpucCellWeights(w, cuda_device)
    x = torch.zeros((2, 5, F), device=cuda_device)
    with pytest.raises(ValueError):
        mpuc.recurrent_scan(cell, x, torch.zeros((2, 5, M + 1), device=cuda_device), torch.zeros((2, 5, S),
                                                                                                device=cuda_device))
    with pytest.raises(RuntimeError):
        mpuc.recurrent_scan(cell, x.cpu(), torch.zeros((2, 5, M)), torch.zeros((2, 5, S)))
    w2 = dict(w)
    w2["fast_gate_w"] = w["fast_gate_w"][:, :-2]
    with pytest.raises(ValueError):
        mpuc.MpucCellWeights(w2, cuda_device)
