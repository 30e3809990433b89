"""The whole streaming step against the token-by-token oracle.

``StreamingStep`` runs a block of L tokens per call (frames kernel, top-k over
the committed summaries, readout over the selected blocks, open-block merge,
commit).  ``oracle.gfst_oracle.streaming_pass`` composes the same pieces one
token at a time in the reference's order (frame update + QR, exact-store
append, retrieval over the committed summaries, readout over the selected
blocks and the open prefix, summary append after the block's last token), so
this pins which memory each query sees, not just each kernel.

Workloads: the CPU-runnable configuration (2 batch x 4 heads, 256 tokens,
64 x 8 frames, rank 1, L=16, 16 blocks, top-2, fp32) and a slice of the
mid-scale one (8 streams, 512 tokens, 128 x 16 frames, rank 2, L=64, 64 slots,
top-4, bf16), plus the same slice in a 3-slot ring that wraps.

Bars: frames within 1e-5 orthogonality error and
1e-4 principal-angle distance of the oracle's fp32 frames at every block end;
selected blocks bit-exact wherever the oracle's k-th / (k+1)-th margin exceeds
1e-3 relative; the best token bit-exact wherever, in addition, the readout
margin exceeds 1e-3 relative; the value row an exact copy of the winner's.
"""
import math

import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import workloads as wl
from gfst_hmb_public_b200.step import StreamingStep
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu


def _inputs(S, T, d, r, m, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    std = 1.0 / math.sqrt(d)
    U0 = wl.random_orthonormal_frames(S, d, r, seed=seed + 1)
    A = torch.randn((S, T, d, m), generator=g) * std
    B = torch.randn((S, T, r, m), generator=g) * std
    K, V, Q = (torch.randn((S, T, d), generator=g).to(dtype) for _ in range(3))
    return U0, A, B, K, V, Q


def _run(dev, S, T, d, r, m, L, n_slots, k, dtype, seed):
    U0, A, B, K, V, Q = _inputs(S, T, d, r, m, dtype, seed)
    st = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, dtype=dtype, device=dev)
    st.set_frames(U0.to(dev))
    got = {"best_tok": [], "best_score": [], "value": [], "top_idx": [], "frames": []}
    for b in range(T // L):
        sl = slice(b * L, (b + 1) * L)
        out = st.step(*(x[:, sl].contiguous().to(dev) for x in (A, B, K, V, Q)))
        got["best_tok"].append(out.best_tok.cpu())
        got["best_score"].append(out.best_score.cpu())
        got["value"].append(out.value.float().cpu())
        got["top_idx"].append(out.top_idx.cpu())
        got["frames"].append(st.U.cpu().clone())
        assert out.open_base == n_slots * L and out.slot == b % n_slots
    torch.cuda.synchronize()
    got = {key: torch.stack(v, 1) if key == "frames" else torch.cat(v, 1) for key, v in got.items()}
    f = lambda x: x.float().numpy()  # noqa: E731
    ref = go.streaming_pass(f(U0), f(A), f(B), f(K), f(V), f(Q), block_len=L, n_slots=n_slots, k=k,
                            memory_bf16=dtype == torch.bfloat16)
    return {key: v.numpy() for key, v in got.items()}, ref


def _check(got, ref, L):
    top_ok = ref["top_ok"]
    assert np.array_equal(got["top_idx"][top_ok], ref["top_idx"][top_ok])
    ok = top_ok & ref["read_ok"]
    assert ok.mean() > 0.9  # the bars bind on almost every query
    assert np.array_equal(got["best_tok"][ok], ref["best_tok"][ok])
    valid = ok & (ref["best_tok"] >= 0)
    assert np.allclose(got["best_score"][valid], ref["best_score"][valid], rtol=1e-5, atol=1e-4)
    same = got["best_tok"] == ref["best_tok"]
    assert np.array_equal(got["value"][same], ref["value"][same])
    # frames at every block end
    T = ref["frames"].shape[1]
    ends = ref["frames"][:, L - 1::L]
    assert ends.shape[1] == T // L
    for b in range(T // L):
        q = got["frames"][:, b]
        assert go.orthogonality_error(q).max() <= 1e-5
        assert go.max_prefix_subspace_distance(q, ends[:, b]).max() <= 1e-4
    # the open block is part of the readout: some queries are answered from it
    assert (got["best_tok"] >= got["open_base"]).any()


def test_step_cpu_runnable_configuration(cuda_device):
    spec = wl.STREAM_SMALL
    got, ref = _run(cuda_device, spec.streams, spec.tokens, spec.d, spec.r, spec.m, spec.block_len, spec.n_blocks,
                    spec.k, torch.float32, spec.seed)
    got["open_base"] = spec.n_blocks * spec.block_len
    _check(got, ref, spec.block_len)
    # no committed block for the first block's queries: open prefix or nothing
    L = spec.block_len
    assert (got["top_idx"][:, :L] == -1).all()
    assert (got["best_tok"][:, L - 1] == -1).all()


def test_step_mid_scale_slice(cuda_device):
    spec = wl.STREAM_MID
    S, T = 8, 512
    got, ref = _run(cuda_device, S, T, spec.d, spec.r, spec.m, spec.block_len, spec.n_blocks, spec.k,
                    torch.bfloat16, spec.seed)
    got["open_base"] = spec.n_blocks * spec.block_len
    _check(got, ref, spec.block_len)


def test_step_ring_wraps(cuda_device):
    spec = wl.STREAM_MID
    S, T, n_slots = 6, 512, 3
    got, ref = _run(cuda_device, S, T, spec.d, spec.r, spec.m, spec.block_len, n_slots, spec.k, torch.bfloat16,
                    spec.seed + 5)
    got["open_base"] = n_slots * spec.block_len
    _check(got, ref, spec.block_len)
    # after the wrap, selections name ring slots below n_slots only
    assert got["top_idx"].max() < n_slots
