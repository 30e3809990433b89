"""The host-buffer pipeline (the end-to-end path: inputs in pinned host memory,
uploaded on a copy stream while the previous step computes, results copied
back) gives exactly what the streaming step gives on device-resident inputs.

Bar: bit-exact -- the same kernels run on the same bytes; only where the bytes
come from differs.
"""
import pytest
import torch

from gfst_hmb_public_b200 import workloads as wl
from gfst_hmb_public_b200.step import HostPipeline, StreamingStep

pytestmark = pytest.mark.gpu


def _inputs(S, L, d, r, m, step, device):
    g = torch.Generator(device="cpu").manual_seed(100 + step)
    A = torch.randn((S, L, d, m), generator=g) / d ** 0.5
    B = torch.randn((S, L, r, m), generator=g) / d ** 0.5
    K, V, Q = (torch.randn((S, L, d), generator=g).to(torch.bfloat16) for _ in range(3))
    return [t.to(device) for t in (A, B, K, V, Q)]


def _make(S, d, r, L, n_slots, k, device):
    st = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, device=device)
    U0 = wl.random_orthonormal_frames(S, d, r, seed=7, device=device)
    st.set_frames(U0)
    return st


def test_host_pipeline_matches_device_steps(cuda_device):
    S, d, r, L, n_slots, k, m, n_steps = 12, 128, 32, 64, 6, 4, 4, 5
    steps = [_inputs(S, L, d, r, m, i, cuda_device) for i in range(n_steps)]
    ref = _make(S, d, r, L, n_slots, k, cuda_device)
    want = []
    for x in steps:
        out = ref.step(*x)
        want.append((out.best_tok.clone(), out.best_score.clone(), out.value.clone()))
    torch.cuda.synchronize()

    st = _make(S, d, r, L, n_slots, k, cuda_device)
    host_in = [[t.cpu().pin_memory() for t in x] for x in steps]
    host_out = [(torch.empty((S, L), dtype=torch.int32).pin_memory(),
                 torch.empty((S, L), dtype=torch.float32).pin_memory(),
                 torch.empty((S, L, d), dtype=torch.bfloat16).pin_memory()) for _ in range(n_steps)]
    pipe = HostPipeline(st, steps[0])
    pipe.run(host_in, host_out)
    torch.cuda.synchronize()
    for (tok, score, value), (wt, ws, wv) in zip(host_out, want):
        assert torch.equal(tok, wt.cpu())
        assert torch.equal(score, ws.cpu())
        assert torch.equal(value, wv.cpu())
    assert torch.equal(st.U.cpu(), ref.U.cpu())
    # the frames are still orthonormal after five 64-token blocks
    eye = torch.eye(r)
    assert (st.U.cpu().transpose(1, 2) @ st.U.cpu() - eye).abs().max() < 1e-5


@pytest.mark.parametrize("shape", ["small_fp32", "mid_bf16"])
def test_graph_captured_pass_matches_eager_pass(cuda_device, shape):
    # a whole pass (empty ring -> frames -> one step per block) captured once
    # as a CUDA graph and replayed twice gives, bit for bit, what the eager
    # pass gives; the ring wraps in the bf16 case (6 blocks into 4 slots)
    from gfst_hmb_public_b200.step import StreamingPass

    if shape == "small_fp32":
        S, d, r, m, L, n_slots, k, n_blk, dt = 8, 64, 8, 1, 16, 16, 2, 5, torch.float32
    else:
        S, d, r, m, L, n_slots, k, n_blk, dt = 10, 128, 16, 2, 64, 4, 3, 6, torch.bfloat16
    g = torch.Generator().manual_seed(55)
    blocks = []
    for _ in range(n_blk):
        A = torch.randn((S, L, d, m), generator=g) / d ** 0.5
        B = torch.randn((S, L, r, m), generator=g) / d ** 0.5
        K, V, Q = (torch.randn((S, L, d), generator=g).to(dt) for _ in range(3))
        blocks.append(tuple(t.to(cuda_device) for t in (A, B, K, V, Q)))
    U0 = wl.random_orthonormal_frames(S, d, r, seed=56, device=cuda_device)

    eager = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, dtype=dt, device=cuda_device)
    eager.set_frames(U0)
    want = []
    for blk in blocks:
        o = eager.step(*blk)
        want.append([t.clone() for t in (o.best_tok, o.best_score, o.value, o.top_idx)])
    torch.cuda.synchronize()

    st = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, dtype=dt, device=cuda_device)
    sp = StreamingPass(st, U0, blocks)
    for _ in range(2):
        outs = sp.replay()
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            for got, exp in zip((o.best_tok, o.best_score, o.value, o.top_idx), w):
                assert torch.equal(got, exp)
        assert torch.equal(st.U, eager.U)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_multi_block_run_matches_consecutive_steps(cuda_device, dt):
    # StreamingStep.run enqueues the frame chain and the memory chain of
    # several blocks on their own streams with no join between blocks; its
    # results equal those of one step() per block, bit for bit, through a
    # ring wrap (7 blocks into 4 slots) and a second call that continues
    S, d, r, m, L, n_slots, k = 9, 128, 32, 4, 64, 4, 3
    g = torch.Generator().manual_seed(71)
    blocks = []
    for _ in range(7):
        A = torch.randn((S, L, d, m), generator=g) / d ** 0.5
        B = torch.randn((S, L, r, m), generator=g) / d ** 0.5
        K, V, Q = (torch.randn((S, L, d), generator=g).to(dt) for _ in range(3))
        blocks.append(tuple(t.to(cuda_device) for t in (A, B, K, V, Q)))
    U0 = wl.random_orthonormal_frames(S, d, r, seed=72, device=cuda_device)
    a = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, dtype=dt, device=cuda_device)
    b = StreamingStep(S, d=d, r=r, block_len=L, n_slots=n_slots, k=k, dtype=dt, device=cuda_device)
    a.set_frames(U0)
    b.set_frames(U0)
    want = [a.step(*blk) for blk in blocks]
    got = b.run(blocks[:5]) + b.run(blocks[5:])
    torch.cuda.synchronize()
    assert len(got) == len(want)
    for o, w in zip(got, want):
        for x, y in zip((o.best_tok, o.best_score, o.value, o.top_idx), (w.best_tok, w.best_score, w.value,
                                                                          w.top_idx)):
            assert torch.equal(x, y)
        assert o.slot == w.slot and o.open_base == w.open_base
    assert torch.equal(a.U, b.U)
    assert b.run([]) == []
