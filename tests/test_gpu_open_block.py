"""Open-block readout (gfst_open_block_readout) against the oracle.

The kernel merges the readout over the open block's prefix into the result of
the committed-block readout.  The oracle scores both candidate sets together
in float64 (oracle.gfst_oracle.exact_readout with the open block).

Bars: the best token bit-exact wherever the oracle's margin to the runner-up
exceeds 1e-3 relative; its score within 1e-5 relative (fp32 sums against
float64); the value row an exact copy of the winner's row.
"""
import numpy as np
import pytest
import torch

from gfst_hmb_public_b200 import readout
from oracle import gfst_oracle as go

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def _case(dev, dtype, S, Nq, Lo, d, dv, *, NB=6, Lc=16, k=3, rule=True, seed=0, nan_rows=False, ties=False,
          no_value=False, empty_sel_frac=0.2):
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn((S, Nq, d), generator=g).to(dtype)
    K_open = torch.randn((S, Lo, d), generator=g).to(dtype)
    V_open = torch.randn((S, Lo, dv), generator=g).to(dtype)
    pool_K = torch.randn((S, NB, Lc, d), generator=g).to(dtype)
    pool_V = torch.randn((S, NB, Lc, dv), generator=g).to(dtype)
    top_idx = torch.randint(0, NB, (S, Nq, k), generator=g, dtype=torch.int32)
    drop = torch.rand((S, Nq), generator=g) < empty_sel_frac
    top_idx[drop] = -1  # nothing committed for these queries
    if ties:
        # open position 1 repeats the committed block's token 3 and position 4
        # repeats position 2: equal scores must resolve to the lower index
        K_open[:, 1] = pool_K[:, 0, 3]
        K_open[:, 4] = K_open[:, 2]
    if nan_rows:
        K_open[:, 0] = float("nan")
    open_len = None
    if rule:
        lens = np.broadcast_to(go.streaming_open_len(Nq, Lo), (S, Nq)).copy()
    else:
        open_len = torch.randint(-2, Lo + 3, (S, Nq), generator=g, dtype=torch.int32)
        lens = np.clip(open_len.numpy(), 0, Lo)
    base = NB * Lc
    dQ, dKo, dVo, dK, dV, dsel = (t.to(dev) for t in (Q, K_open, V_open, pool_K, pool_V, top_idx))
    if no_value:
        bt, bs, ov = readout.exact_readout(dQ, dK, None, dsel)
        readout.open_block_readout(dQ, dKo, None, bt, bs, None, open_base=base,
                                   open_len=None if open_len is None else open_len.to(dev))
    else:
        bt, bs, ov = readout.exact_readout(dQ, dK, dV, dsel)
        readout.open_block_readout(dQ, dKo, dVo, bt, bs, ov, open_base=base,
                                   open_len=None if open_len is None else open_len.to(dev))
    torch.cuda.synchronize()
    rt, rs, rv, ok = go.exact_readout(_np(Q), _np(pool_K), None if no_value else _np(pool_V), top_idx.numpy(),
                                      _np(K_open), None if no_value else _np(V_open), lens, base)
    got_t, got_s = bt.cpu().numpy(), bs.cpu().numpy()
    assert np.array_equal(got_t[ok], rt[ok])
    valid = ok & (rt >= 0)
    assert np.allclose(got_s[valid], rs[valid], rtol=1e-5, atol=1e-5)
    if not no_value:
        same = got_t == rt
        assert np.array_equal(_np(ov)[same], rv[same])
    return got_t, rt, lens


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("S,Nq,Lo,d,dv", [(4, 64, 64, 128, 128), (3, 16, 16, 64, 64), (2, 100, 100, 256, 32),
                                         (5, 1, 1, 8, 8), (2, 130, 64, 128, 64)])
def test_open_block_streaming_rule(cuda_device, dtype, S, Nq, Lo, d, dv):
    got, ref, lens = _case(cuda_device, dtype, S, Nq, Lo, d, dv, rule=True, seed=S * 100 + Nq)
    # open tokens win only where the query's prefix is open (never at the
    # block's last position or beyond)
    assert ((got >= 6 * 16) <= (lens > 0)).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_open_block_explicit_lengths(cuda_device, dtype):
    got, ref, lens = _case(cuda_device, dtype, 6, 96, 80, 128, 128, rule=False, seed=11)
    assert (lens == 0).any() and (lens == 80).any()


def test_open_block_ties_and_nan(cuda_device):
    got, ref, lens = _case(cuda_device, torch.float32, 4, 64, 64, 64, 64, rule=True, seed=5, ties=True,
                           nan_rows=True, empty_sel_frac=0.0)
    base = 6 * 16
    # NaN keys at position 0 never win; position 4 never wins over its twin at 2
    assert not (got == base + 0).any()
    assert not (got == base + 4).any()


def test_open_block_without_values(cuda_device):
    _case(cuda_device, torch.bfloat16, 3, 64, 64, 128, 128, rule=True, seed=9, no_value=True)


def test_open_block_argument_checks(cuda_device):
    dev = cuda_device
    Q = torch.randn((2, 4, 64), device=dev)
    K = torch.randn((2, 4, 64), device=dev)
    bt = torch.full((2, 4), -1, dtype=torch.int32, device=dev)
    bs = torch.full((2, 4), float("-inf"), device=dev)
    with pytest.raises(RuntimeError):
        readout.open_block_readout(Q, K.to(torch.bfloat16), None, bt, bs, None, open_base=0)
    with pytest.raises(RuntimeError):
        readout.open_block_readout(Q, K, None, bt, bs, None, open_base=(1 << 31) - 2)
    with pytest.raises(RuntimeError):
        readout.open_block_readout(Q[:, :, :62], K[:, :, :62], None, bt, bs, None, open_base=0)
    with pytest.raises(RuntimeError):
        readout.open_block_readout(Q.cpu(), K.cpu(), None, bt.cpu(), bs.cpu(), None, open_base=0)
