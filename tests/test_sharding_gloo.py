"""Multi-rank logic on CPU: block-range-sharded readout with world_size 2 gloo
ranks, driven by the CPU oracle in place of the kernels, must equal the
unsharded readout; stream sharding covers every stream exactly once."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gfst_hmb_public_b200 import sharding


def test_stream_shard_partition():
    for n in (1, 7, 2048, 2049):
        for world in (1, 2, 3, 8):
            spans = [sharding.stream_shard(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


class OracleOps:
    """The oracle in place of the kernels (CPU tensors in and out)."""

    @staticmethod
    def block_topk(Q, Ksum, k, n_blocks=None):
        from oracle import gfst_oracle as go

        nb = Ksum.shape[1] if n_blocks is None else n_blocks
        s, i, _ = go.block_topk(Q.numpy(), Ksum[:, :nb].numpy(), k)
        return torch.from_numpy(s), torch.from_numpy(i)

    @staticmethod
    def merge(scores, idx, k):
        s = scores.numpy().astype(np.float64)
        i = idx.numpy().astype(np.int64)
        out_s = np.full(s.shape[:-1] + (k,), -np.inf, np.float32)
        out_i = np.full(s.shape[:-1] + (k,), -1, np.int32)
        for pos in np.ndindex(*s.shape[:-1]):
            cand = [(-s[pos][c], i[pos][c]) for c in range(s.shape[-1]) if i[pos][c] >= 0 and s[pos][c] > -np.inf]
            for j, (ns, ii) in enumerate(sorted(cand)[:k]):
                out_s[pos + (j,)] = -ns
                out_i[pos + (j,)] = ii
        return torch.from_numpy(out_s), torch.from_numpy(out_i)

    @staticmethod
    def exact_readout(Q, pool_K, pool_V, sel):
        from oracle import gfst_oracle as go

        t, s, v, _ = go.exact_readout(Q.numpy(), pool_K.numpy(), pool_V.numpy(), sel.numpy())
        return torch.from_numpy(t), torch.from_numpy(s), torch.from_numpy(v)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    g = torch.Generator().manual_seed(5)
    S, NB, L, d, Nq, k = 3, 12, 8, 16, 6, 3
    pool = torch.randn((S, NB, L, d), generator=g)
    vals = torch.randn((S, NB, L, d), generator=g)
    Q = torch.randn((S, Nq, d), generator=g)
    summary = pool.mean(dim=2)
    return pool, vals, Q, summary, k


def _worker(rank, world, port, out_path, n_committed, layout):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pool, vals, Q, summary, k = _data()
        if n_committed is not None:  # slots past the committed blocks hold nothing (zeros)
            pool[:, n_committed:] = 0
            vals[:, n_committed:] = 0
            summary[:, n_committed:] = 0
        shard = sharding.BlockRange(rank, world, pool.shape[1])
        sl = slice(shard.lo, shard.hi)
        n_valid = None if n_committed is None else max(0, min(n_committed, shard.hi) - shard.lo)
        res = sharding.sharded_readout(Q, summary[:, sl].contiguous(), pool[:, sl].contiguous(),
                                       vals[:, sl].contiguous(), k, shard, ops=OracleOps, n_valid=n_valid,
                                       value_layout=layout)
        torch.save([t for t in res], f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_committed,layout", [(2, None, "replicated"), (2, None, "stream_shard"),
                                                      (2, 7, "replicated"), (3, 5, "stream_shard")])
def test_block_range_sharded_readout_equals_unsharded(tmp_path, world, n_committed, layout):
    out = str(tmp_path / "res")
    mp.start_processes(_worker, args=(world, _free_port(), out, n_committed, layout), nprocs=world,
                       start_method="spawn")
    pool, vals, Q, summary, k = _data()
    nb = pool.shape[1] if n_committed is None else n_committed
    ref_ts, ref_ti = OracleOps.block_topk(Q, summary, k, n_blocks=nb)
    ref_t, ref_s, ref_v = OracleOps.exact_readout(Q, pool, vals, ref_ti)
    S = Q.shape[0]
    for r in range(world):
        best_t, best_s, value, top_i, top_s = torch.load(f"{out}.{r}")
        assert torch.equal(top_i.to(torch.int32), ref_ti.to(torch.int32))
        assert torch.equal(best_t.to(torch.int32), ref_t.to(torch.int32))
        assert torch.allclose(best_s, ref_s)
        if layout == "replicated":
            assert torch.equal(value, ref_v)
        else:
            lo, hi = sharding.stream_shard(S, r, world)
            assert torch.equal(value, ref_v[lo:hi])


def test_owner_of_matches_block_ranges():
    for n_blocks in (1, 5, 12, 8192, 8195):
        for world in (1, 2, 3, 8):
            L = 4
            tok = torch.arange(-1, n_blocks * L)
            own = sharding._owner_of(tok, L, n_blocks, world)
            assert own[0] == -1
            for r in range(world):
                br = sharding.BlockRange(r, world, n_blocks)
                sel = own[1:] == r
                blocks = torch.unique(tok[1:][sel] // L)
                assert blocks.numel() == br.size
                if br.size:
                    assert int(blocks.min()) == br.lo and int(blocks.max()) == br.hi - 1
