"""Multi-rank paths with the sm_100a kernels.  Two ranks share cuda:0 through
gloo (collectives staged on the host, no kernel waits on another rank), so the
test runs on one GPU; the block-range-sharded readout must equal the
single-rank readout bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gfst_hmb_public_b200 import readout, retrieval, sharding

pytestmark = pytest.mark.gpu


def test_topk_merge_kernel(cuda_device):
    g = torch.Generator().manual_seed(3)
    s = torch.randn((50, 24), generator=g)
    i = torch.randperm(1000, generator=g)[:24].repeat(50, 1).to(torch.int32)
    s[0, :5] = 2.0  # ties: lowest index first
    i[0, :5] = torch.tensor([9, 3, 7, 1, 5], dtype=torch.int32)
    i[1, 3] = -1
    s[2, 4] = float("nan")
    out_s, out_i = retrieval.topk_merge(s.to(cuda_device), i.to(cuda_device), 4)
    for r in range(50):
        cand = sorted((-float(s[r, c]), int(i[r, c])) for c in range(24)
                      if int(i[r, c]) >= 0 and not np.isnan(float(s[r, c])))[:4]
        assert out_i[r].tolist() == [c[1] for c in cand]
    assert out_i[0].tolist() == [1, 3, 5, 7]


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _data(device, S=3):
    g = torch.Generator().manual_seed(11)
    NB, L, d, Nq, k = 40, 64, 128, 100, 8
    pool = torch.randn((S, NB, L, d), generator=g).to(torch.bfloat16)
    vals = torch.randn((S, NB, L, d), generator=g).to(torch.bfloat16)
    vals[..., :2] = -0.0  # signed zeros in every value row: the exchanges must keep the sign bit
    needles = torch.randint(0, NB * L, (S, Nq), generator=g)
    flat = pool.reshape(S, NB * L, d).float()
    Q = (flat[torch.arange(S)[:, None], needles] + 0.1 * torch.randn((S, Nq, d), generator=g)).to(torch.bfloat16)
    summary = pool.float().mean(dim=2).to(torch.bfloat16)
    return [t.to(device) for t in (pool, vals, Q, summary)] + [k]


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pool, vals, Q, summary, k = _data(torch.device("cuda:0"))
        shard = sharding.BlockRange(rank, world, pool.shape[1])
        sl = slice(shard.lo, shard.hi)
        res = sharding.sharded_readout(Q, summary[:, sl].contiguous(), pool[:, sl].contiguous(),
                                       vals[:, sl].contiguous(), k, shard)
        torch.cuda.synchronize()
        torch.save([t.cpu() for t in res], f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_block_range_sharded_readout_two_ranks(cuda_device, tmp_path):
    world = 2
    out = str(tmp_path / "res")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    pool, vals, Q, summary, k = _data(cuda_device)
    ref_s, ref_i = retrieval.block_topk(Q, summary, k)
    ref_t, ref_bs, ref_v = readout.exact_readout(Q, pool, vals, ref_i)
    for r in range(world):
        best_t, best_s, value, top_i, top_s = torch.load(f"{out}.{r}")
        assert torch.equal(top_i, ref_i.cpu())
        assert torch.equal(top_s, ref_s.cpu())
        assert torch.equal(best_t, ref_t.cpu())
        assert torch.equal(best_s, ref_bs.cpu())
        assert torch.equal(value, ref_v.cpu())


def _bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


def _nccl_worker(rank, world, port, out_path, layout, n_committed, S):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        pool, vals, Q, summary, k = _data(dev, S)
        if n_committed is not None:
            pool[:, n_committed:] = 0
            vals[:, n_committed:] = 0
            summary[:, n_committed:] = 0
        shard = sharding.BlockRange(rank, world, pool.shape[1])
        sl = slice(shard.lo, shard.hi)
        n_valid = None if n_committed is None else max(0, min(n_committed, shard.hi) - shard.lo)
        timings = {}
        res = sharding.sharded_readout(Q, summary[:, sl].contiguous(), pool[:, sl].contiguous(),
                                       vals[:, sl].contiguous(), k, shard, n_valid=n_valid, value_layout=layout,
                                       timings=timings)
        torch.cuda.synchronize(dev)
        assert set(timings) == {"local_topk", "gather_candidates", "merge", "readout", "gather_winners",
                                "value_exchange"}
        torch.save([t.cpu() for t in res], f"{out_path}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("layout,n_committed,S", [("replicated", None, 3), ("stream_shard", None, 3),
                                                  ("stream_shard", None, 4), ("replicated", 27, 3),
                                                  ("stream_shard", 27, 4)])
def test_block_range_sharded_readout_nccl_two_gpus(cuda_device, tmp_path, layout, n_committed, S):
    # one rank per GPU over NCCL: all-gather of candidates and winners, then the
    # winners' value rows from their owners (an odd stream count: one
    # all-to-all; an even one: one reduce-scatter); equal to the single-GPU
    # readout bit for bit, signed zeros included (on a part-filled memory: the
    # readout of its committed blocks)
    world = 2
    out = str(tmp_path / "nccl")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), out, layout, n_committed, S), nprocs=world,
                       start_method="spawn")
    pool, vals, Q, summary, k = _data(cuda_device, S)
    nb = pool.shape[1] if n_committed is None else n_committed
    ref_s, ref_i = retrieval.block_topk(Q, summary, k, n_blocks=nb)
    ref_t, ref_bs, ref_v = readout.exact_readout(Q, pool, vals, ref_i)
    S = Q.shape[0]
    for r in range(world):
        best_t, best_s, value, top_i, top_s = torch.load(f"{out}.{r}")
        assert torch.equal(top_i, ref_i.cpu())
        assert torch.equal(top_s, ref_s.cpu())
        assert torch.equal(best_t, ref_t.cpu())
        assert torch.equal(best_s, ref_bs.cpu())
        if layout == "replicated":
            assert torch.equal(_bits(value), _bits(ref_v.cpu()))
        else:
            lo, hi = sharding.stream_shard(S, r, world)
            assert torch.equal(_bits(value), _bits(ref_v.cpu()[lo:hi]))


def _exchange_case():
    g = torch.Generator().manual_seed(3)
    world, S, Nq, dv = 2, 6, 5, 16
    bv = torch.randn((world, S, Nq, dv), generator=g).to(torch.bfloat16)  # each rank's local best rows
    bv[..., :3] = -0.0
    best_t = torch.randint(-1, 40, (S, Nq), generator=g)
    best_t[0, :2] = -1                                                    # queries with no winner
    owner = torch.where(best_t >= 0, (best_t // 7) % world, torch.full_like(best_t, -1))
    return world, bv, best_t, owner


def _nccl_exchange_worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        _, bv, best_t, owner = _exchange_case()
        v = sharding._reduce_scatter_to_stream_shards(bv[rank].to(dev), best_t.to(dev), (owner == rank).to(dev),
                                                      rank, world, None)
        torch.cuda.synchronize(dev)
        torch.save(v.cpu(), f"{out_path}.{rank}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_reduce_scatter_value_delivery_keeps_every_bit(cuda_device, tmp_path):
    # the reduce-scatter delivery: every found winner's row from its owner bit
    # for bit (-0.0 entries included), +0.0 rows for queries without a winner
    world, bv, best_t, owner = _exchange_case()
    out = str(tmp_path / "rs")
    mp.start_processes(_nccl_exchange_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    S = best_t.shape[0]
    want = torch.zeros_like(bv[0])
    for r in range(world):
        want = torch.where((owner == r)[..., None], bv[r], want)
    for r in range(world):
        lo, hi = sharding.stream_shard(S, r, world)
        got = torch.load(f"{out}.{r}")
        assert torch.equal(_bits(got), _bits(want[lo:hi]))
        assert not torch.signbit(got[best_t[lo:hi] < 0].float()).any()
