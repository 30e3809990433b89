"""Multi-GPU layouts of the hot path.

Two partitions, one process per GPU over ``torch.distributed`` (NCCL on NVLink):

* Stream sharding -- the (batch, head) streams are independent: every rank owns
  a batch shard with its own frames and block memory; nothing is exchanged on
  the data path (``stream_shard``).

* Block-range sharding of a long memory -- every rank holds blocks [lo, hi) of
  every stream (pool slab and summaries).  A readout is one exchange step:
    1. local score GEMM + top-k over the rank's summaries (tensor cores);
    2. all-gather of the (score, global block) candidates, then the same
       deterministic merge on every rank -> the global top-k;
    3. each rank scores the tokens of the global top-k blocks it owns;
    4. all-gather of the per-rank best (score, global token) and a merge ->
       the winner; the owner's value row is combined with an all-reduce in
       which every other rank contributes zeros (an exact sum).
  The result equals the single-GPU readout: scores of a (query, block) pair do
  not depend on which rank computes them, and the merges use the same total
  order (score descending, index ascending).

The reference runs on one device (no distributed code); these layouts are new.
The collective and merge logic is written against an ``ops`` object so the
CPU tests can drive it with gloo ranks and the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def stream_shard(n_total: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of ``n_total`` independent streams owned by ``rank`` (even split,
    the first n_total % world ranks take one extra)."""
    base, extra = divmod(n_total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class BlockRange:
    rank: int
    world: int
    n_blocks: int

    @property
    def lo(self) -> int:
        return stream_shard(self.n_blocks, self.rank, self.world)[0]

    @property
    def hi(self) -> int:
        return stream_shard(self.n_blocks, self.rank, self.world)[1]

    @property
    def size(self) -> int:
        return self.hi - self.lo


class GpuOps:
    """The sm_100a kernels."""

    @staticmethod
    def block_topk(Q, Ksum, k):
        from . import retrieval
        return retrieval.block_topk(Q, Ksum, k)

    @staticmethod
    def merge(scores, idx, k):
        from . import retrieval
        return retrieval.topk_merge(scores, idx, k)

    @staticmethod
    def exact_readout(Q, pool_K, pool_V, sel):
        from . import readout
        return readout.exact_readout(Q, pool_K, pool_V, sel)


def _gather_pairs(scores: torch.Tensor, idx: torch.Tensor, group=None):
    """All-gather (score, index) tensors [..., c] from every rank and concatenate
    along the last axis in rank order -> [..., world * c]."""
    world = dist.get_world_size(group)
    packed = torch.stack((scores.to(torch.float32), idx.to(torch.int32).view(torch.float32)), dim=-1).contiguous()
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    allp = torch.cat(parts, dim=-2)
    return allp[..., 0].contiguous(), allp[..., 1].contiguous().view(torch.int32)


def sharded_readout(Q: torch.Tensor, summary: torch.Tensor, pool_K: torch.Tensor, pool_V: torch.Tensor | None,
                    k: int, shard: BlockRange, *, ops=GpuOps, group=None):
    """Readout against a block-range-sharded memory.  This rank's summary /
    pool_K / pool_V hold blocks [shard.lo, shard.hi) of every stream
    (summary [S, size, d], pools [S, size, L, d]).  Returns (best_tok [S, Nq]
    global token index, best_score, value [S, Nq, dv] or None, top_idx [S, Nq, k]
    global block indices, top_scores) -- identical on every rank."""
    L = pool_K.shape[2]
    # 1. local candidates
    ls, li = ops.block_topk(Q, summary, k)
    gi = torch.where(li >= 0, li + shard.lo, li)
    # 2. gather and merge -> global top-k
    cs, ci = _gather_pairs(ls, gi, group)
    top_s, top_i = ops.merge(cs, ci, k)
    # 3. exact readout over the owned part of the global top-k
    own = (top_i >= shard.lo) & (top_i < shard.hi)
    local_sel = torch.where(own, top_i - shard.lo, torch.full_like(top_i, -1)).to(torch.int32)
    bt, bs, bv = ops.exact_readout(Q, pool_K, pool_V, local_sel)
    gt = torch.where(bt >= 0, bt + shard.lo * L, bt)
    # 4. gather per-rank winners, merge -> global winner
    ws, wi = _gather_pairs(bs.unsqueeze(-1), gt.unsqueeze(-1), group)
    best_s, best_t = ops.merge(ws, wi, 1)
    best_s, best_t = best_s[..., 0], best_t[..., 0]
    value = None
    if pool_V is not None:
        mine = (gt == best_t) & (best_t >= 0)
        value = torch.where(mine.unsqueeze(-1), bv, torch.zeros_like(bv))
        dist.all_reduce(value, group=group)  # one non-zero contribution per row: exact
    return best_t, best_s, value, top_i, top_s
