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
       the winner, identical on every rank;
    5. value exchange: the winner's owner is known on every rank (its block
       range), so only owners send value rows -- either all-gathered
       ("replicated": every rank gets every row) or delivered to the rank that
       owns the query's stream ("stream_shard": each rank gets the rows of its
       own stream shard).  Counts follow from the winners, so no sizes are
       exchanged.  For equal stream shards over NCCL the stream-shard delivery
       is one reduce-scatter: each rank contributes the rows it owns and -0.0
       elsewhere (x + -0.0 = x for every x, so the sum is the owner's row bit
       for bit), with no host synchronisation and no sorting; otherwise one
       all-to-all of the owned rows, split sizes counted on the device.
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
    def block_topk(Q, Ksum, k, n_blocks=None):
        from . import retrieval
        return retrieval.block_topk(Q, Ksum, k, n_blocks=n_blocks)

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
    if dist.get_backend(group) == "nccl":  # one buffer, one collective
        buf = torch.empty((world,) + tuple(packed.shape), dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(buf, packed, group=group)
        parts = list(buf.unbind(0))
    else:
        parts = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(parts, packed, group=group)
    allp = torch.cat(parts, dim=-2)
    return allp[..., 0].contiguous(), allp[..., 1].contiguous().view(torch.int32)


class _PhaseTimer:
    """CUDA events between the phases of one sharded readout (current stream)."""

    def __init__(self, out: dict | None, enabled: bool):
        self.out = out if enabled else None
        self.marks: list = []

    def mark(self, name: str) -> None:
        if self.out is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.marks.append((name, e))

    def finish(self) -> None:
        if self.out is None or len(self.marks) < 2:
            return
        self.marks[-1][1].synchronize()
        for (_, e0), (name, e1) in zip(self.marks, self.marks[1:]):
            self.out[name] = self.out.get(name, 0.0) + e0.elapsed_time(e1)


def _owner_of(tok: torch.Tensor, L: int, n_blocks: int, world: int) -> torch.Tensor:
    """Rank owning each global token index (-1 for none) under BlockRange."""
    blk = torch.where(tok >= 0, tok // L, torch.zeros_like(tok)).to(torch.int64)
    base, extra = divmod(n_blocks, world)
    # ranks < extra hold base + 1 blocks, the rest base blocks
    cut = extra * (base + 1)
    own = torch.where(blk < cut, blk // (base + 1), extra + (blk - cut) // max(base, 1))
    return torch.where(tok >= 0, own, torch.full_like(own, -1))


def sharded_readout(Q: torch.Tensor, summary: torch.Tensor, pool_K: torch.Tensor, pool_V: torch.Tensor | None,
                    k: int, shard: BlockRange, *, ops=GpuOps, group=None, n_valid: int | None = None,
                    value_layout: str = "replicated", timings: dict | None = None):
    """Readout against a block-range-sharded memory.  This rank's summary /
    pool_K / pool_V hold blocks [shard.lo, shard.hi) of every stream
    (summary [S, size, d], pools [S, size, L, d]); ``n_valid`` of them (its
    first slots; default all) hold committed blocks.  Returns (best_tok
    [S, Nq] global token index, best_score, value, top_idx [S, Nq, k] global
    block indices, top_scores); all but ``value`` are identical on every rank.
    value_layout "replicated": value [S, Nq, dv] on every rank; "stream_shard":
    value [hi - lo, Nq, dv] for this rank's streams [lo, hi) =
    stream_shard(S, rank, world).  ``timings`` (a dict, CUDA tensors only)
    accumulates milliseconds per phase: local_topk, gather_candidates, merge,
    readout, gather_winners, value_exchange."""
    if value_layout not in ("replicated", "stream_shard"):
        raise ValueError(f"value_layout must be 'replicated' or 'stream_shard', got {value_layout!r}")
    S, Nq = Q.shape[0], Q.shape[1]
    L = pool_K.shape[2]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    tm = _PhaseTimer(timings, timings is not None and Q.is_cuda)
    tm.mark("start")
    # 1. local candidates over the committed blocks of this shard
    nv = shard.size if n_valid is None else max(0, min(int(n_valid), shard.size))
    if nv > 0:
        ls, li = ops.block_topk(Q, summary, k, n_blocks=nv)
    else:
        ls = torch.full((S, Nq, k), float("-inf"), dtype=torch.float32, device=Q.device)
        li = torch.full((S, Nq, k), -1, dtype=torch.int32, device=Q.device)
    gi = torch.where(li >= 0, li + shard.lo, li)
    tm.mark("local_topk")
    # 2. gather and merge -> global top-k
    cs, ci = _gather_pairs(ls, gi, group)
    tm.mark("gather_candidates")
    top_s, top_i = ops.merge(cs, ci, k)
    tm.mark("merge")
    # 3. exact readout over the owned part of the global top-k
    own = (top_i >= shard.lo) & (top_i < shard.hi)
    local_sel = torch.where(own, top_i - shard.lo, torch.full_like(top_i, -1)).to(torch.int32)
    bt, bs, bv = ops.exact_readout(Q, pool_K, pool_V, local_sel)
    gt = torch.where(bt >= 0, bt + shard.lo * L, bt)
    tm.mark("readout")
    # 4. gather per-rank winners, merge -> global winner
    ws, wi = _gather_pairs(bs.unsqueeze(-1), gt.unsqueeze(-1), group)
    best_s, best_t = ops.merge(ws, wi, 1)
    best_s, best_t = best_s[..., 0], best_t[..., 0]
    tm.mark("gather_winners")
    value = None
    if pool_V is not None:
        owner = _owner_of(best_t, L, shard.n_blocks, world)
        mine = owner == rank  # the winner is this rank's own best for that query
        if value_layout == "replicated":
            value = _exchange_replicated(bv, owner, mine, world, group)
        elif S % world == 0 and dist.get_backend(group) == "nccl":
            value = _reduce_scatter_to_stream_shards(bv, best_t, mine, rank, world, group)
        else:
            value = _exchange_to_stream_shards(bv, owner, mine, rank, world, group)
    tm.mark("value_exchange")
    tm.finish()
    return best_t, best_s, value, top_i, top_s


def _exchange_replicated(bv: torch.Tensor, owner: torch.Tensor, mine: torch.Tensor, world: int, group):
    """Every rank ends with every winner's value row: each owner contributes its
    rows (query order) padded to the largest owner's count; one all-gather.
    The per-owner counts come to the host in one copy (the collective's size)."""
    S, Nq, dv = bv.shape
    own_flat = owner.reshape(-1)
    key = torch.where(own_flat >= 0, own_flat, torch.full_like(own_flat, world))
    counts = torch.bincount(key, minlength=world + 1)[:world].tolist()  # the one host sync
    width = max(max(counts), 1)
    mine_flat = mine.reshape(-1)
    n_mine = counts[dist.get_rank(group)]
    # this rank's rows in query order: a stable sort puts them first
    order = torch.argsort((~mine_flat).to(torch.int8), stable=True)[:n_mine]
    send = torch.zeros((width, dv), dtype=bv.dtype, device=bv.device)
    send[:n_mine] = bv.reshape(S * Nq, dv)[order]
    parts = torch.empty((world, width, dv), dtype=bv.dtype, device=bv.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(parts, send, group=group)
    else:  # gloo has no all_gather_into_tensor
        dist.all_gather(list(parts.unbind(0)), send, group=group)
    # row j of owner r's part is owner r's j-th winner in query order
    by_owner = torch.argsort(key, stable=True)
    starts = [0]
    for c in counts:
        starts.append(starts[-1] + c)
    value = torch.zeros((S * Nq, dv), dtype=bv.dtype, device=bv.device)
    for r in range(world):
        if counts[r]:
            value[by_owner[starts[r]:starts[r + 1]]] = parts[r, :counts[r]]
    return value.reshape(S, Nq, dv)


def _reduce_scatter_to_stream_shards(bv: torch.Tensor, best_t: torch.Tensor, mine: torch.Tensor, rank: int,
                                     world: int, group):
    """Equal stream shards: the rows this rank owns, -0.0 elsewhere, summed over
    the ranks by one reduce-scatter along the stream axis.  Exactly one rank
    owns each found winner and -0.0 is the identity of the addition, so every
    row arrives bit for bit; rows without a winner come out as +0.0, as the
    single-GPU readout writes them."""
    S, Nq, dv = bv.shape
    contrib = torch.where(mine[..., None], bv, torch.full((), -0.0, dtype=bv.dtype, device=bv.device))
    value = torch.empty((S // world, Nq, dv), dtype=bv.dtype, device=bv.device)
    dist.reduce_scatter_tensor(value, contrib.contiguous(), op=dist.ReduceOp.SUM, group=group)
    lo = rank * (S // world)
    found = best_t[lo:lo + S // world] >= 0
    return torch.where(found[..., None], value, torch.zeros((), dtype=bv.dtype, device=bv.device))


def _exchange_to_stream_shards(bv: torch.Tensor, owner: torch.Tensor, mine: torch.Tensor, rank: int, world: int,
                               group):
    """Each rank ends with the value rows of its stream shard: owners send each
    row to the rank of the query's stream with one all-to-all.  Split sizes are
    counted on the device and reach the host in one copy; rows are placed by
    index (stable sorts keep query order inside each source)."""
    S, Nq, dv = bv.shape
    dest = torch.empty((S,), dtype=torch.int64, device=bv.device)
    spans = [stream_shard(S, r, world) for r in range(world)]
    for r, (lo_r, hi_r) in enumerate(spans):
        dest[lo_r:hi_r] = r
    dest_q = dest[:, None].expand(S, Nq).reshape(-1)
    send_key = torch.where(mine.reshape(-1), dest_q, torch.full_like(dest_q, world))
    lo, hi = spans[rank]
    my_owner = owner[lo:hi].reshape(-1)
    recv_key = torch.where(my_owner >= 0, my_owner, torch.full_like(my_owner, world))
    counts = torch.cat((torch.bincount(send_key, minlength=world + 1)[:world],
                        torch.bincount(recv_key, minlength=world + 1)[:world])).tolist()  # the one host sync
    in_counts, out_counts = counts[:world], counts[world:]
    n_send, n_recv = sum(in_counts), sum(out_counts)
    order = torch.argsort(send_key, stable=True)[:n_send]
    send = bv.reshape(S * Nq, dv)[order].contiguous()
    recv = torch.empty((n_recv, dv), dtype=bv.dtype, device=bv.device)
    dist.all_to_all_single(recv, send, output_split_sizes=out_counts, input_split_sizes=in_counts, group=group)
    # recv holds source 0's rows, then source 1's, ..., each in query order
    place = torch.argsort(recv_key, stable=True)[:n_recv]
    value = torch.zeros(((hi - lo) * Nq, dv), dtype=bv.dtype, device=bv.device)
    value[place] = recv
    return value.reshape(hi - lo, Nq, dv)
