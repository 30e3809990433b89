"""Block memory: the per-stream pool of committed L-token blocks and their
summary keys, committed with the sm_100a commit kernel.

Reference (pkhairkh/gfst-hmb-public): GfstDecodeState's exact-token store
commits one packed block every block_len tokens (src/gfst_hmb_mpuc/state.py:651-815,
records at state.py:34-77) and the sublayer appends a block summary at the same
boundary (src/gfst_hmb_mpuc/modeling.py:3482-3550, which also invalidates the
summary cache; here ``state_version`` is bumped instead, like
``GfstDecodeState.mark_mutated``).  The summary key is the mean of the block's
token keys.

Layout in HBM (row-major): pool_K [S, n_slots, L, d], pool_V [S, n_slots, L, dv],
summary [S, n_slots, d].  A block is one contiguous L x d slab, so a commit is
a 16-byte-vector copy and a gather of a selected block is a contiguous read.
Slots form a ring: once all n_slots are full the oldest block is overwritten.
"""
from __future__ import annotations

import torch

from . import _native as nat


def block_commit_mean(K: torch.Tensor, V: torch.Tensor | None, pool_K: torch.Tensor, pool_V: torch.Tensor | None,
                      summary: torch.Tensor, slot: int) -> None:
    """Write block K [S, L, d] (and V [S, L, dv]) into ``slot`` of the pools and
    store summary[:, slot] = mean of K over L (fp32 sum in token order, one rounding)."""
    nat.require_cuda(K, V, pool_K, pool_V, summary, what="block_commit_mean")
    if K.ndim != 3 or pool_K.ndim != 4 or summary.ndim != 3:
        raise ValueError("block_commit_mean expects K [S,L,d], pool_K [S,slots,L,d], summary [S,slots,d]")
    S, L, d = K.shape
    n_slots = pool_K.shape[1]
    if tuple(pool_K.shape) != (S, n_slots, L, d) or tuple(summary.shape) != (S, n_slots, d):
        raise ValueError(f"shape mismatch K{tuple(K.shape)} pool_K{tuple(pool_K.shape)} summary{tuple(summary.shape)}")
    dv = 0
    if V is not None:
        dv = V.shape[-1]
        if pool_V is None or tuple(V.shape) != (S, L, dv) or tuple(pool_V.shape) != (S, n_slots, L, dv):
            raise ValueError("block_commit_mean: V / pool_V shapes do not match")
    dtypes = {t.dtype for t in (K, V, pool_K, pool_V, summary) if t is not None}
    if len(dtypes) != 1:
        raise RuntimeError(f"block_commit_mean: mixed dtypes {dtypes}")
    for t in (pool_K, pool_V, summary):
        if t is not None and not t.is_contiguous():
            raise ValueError("block_commit_mean: pools and summary must be contiguous")
    K = K.contiguous()
    V = V.contiguous() if V is not None else None
    with torch.cuda.device(K.device):
        nat.call("gfst_block_commit_mean", nat.ptr(K), nat.ptr(V), nat.ptr(pool_K), nat.ptr(pool_V),
                 nat.ptr(summary), S, n_slots, int(slot), L, d, dv, nat.dtype_code(K.dtype, "block_commit_mean"),
                 nat.stream_of(K))


class BlockMemory:
    """Ring of ``n_slots`` committed blocks per stream (keys, values, summaries)."""

    def __init__(self, n_streams: int, n_slots: int, block_len: int, d: int, dv: int | None = None, *,
                 dtype: torch.dtype = torch.bfloat16, device="cuda"):
        dv = d if dv is None else dv
        self.n_streams, self.n_slots, self.block_len, self.d, self.dv = n_streams, n_slots, block_len, d, dv
        self.dtype = dtype
        self.pool_K = torch.zeros((n_streams, n_slots, block_len, d), dtype=dtype, device=device)
        self.pool_V = torch.zeros((n_streams, n_slots, block_len, dv), dtype=dtype, device=device)
        self.summary = torch.zeros((n_streams, n_slots, d), dtype=dtype, device=device)
        self.blocks_committed = 0      # total blocks ever committed
        self.state_version = 0         # bumped on every mutation (retrieval caches key on it)

    @property
    def device(self) -> torch.device:
        return self.pool_K.device

    @property
    def n_valid(self) -> int:
        """Slots holding a committed block."""
        return min(self.blocks_committed, self.n_slots)

    def slot_of(self, block_index: int) -> int:
        return block_index % self.n_slots

    def next_slot(self) -> int:
        return self.blocks_committed % self.n_slots

    def commit(self, K: torch.Tensor, V: torch.Tensor | None = None) -> int:
        """Commit one block per stream; returns the slot written."""
        slot = self.next_slot()
        block_commit_mean(K, V, self.pool_K, self.pool_V if V is not None else None, self.summary, slot)
        self.blocks_committed += 1
        self.mark_mutated()
        return slot

    def mark_mutated(self) -> None:
        self.state_version += 1

    def reset(self) -> None:
        """Forget every committed block (the pools keep their bytes; nothing
        reads a slot before a commit writes it again)."""
        self.blocks_committed = 0
        self.mark_mutated()

    def slot_block_index(self) -> torch.Tensor:
        """Block index (position in the stream / L) held by each slot, -1 for empty."""
        idx = torch.full((self.n_slots,), -1, dtype=torch.int64)
        for b in range(max(0, self.blocks_committed - self.n_slots), self.blocks_committed):
            idx[b % self.n_slots] = b
        return idx


def exact_block_materialize(packed: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """runtime_backends.exact_block_materialize (native
    exact_block_materialize_forward, src/gfst_hmb_mpuc/csrc/sm120_stub.cu:225-245;
    called at state.py:568): a new tensor holding packed[start:end] of a 1-D
    contiguous CUDA tensor, copied by the sm_100a copy kernel.  Raises
    RuntimeError for a range outside the tensor, as the reference's checks do."""
    nat.require_cuda(packed, what="exact_block_materialize")
    if packed.ndim != 1:
        raise RuntimeError("exact_block_materialize: packed must be rank 1")
    if not packed.is_contiguous():
        raise RuntimeError("exact_block_materialize: packed must be contiguous")
    start, end = int(start), int(end)
    out = torch.empty((max(end - start, 0),), dtype=packed.dtype, device=packed.device)
    with torch.cuda.device(packed.device):
        nat.call("gfst_exact_block_materialize", nat.ptr(packed), int(packed.numel()), int(packed.element_size()),
                 start, end, nat.ptr(out), nat.stream_of(packed))
    return out
