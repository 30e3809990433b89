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


def block_commit_i8(K: torch.Tensor, pool_K8: torch.Tensor, k8_scale: torch.Tensor, slot: int) -> None:
    """Write the int8 copy of block K [S, L, d] (bf16, d = 128 or 256) into
    ``slot`` of pool_K8 [S, n_slots, L, d] int8, with the per-token scales and
    the block's error / key norm bounds in k8_scale [S, n_slots, L + 4]
    float32 (gfst_block_commit_i8): the side data that lets exact_readout bound
    exact scores from the int8 copies."""
    nat.require_cuda(K, pool_K8, k8_scale, what="block_commit_i8")
    S, L, d = K.shape
    n_slots = pool_K8.shape[1]
    if K.dtype != torch.bfloat16 or pool_K8.dtype != torch.int8 or k8_scale.dtype != torch.float32:
        raise RuntimeError("block_commit_i8: bf16 keys, int8 copies, float32 side data")
    if tuple(pool_K8.shape) != (S, n_slots, L, d) or tuple(k8_scale.shape) != (S, n_slots, L + 4):
        raise ValueError("block_commit_i8: shape mismatch")
    if not (pool_K8.is_contiguous() and k8_scale.is_contiguous()):
        raise ValueError("block_commit_i8: int8 copies and side data must be contiguous")
    K = K.contiguous()
    with torch.cuda.device(K.device):
        nat.call("gfst_block_commit_i8", nat.ptr(K), nat.ptr(pool_K8), nat.ptr(k8_scale), S, n_slots, int(slot), L, d,
                 nat.stream_of(K))


class BlockMemory:
    """Ring of ``n_slots`` committed blocks per stream (keys, values, summaries).

    ``int8_keys``: also keep an int8 copy of every key with its side data
    (``pool_K8``, ``k8_scale``; block_commit_i8), which exact_readout streams in
    place of the bf16 keys (bf16 memories, d = 128 or 256)."""

    def __init__(self, n_streams: int, n_slots: int, block_len: int, d: int, dv: int | None = None, *,
                 dtype: torch.dtype = torch.bfloat16, device="cuda", int8_keys: bool = False):
        dv = d if dv is None else dv
        self.n_streams, self.n_slots, self.block_len, self.d, self.dv = n_streams, n_slots, block_len, d, dv
        self.dtype = dtype
        self.pool_K = torch.zeros((n_streams, n_slots, block_len, d), dtype=dtype, device=device)
        self.pool_V = torch.zeros((n_streams, n_slots, block_len, dv), dtype=dtype, device=device)
        self.summary = torch.zeros((n_streams, n_slots, d), dtype=dtype, device=device)
        self.pool_K8 = self.k8_scale = None
        if int8_keys:
            if dtype != torch.bfloat16 or d not in (128, 256):
                raise ValueError("BlockMemory: int8 key copies need bf16 keys with d = 128 or 256")
            self.pool_K8 = torch.zeros((n_streams, n_slots, block_len, d), dtype=torch.int8, device=device)
            self.k8_scale = torch.zeros((n_streams, n_slots, block_len + 4), dtype=torch.float32, device=device)
        self.blocks_committed = 0      # total blocks ever committed
        self.state_version = 0         # bumped on every mutation (retrieval caches key on it)

    @property
    def device(self) -> torch.device:
        return self.pool_K.device

    @property
    def k8(self) -> tuple | None:
        """(pool_K8, k8_scale) for exact_readout, or None without int8 copies."""
        return None if self.pool_K8 is None else (self.pool_K8, self.k8_scale)

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
        if self.pool_K8 is not None:
            block_commit_i8(K, self.pool_K8, self.k8_scale, slot)
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
