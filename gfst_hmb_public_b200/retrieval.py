"""Coarse block retrieval: query x block-summary scores and a deterministic
top-k, on the sm_100a kernels.

Drop-in for the reference's ``FaissGpuRetriever`` (pkhairkh/gfst-hmb-public,
src/gfst_hmb_mpuc/retrieval.py:29-172): same constructor shape, same keyword
``search`` signature, same error behaviour (RuntimeError for CPU tensors, a
missing CUDA device, or a device other than the pinned one; an empty bank
returns empty tensors), and a per-(state, layer, batch) record cache keyed on
``state.state_version``.  Search is exact (what FAISS approximates): every
summary is scored, and ties break toward the lower block index.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import _native as nat


def block_topk(Q: torch.Tensor, Ksum: torch.Tensor, k: int, n_blocks: int | None = None):
    """Top-k blocks per query.  Q [S, Nq, d]; Ksum [S, NB, d] (the first
    ``n_blocks`` rows are scored).  Returns (scores f32 [S,Nq,k], idx int32 [S,Nq,k])
    in the order (score desc, block asc); empty slots hold (-inf, -1).
    float32 inputs are scored with fp32 FMAs, bfloat16 inputs on the tensor cores."""
    nat.require_cuda(Q, Ksum, what="block_topk")
    if Q.ndim != 3 or Ksum.ndim != 3 or Q.shape[0] != Ksum.shape[0] or Q.shape[2] != Ksum.shape[2]:
        raise ValueError(f"block_topk expects Q [S,Nq,d], Ksum [S,NB,d]; got {tuple(Q.shape)}, {tuple(Ksum.shape)}")
    if Q.dtype != Ksum.dtype:
        raise RuntimeError(f"block_topk: dtype mismatch {Q.dtype} vs {Ksum.dtype}")
    S, Nq, d = Q.shape
    NBs = Ksum.shape[1]
    NB = NBs if n_blocks is None else int(n_blocks)
    Q = Q.contiguous()
    Ksum = Ksum.contiguous()
    scores = torch.empty((S, Nq, k), dtype=torch.float32, device=Q.device)
    idx = torch.empty((S, Nq, k), dtype=torch.int32, device=Q.device)
    with torch.cuda.device(Q.device):
        nat.call("gfst_block_topk", nat.ptr(Q), nat.ptr(Ksum), S, Nq, NB, NBs, d, int(k),
                 nat.dtype_code(Q.dtype, "block_topk"), nat.ptr(scores), nat.ptr(idx), nat.stream_of(Q))
    return scores, idx


@dataclass
class RetrievalConfig:
    """Mirror of the fields of the reference's FaissGpuRetrievalConfig
    (src/gfst_hmb_mpuc/config.py:211-245) that affect the exact search."""
    gpu_device: int = 0
    index_type: str = "exact"
    nlist: int = 0
    nprobe: int = 0
    flat_fallback_threshold: int = 0
    use_float16: bool = False
    temp_memory_bytes: int = 0


@dataclass
class _IndexRecord:
    state_version: int
    summary_count: int
    device_index: int
    index_type: str


class BlockRetriever:
    """Exact replacement of FaissGpuRetriever (retrieval.py:29-163)."""

    def __init__(self, config: Any | None = None) -> None:
        self.config = config if config is not None else RetrievalConfig()
        self._index_cache: dict[tuple[int, int, int], _IndexRecord] = {}

    def _ensure_runtime_device(self, tensor: torch.Tensor) -> int:
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is required for block retrieval")
        if tensor.device.type != "cuda":
            raise RuntimeError("block retrieval requires CUDA tensors")
        if tensor.device.index != int(self.config.gpu_device):
            raise RuntimeError(f"block retrieval is pinned to cuda:{self.config.gpu_device}, got {tensor.device}")
        return int(tensor.device.index)

    def _get_record(self, *, state: Any, layer_idx: int, batch_idx: int, keys_tensor: torch.Tensor) -> _IndexRecord:
        key = (id(state), int(layer_idx), int(batch_idx))
        record = self._index_cache.get(key)
        count = int(keys_tensor.shape[0])
        version = int(getattr(state, "state_version", 0))
        if (record is None or record.state_version != version or record.summary_count != count
                or record.device_index != int(self.config.gpu_device)):
            record = _IndexRecord(version, count, self._ensure_runtime_device(keys_tensor), "exact")
            self._index_cache[key] = record
        return record

    def search(self, *, state: Any, layer_idx: int, batch_idx: int, keys_tensor: torch.Tensor,
               query_tensor: torch.Tensor, top_k: int):
        """Best ``min(top_k, count)`` summaries for query row 0: (indices int64, scores f32)."""
        if int(keys_tensor.shape[0]) == 0:
            return (torch.empty(0, device=query_tensor.device, dtype=torch.long),
                    torch.empty(0, device=query_tensor.device, dtype=torch.float32))
        self._ensure_runtime_device(query_tensor)
        self._ensure_runtime_device(keys_tensor)
        self._get_record(state=state, layer_idx=layer_idx, batch_idx=batch_idx, keys_tensor=keys_tensor)
        return self.exact_topk(keys_tensor, query_tensor, top_k)

    @staticmethod
    def exact_topk(keys_tensor: torch.Tensor, query_tensor: torch.Tensor, top_k: int):
        """retrieval.py:165-172: scores = keys @ q (row 0 of a 2-D query), the
        best min(top_k, count) of them, as (indices int64, scores float32).
        bfloat16 keys score as the reference's bf16 matmul returns them (the
        fp32 sum rounded to bf16); equal scores rank the lower index first.
        Keys of other dtypes are scored in float32."""
        return exact_topk(keys_tensor, query_tensor, top_k)


def exact_topk(keys_tensor: torch.Tensor, query_tensor: torch.Tensor, top_k: int):
    """One query against a bank of keys, any top_k (gfst_exact_topk); see
    BlockRetriever.exact_topk."""
    nat.require_cuda(keys_tensor, query_tensor, what="exact_topk")
    if keys_tensor.ndim != 2:
        raise ValueError(f"exact_topk expects keys [count, d], got {tuple(keys_tensor.shape)}")
    q = query_tensor if query_tensor.ndim == 1 else query_tensor[0]
    if q.numel() != keys_tensor.shape[1]:
        raise ValueError(f"exact_topk: query of {q.numel()} values for keys of width {keys_tensor.shape[1]}")
    count = int(keys_tensor.shape[0])
    k = min(int(top_k), count)
    if k <= 0:
        return (torch.empty(0, device=q.device, dtype=torch.long),
                torch.empty(0, device=q.device, dtype=torch.float32))
    dtype = keys_tensor.dtype if keys_tensor.dtype in (torch.float32, torch.bfloat16) else torch.float32
    keys = keys_tensor.to(dtype).contiguous()
    q = q.to(dtype).contiguous()
    lib = nat.load()
    ws_bytes = int(lib.gfst_exact_topk_workspace_bytes(count, k))
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=q.device) if ws_bytes else None
    scores = torch.empty((k,), dtype=torch.float32, device=q.device)
    idx = torch.empty((k,), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        nat.call("gfst_exact_topk", nat.ptr(keys), nat.ptr(q), count, int(keys.shape[1]), k,
                 nat.dtype_code(dtype, "exact_topk"), 1, nat.ptr(scores), nat.ptr(idx), nat.ptr(ws), ws_bytes,
                 nat.stream_of(q))
    return idx, scores


# the reference's class name, for drop-in imports
FaissGpuRetriever = BlockRetriever


def topk_merge(scores: torch.Tensor, idx: torch.Tensor, k: int):
    """Top-k of candidate lists (score desc, index asc): scores/idx [..., n_cand]
    -> ([..., k] f32, [..., k] int32).  Negative indices, NaN and -inf skipped."""
    nat.require_cuda(scores, idx, what="topk_merge")
    if scores.shape != idx.shape:
        raise ValueError("topk_merge: scores and idx shapes differ")
    lead = tuple(scores.shape[:-1])
    n_cand = int(scores.shape[-1])
    s2 = scores.to(torch.float32).contiguous().reshape(-1, n_cand)
    i2 = idx.to(torch.int32).contiguous().reshape(-1, n_cand)
    rows = s2.shape[0]
    out_s = torch.empty((rows, k), dtype=torch.float32, device=scores.device)
    out_i = torch.empty((rows, k), dtype=torch.int32, device=scores.device)
    with torch.cuda.device(scores.device):
        nat.call("gfst_topk_merge", nat.ptr(s2), nat.ptr(i2), rows, n_cand, int(k), nat.ptr(out_s), nat.ptr(out_i),
                 nat.stream_of(s2))
    return out_s.reshape(*lead, k), out_i.reshape(*lead, k)
