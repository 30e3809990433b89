"""Seeded synthetic workloads of the GFST-HMB hot path.

There is no public dataset for this path; every input is drawn from a seeded
``torch.Generator`` with the shapes and distributions below.  The same call
with ``device="cpu"`` produces the small inputs the CPU oracle checks.

Workloads (units: B = batch, H = heads, T = tokens, d x r frames, rank-m
updates, L-token blocks, NB blocks, k blocks selected per query):

* ``stream_small``  B=2,  H=4,  T=256,    d=64,  r=8,  m=1, L=16,  NB=16,   k=2,  fp32 memory
* ``batched_qr``    65,536 independent 64 x 8 frames (column j scaled by 10^(-j/2),
                    1% with two columns at cosine 0.9999)
* ``stream_mid``    B=16, H=16, T=4096,   d=128, r=16, m=2, L=64,  NB=64,   k=4,  bf16 memory
* ``long_memory``   B=8,  H=32, 1,048,576-token memory, d=128, L=128, NB=8192, k=8,
                    1024 needle queries per (b, h), bf16 memory
* ``stream_full``   B=64, H=32, T=32768,  d=128, r=32, m=4, L=64,  NB=512,  k=16, bf16 memory
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

SEED_BASE = 20261201


@dataclass(frozen=True)
class StreamSpec:
    name: str
    batch: int
    heads: int
    tokens: int
    d: int
    r: int
    m: int
    block_len: int
    n_blocks: int
    k: int
    memory_dtype: torch.dtype
    seed: int

    @property
    def streams(self) -> int:
        return self.batch * self.heads


STREAM_SMALL = StreamSpec("stream_small", 2, 4, 256, 64, 8, 1, 16, 16, 2, torch.float32, SEED_BASE + 0)
STREAM_MID = StreamSpec("stream_mid", 16, 16, 4096, 128, 16, 2, 64, 64, 4, torch.bfloat16, SEED_BASE + 2)
STREAM_FULL = StreamSpec("stream_full", 64, 32, 32768, 128, 32, 4, 64, 512, 16, torch.bfloat16, SEED_BASE + 4)


@dataclass(frozen=True)
class LongMemorySpec:
    name: str
    batch: int
    heads: int
    memory_tokens: int
    d: int
    block_len: int
    n_queries: int
    k: int
    needle_noise: float
    seed: int

    @property
    def streams(self) -> int:
        return self.batch * self.heads

    @property
    def n_blocks(self) -> int:
        return self.memory_tokens // self.block_len


LONG_MEMORY = LongMemorySpec("long_memory", 8, 32, 1 << 20, 128, 128, 1024, 8, 0.1, SEED_BASE + 3)

BATCHED_QR = dict(name="batched_qr", n=65536, d=64, r=8, collinear_frac=0.01, cosine=0.9999, seed=SEED_BASE + 1)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(int(seed))
    return g


# ---------------------------------------------------------------------------
# frames
# ---------------------------------------------------------------------------
def batched_qr_inputs(n: int, d: int, r: int, *, seed: int, device="cpu", collinear_frac: float = 0.01,
                      cosine: float = 0.9999) -> torch.Tensor:
    """[n, d, r] float32: N(0,1) entries, column j scaled by 10^(-j/2); in
    round(collinear_frac*n) frames (chosen by a seeded permutation) a random
    column j+1 is replaced by cos*c_j_hat + sin*p_hat (p orthogonal to c_j), scaled
    to its original norm, giving two columns at the given cosine."""
    g = _gen(device, seed)
    x = torch.randn((n, d, r), generator=g, device=device, dtype=torch.float32)
    scale = torch.pow(10.0, -torch.arange(r, device=device, dtype=torch.float32) / 2.0)
    x = x * scale
    n_col = int(round(n * collinear_frac))
    if n_col > 0 and r >= 2:
        idx = torch.randperm(n, generator=g, device=device)[:n_col]
        j = torch.randint(0, r - 1, (n_col,), generator=g, device=device)
        rows = torch.arange(n_col, device=device)
        sub = x[idx]                                   # [n_col, d, r]
        cj = sub[rows, :, j]                           # [n_col, d]
        cn = sub[rows, :, j + 1]
        cj_hat = cj / cj.norm(dim=-1, keepdim=True)
        p = torch.randn((n_col, d), generator=g, device=device, dtype=torch.float32)
        p = p - (p * cj_hat).sum(-1, keepdim=True) * cj_hat
        p_hat = p / p.norm(dim=-1, keepdim=True)
        sin = math.sqrt(1.0 - cosine * cosine)
        new = (cosine * cj_hat + sin * p_hat) * cn.norm(dim=-1, keepdim=True)
        sub[rows, :, j + 1] = new
        x[idx] = sub
    return x.contiguous()


def random_orthonormal_frames(n: int, d: int, r: int, *, seed: int, device="cpu") -> torch.Tensor:
    """N(0,1) [n, d, r] frames orthonormalised by QR with positive R diagonal,
    computed with torch.linalg.qr on the CPU (set-up only)."""
    g = _gen("cpu", seed)
    x = torch.randn((n, d, r), generator=g, dtype=torch.float64)
    q, rr = torch.linalg.qr(x, mode="reduced")
    q = q * torch.where(torch.diagonal(rr, dim1=-2, dim2=-1) < 0, -1.0, 1.0).unsqueeze(-2)
    return q.to(torch.float32).to(device).contiguous()


def stream_update_factors(n: int, T: int, d: int, r: int, m: int, *, seed: int, device="cpu"):
    """Rank-m per-token factors A [n, T, d, m], B [n, T, r, m] with entries
    N(0, 1/d): the update U + sum_i u_i v_i^T with u, v ~ N(0, 1/d)."""
    g = _gen(device, seed)
    std = 1.0 / math.sqrt(d)
    A = torch.randn((n, T, d, m), generator=g, device=device, dtype=torch.float32) * std
    B = torch.randn((n, T, r, m), generator=g, device=device, dtype=torch.float32) * std
    return A, B


def token_tensors(n: int, T: int, d: int, *, seed: int, device="cpu", dtype=torch.float32, count: int = 3):
    """``count`` N(0,1) tensors [n, T, d] (keys, values, queries) in ``dtype``."""
    g = _gen(device, seed)
    return [torch.randn((n, T, d), generator=g, device=device, dtype=torch.float32).to(dtype).contiguous()
            for _ in range(count)]


def mpuc_cell_weights(hidden: int, *, seed: int, device="cpu"):
    """Weights of an MPUC cell of width ``hidden`` with the reference's sizes
    (MpucGfstHmbBlock.__init__, modeling.py:4259-4315 of
    pkhairkh/gfst-hmb-public: fast H/2, mid H/4, slow the rest, bridge and
    semantic rank max(64, H/16), boundary hidden max(8, H/16)) and nn.Linear's
    default scale (uniform in +-1/sqrt(fan_in)), as an mpuc.MpucCellWeights."""
    from .mpuc import MpucCellWeights

    g = _gen("cpu", seed)
    H = int(hidden)
    F, M = H // 2, H // 4
    S = H - F - M
    C = SR = max(64, H // 16)
    BH = max(8, H // 16)

    def lin(o, i):
        return (torch.rand((o, i), generator=g) * 2 - 1) / math.sqrt(i)

    def bias(o, i):
        return (torch.rand((o,), generator=g) * 2 - 1) / math.sqrt(i)

    w = {"fast_gate_w": lin(F, F), "fast_gate_b": bias(F, F), "fast_cand_w": lin(F, F), "fast_cand_b": bias(F, F),
         "mid_gate_w": lin(M, M), "mid_gate_b": bias(M, M), "mid_cand_w": lin(M, M), "mid_cand_b": bias(M, M),
         "slow_gate_w": lin(S, S), "slow_gate_b": bias(S, S), "slow_cand_w": lin(S, S), "slow_cand_b": bias(S, S),
         "fm_down": lin(C, M), "fm_up": lin(F, C), "fs_down": lin(C, S), "fs_up": lin(F, C),
         "mf_down": lin(C, F), "mf_up": lin(M, C), "ms_down": lin(C, S), "ms_up": lin(M, C),
         "sf_down": lin(C, F), "sf_up": lin(S, C), "sm_down": lin(C, M), "sm_up": lin(S, C),
         "bnd_w1": lin(BH, 4), "bnd_b1": bias(BH, 4), "bnd_w2": lin(1, BH), "bnd_b2": bias(1, BH),
         "sem_in": lin(SR, H), "sem_cond": lin(SR, M + S), "sem_out": lin(H, SR), "fusion": lin(H, H)}
    return MpucCellWeights(w, device)
