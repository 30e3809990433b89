"""The MPUC recurrent scan on B200 (gfst_mpuc_recurrent_scan).

Replaces the token loop of MpucGfstHmbBlock._forward_sequence_tensors
(src/gfst_hmb_mpuc/modeling.py:4449-4476 of pkhairkh/gfst-hmb-public): the
three-band recurrent cell (_token_step, 4363-4411) runs in one cooperative
kernel per 8 sequences, and the non-recurrent output projection
(fusion_proj + _semantic_residual, 4358-4361 and 4406-4410) runs afterwards
as batched products over all tokens.  The reference's native
``mpuc_recurrent_scan_forward`` (csrc/sm120_stub.cu:210-224) takes no weights
and returns zeros; here the weights come from the reference's module (or a
dict with the same parameter names).
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

# gfst_mpuc_weights field -> the reference module's parameter
WEIGHT_FIELDS = (
    ("fast_gate_w", "fast_gate_proj.weight"), ("fast_gate_b", "fast_gate_proj.bias"),
    ("fast_cand_w", "fast_cand_proj.weight"), ("fast_cand_b", "fast_cand_proj.bias"),
    ("mid_gate_w", "mid_gate_proj.weight"), ("mid_gate_b", "mid_gate_proj.bias"),
    ("mid_cand_w", "mid_cand_proj.weight"), ("mid_cand_b", "mid_cand_proj.bias"),
    ("slow_gate_w", "slow_gate_proj.weight"), ("slow_gate_b", "slow_gate_proj.bias"),
    ("slow_cand_w", "slow_cand_proj.weight"), ("slow_cand_b", "slow_cand_proj.bias"),
    ("fm_down", "fast_from_mid.down.weight"), ("fm_up", "fast_from_mid.up.weight"),
    ("fs_down", "fast_from_slow.down.weight"), ("fs_up", "fast_from_slow.up.weight"),
    ("mf_down", "mid_from_fast.down.weight"), ("mf_up", "mid_from_fast.up.weight"),
    ("ms_down", "mid_from_slow.down.weight"), ("ms_up", "mid_from_slow.up.weight"),
    ("sf_down", "slow_from_fast.down.weight"), ("sf_up", "slow_from_fast.up.weight"),
    ("sm_down", "slow_from_mid.down.weight"), ("sm_up", "slow_from_mid.up.weight"),
    ("bnd_w1", "boundary_mlp.0.weight"), ("bnd_b1", "boundary_mlp.0.bias"),
    ("bnd_w2", "boundary_mlp.2.weight"), ("bnd_b2", "boundary_mlp.2.bias"),
)
# the output projection (applied outside the scan)
OUTPUT_FIELDS = (("sem_in", "semantic_in.weight"), ("sem_cond", "semantic_cond.weight"),
                 ("sem_out", "semantic_out.weight"), ("fusion", "fusion_proj.weight"))


class _WeightsC(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name, _ in WEIGHT_FIELDS]


class MpucCellWeights:
    """fp32, contiguous, device-resident weights of one MPUC cell.

    ``tensors`` maps the short names of WEIGHT_FIELDS / OUTPUT_FIELDS (or the
    reference module's parameter names) to tensors; the output projection is
    optional (the scan alone does not need it)."""

    def __init__(self, tensors: dict, device) -> None:
        self.device = torch.device(device)
        alias = {full: short for short, full in WEIGHT_FIELDS + OUTPUT_FIELDS}
        self.t: dict[str, torch.Tensor] = {}
        for name, v in tensors.items():
            key = alias.get(name, name)
            self.t[key] = torch.as_tensor(v).detach().to(self.device, torch.float32).contiguous()
        missing = [n for n, _ in WEIGHT_FIELDS if n not in self.t]
        if missing:
            raise ValueError(f"MPUC cell weights missing: {missing}")
        self.F = int(self.t["fast_gate_w"].shape[0])
        self.M = int(self.t["mid_gate_w"].shape[0])
        self.S = int(self.t["slow_gate_w"].shape[0])
        self.C = int(self.t["fm_down"].shape[0])
        self.BH = int(self.t["bnd_w1"].shape[0])
        expect = {
            "fast_gate_w": (self.F, self.F), "fast_cand_w": (self.F, self.F), "mid_gate_w": (self.M, self.M),
            "mid_cand_w": (self.M, self.M), "slow_gate_w": (self.S, self.S), "slow_cand_w": (self.S, self.S),
            "fm_down": (self.C, self.M), "fm_up": (self.F, self.C), "fs_down": (self.C, self.S),
            "fs_up": (self.F, self.C), "mf_down": (self.C, self.F), "mf_up": (self.M, self.C),
            "ms_down": (self.C, self.S), "ms_up": (self.M, self.C), "sf_down": (self.C, self.F),
            "sf_up": (self.S, self.C), "sm_down": (self.C, self.M), "sm_up": (self.S, self.C),
            "bnd_w1": (self.BH, 4), "bnd_w2": (1, self.BH),
        }
        for n, shp in expect.items():
            if tuple(self.t[n].shape) != shp:
                raise ValueError(f"MPUC weight {n}: shape {tuple(self.t[n].shape)}, expected {shp}")
        self._c = _WeightsC(**{n: int(self.t[n].data_ptr()) for n, _ in WEIGHT_FIELDS})

    @classmethod
    def from_module(cls, block, device=None) -> "MpucCellWeights":
        """From the reference's MpucGfstHmbBlock (or any module with the same
        submodule names)."""
        params = dict(block.named_parameters())
        names = [full for _, full in WEIGHT_FIELDS + OUTPUT_FIELDS if full in params]
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        return cls({n: params[n] for n in names}, dev)

    @property
    def hidden(self) -> int:
        return self.F + self.M + self.S


def recurrent_scan(weights: MpucCellWeights, fast_in: torch.Tensor, mid_in: torch.Tensor, slow_in: torch.Tensor,
                   state: tuple | None = None):
    """The recurrence over T tokens of B sequences.

    fast_in [B, T, F], mid_in [B, T, M], slow_in [B, T, S] (fp32 CUDA: the
    three branch outputs); ``state`` = (fast [B, F], mid [B, M], slow [B, S])
    before the first token, zeros when None.  Returns (states [B, T, F+M+S],
    boundary_logits [B, T], fast, mid, slow)."""
    dev = nat.require_cuda(fast_in, mid_in, slow_in, what="mpuc recurrent_scan")
    if dev != weights.device:
        raise RuntimeError("mpuc recurrent_scan: inputs and weights on different devices")
    if fast_in.ndim != 3 or mid_in.ndim != 3 or slow_in.ndim != 3:
        raise ValueError("recurrent_scan expects [B, T, width] inputs")
    B, T = int(fast_in.shape[0]), int(fast_in.shape[1])
    W = weights
    for name, x, width in (("fast_in", fast_in, W.F), ("mid_in", mid_in, W.M), ("slow_in", slow_in, W.S)):
        if tuple(x.shape) != (B, T, width):
            raise ValueError(f"recurrent_scan: {name} has shape {tuple(x.shape)}, expected {(B, T, width)}")
    fast_in, mid_in, slow_in = (x.to(torch.float32).contiguous() for x in (fast_in, mid_in, slow_in))
    if state is None:
        st = [torch.zeros((B, n), device=dev, dtype=torch.float32) for n in (W.F, W.M, W.S)]
    else:
        st = [s.to(dev, torch.float32).contiguous().clone() for s in state]
    states = torch.empty((B, T, W.hidden), device=dev, dtype=torch.float32)
    logits = torch.empty((B, T), device=dev, dtype=torch.float32)
    lib = nat.load()
    nbytes = ctypes.c_size_t(0)
    with torch.cuda.device(dev):
        nat.check(lib.gfst_mpuc_scan_workspace_bytes(B, W.F, W.M, W.S, W.C, ctypes.byref(nbytes)),
                  "gfst_mpuc_scan_workspace_bytes")
        ws = torch.empty((max(16, int(nbytes.value)),), device=dev, dtype=torch.uint8)
        nat.call("gfst_mpuc_recurrent_scan", ctypes.addressof(W._c), W.F, W.M, W.S, W.C, W.BH,
                 nat.ptr(fast_in), nat.ptr(mid_in), nat.ptr(slow_in), B, T, nat.ptr(states), nat.ptr(logits),
                 nat.ptr(st[0]), nat.ptr(st[1]), nat.ptr(st[2]), nat.ptr(ws), int(ws.numel()),
                 nat.stream_of(fast_in))
    return states, logits, st[0], st[1], st[2]


def output_projection(weights: MpucCellWeights, normalised: torch.Tensor, states: torch.Tensor) -> torch.Tensor:
    """fusion_proj(cat(fast, mid, slow)) + semantic_out(semantic_in(x) *
    sigmoid(semantic_cond(cat(mid, slow)))) for every token (modeling.py:4358-4361,
    4406-4410): batched products over [B*T] rows."""
    t = weights.t
    for n in ("sem_in", "sem_cond", "sem_out", "fusion"):
        if n not in t:
            raise ValueError(f"output_projection needs weight {n}")
    x = normalised.to(torch.float32)
    base = x @ t["sem_in"].T
    cond = torch.sigmoid(states[..., weights.F:] @ t["sem_cond"].T)
    return states @ t["fusion"].T + (base * cond) @ t["sem_out"].T


def forward_sequence_tensors(block, normalised: torch.Tensor, weights: MpucCellWeights | None = None):
    """MpucGfstHmbBlock._forward_sequence_tensors(normalised) with the token loop
    on B200: the block's own branch modules produce the scan inputs, the
    kernel runs the recurrence, the output projection runs batched.  Returns
    (outputs [B, T, H], boundary_logits [B, T], fast, mid, slow) in the
    block's dtype."""
    if weights is None:
        weights = MpucCellWeights.from_module(block, device=normalised.device)
    with torch.no_grad():
        fast_in = block.fast_branch.forward_sequence(normalised)
        mid_in = block.mid_branch.forward_sequence(normalised)
        slow_in = block.slow_branch.forward_sequence(normalised)
    states, logits, fast, mid, slow = recurrent_scan(weights, fast_in, mid_in, slow_in)
    out = output_projection(weights, normalised, states)
    dt = normalised.dtype
    return out.to(dt), logits.to(dt), fast.to(dt), mid.to(dt), slow.to(dt)
