"""CPU restatement of the reference's MPUC recurrent cell -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/ and bench.py's CPU baseline, never by the product
package.  Restates MpucGfstHmbBlock._forward_sequence_tensors and the cell it
steps (src/gfst_hmb_mpuc/modeling.py of pkhairkh/gfst-hmb-public):

* _forward_sequence_tensors  modeling.py:4449-4476 -- zero states, then one
  _token_step per token with fast_drive = fast_inputs[t] + fast_from_mid(mid)
  + fast_from_slow(slow);
* _token_step                modeling.py:4363-4411;
* _update_band               modeling.py:4343-4356 -- gate = sigmoid(W_g x + b_g)
  (times gate_scale for the slow band), cand = tanh(W_c x + b_c),
  state = (1 - gate) * prev + gate * cand;
* _semantic_residual         modeling.py:4358-4361;
* _LowRankBridge.forward     modeling.py:4182-4183 -- up(silu(down(x))).

Weights are a dict of float32 numpy arrays with nn.Linear's layout
([out, in] weights, [out] biases), named as in ``WEIGHT_NAMES``.
"""
from __future__ import annotations

import numpy as np

# name -> the reference submodule parameter it holds
WEIGHT_NAMES = {
    "fast_gate_w": "fast_gate_proj.weight", "fast_gate_b": "fast_gate_proj.bias",
    "fast_cand_w": "fast_cand_proj.weight", "fast_cand_b": "fast_cand_proj.bias",
    "mid_gate_w": "mid_gate_proj.weight", "mid_gate_b": "mid_gate_proj.bias",
    "mid_cand_w": "mid_cand_proj.weight", "mid_cand_b": "mid_cand_proj.bias",
    "slow_gate_w": "slow_gate_proj.weight", "slow_gate_b": "slow_gate_proj.bias",
    "slow_cand_w": "slow_cand_proj.weight", "slow_cand_b": "slow_cand_proj.bias",
    "fm_down": "fast_from_mid.down.weight", "fm_up": "fast_from_mid.up.weight",
    "fs_down": "fast_from_slow.down.weight", "fs_up": "fast_from_slow.up.weight",
    "mf_down": "mid_from_fast.down.weight", "mf_up": "mid_from_fast.up.weight",
    "ms_down": "mid_from_slow.down.weight", "ms_up": "mid_from_slow.up.weight",
    "sf_down": "slow_from_fast.down.weight", "sf_up": "slow_from_fast.up.weight",
    "sm_down": "slow_from_mid.down.weight", "sm_up": "slow_from_mid.up.weight",
    "bnd_w1": "boundary_mlp.0.weight", "bnd_b1": "boundary_mlp.0.bias",
    "bnd_w2": "boundary_mlp.2.weight", "bnd_b2": "boundary_mlp.2.bias",
    "sem_in": "semantic_in.weight", "sem_cond": "semantic_cond.weight", "sem_out": "semantic_out.weight",
    "fusion": "fusion_proj.weight",
}


def _sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def _silu(x):
    return (x * _sigmoid(x)).astype(np.float32)


def _lin(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return y.astype(np.float32)


def _bridge(x, down, up):
    """_LowRankBridge.forward (modeling.py:4182-4183)."""
    return _lin(_silu(_lin(x, down)), up)


def _band(prev, drive, gw, gb, cw, cb, gate_scale=None):
    """_update_band (modeling.py:4343-4356)."""
    gate = _sigmoid(_lin(drive, gw, gb))
    if gate_scale is not None:
        gate = (gate * gate_scale).astype(np.float32)
    cand = np.tanh(_lin(drive, cw, cb)).astype(np.float32)
    return ((1.0 - gate) * prev + gate * cand).astype(np.float32), gate


def recurrent_scan(w: dict, fast_in, mid_in, slow_in, init=None):
    """The recurrence of _forward_sequence_tensors (modeling.py:4449-4476) and
    _token_step (4363-4411) without the non-recurrent output projection.

    fast_in [B, T, F], mid_in [B, T, M], slow_in [B, T, S] (the three branch
    outputs).  Returns (states [B, T, F + M + S] -- the fast, mid and slow
    states after each token --, boundary_logits [B, T], fast, mid, slow)."""
    B, T, F = fast_in.shape
    M, S = mid_in.shape[2], slow_in.shape[2]
    if init is None:
        fast = np.zeros((B, F), np.float32)
        mid = np.zeros((B, M), np.float32)
        slow = np.zeros((B, S), np.float32)
    else:
        fast, mid, slow = (np.array(v, np.float32) for v in init)
    states = np.zeros((B, T, F + M + S), np.float32)
    logits = np.zeros((B, T), np.float32)
    for t in range(T):
        fast_drive = (fast_in[:, t] + _bridge(mid, w["fm_down"], w["fm_up"])
                      + _bridge(slow, w["fs_down"], w["fs_up"])).astype(np.float32)
        fast_new, fast_gate = _band(fast, fast_drive, w["fast_gate_w"], w["fast_gate_b"], w["fast_cand_w"],
                                    w["fast_cand_b"])
        mid_total = (mid_in[:, t] + _bridge(fast_new, w["mf_down"], w["mf_up"])
                     + _bridge(slow, w["ms_down"], w["ms_up"])).astype(np.float32)
        mid_new, mid_gate = _band(mid, mid_total, w["mid_gate_w"], w["mid_gate_b"], w["mid_cand_w"],
                                  w["mid_cand_b"])
        slow_total = (slow_in[:, t] + _bridge(fast_new, w["sf_down"], w["sf_up"])
                      + _bridge(mid_new, w["sm_down"], w["sm_up"])).astype(np.float32)
        feats = np.stack([
            fast_gate.mean(axis=-1),
            mid_gate.mean(axis=-1),
            np.sqrt(((mid_total - mid) ** 2).mean(axis=-1) + 1e-6),
            np.sqrt(((slow_total - slow) ** 2).mean(axis=-1) + 1e-6),
        ], axis=-1).astype(np.float32)
        logit = _lin(_silu(_lin(feats, w["bnd_w1"], w["bnd_b1"])), w["bnd_w2"], w["bnd_b2"])[:, 0]
        slow_new, _ = _band(slow, slow_total, w["slow_gate_w"], w["slow_gate_b"], w["slow_cand_w"],
                            w["slow_cand_b"], gate_scale=_sigmoid(logit)[:, None])
        fast, mid, slow = fast_new, mid_new, slow_new
        states[:, t] = np.concatenate([fast, mid, slow], axis=-1)
        logits[:, t] = logit
    return states, logits, fast, mid, slow


def fused_outputs(w: dict, normalised, states):
    """fusion_proj(cat(fast, mid, slow)) + _semantic_residual(token, mid, slow)
    for every token (modeling.py:4358-4361, 4406-4410)."""
    F = w["fast_gate_w"].shape[0]
    base = _lin(normalised, w["sem_in"])
    cond = _sigmoid(_lin(states[..., F:], w["sem_cond"]))
    return (_lin(states, w["fusion"]) + _lin((base * cond).astype(np.float32), w["sem_out"])).astype(np.float32)


def forward_sequence_tensors(w: dict, normalised, fast_in, mid_in, slow_in):
    """(outputs [B, T, H], boundary_logits [B, T], fast, mid, slow) as
    _forward_sequence_tensors returns them, from the branch outputs."""
    states, logits, fast, mid, slow = recurrent_scan(w, fast_in, mid_in, slow_in)
    out = fused_outputs(w, normalised, states)
    return out, logits, fast, mid, slow
