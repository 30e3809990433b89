"""Import the reference's own Python modules -- TEST INFRASTRUCTURE ONLY.

The reference package (pkhairkh/gfst-hmb-public, import name ``gfst_hmb_mpuc``)
cannot be imported as shipped: its ``__init__`` pulls in training modules that
the public release leaves out, and ``runtime_backends/__init__.py`` re-exports
from ``runtime_backends/sm120.py``, which the release also omits.  This module
registers namespace packages that point into a copy of its source tree and a
``runtime_backends.sm120`` module of the caller's choice:

* ``backend=None``: every accelerated op returns ``None`` / ``False``, so each
  caller takes the reference's own torch branch (the reference as published,
  run on the CPU);
* ``backend=<module>``: the ops of that module (e.g. this repository's B200
  binding, ``gfst_hmb_public_b200.sm120_binding``), so the reference's own
  callers run through it.

Two places hold a copy of the reference: the source checkout (``<root>/src``)
and the offline install ``baseline/_ref`` (``pip install --target``), which
travels with this repository to GPU hosts.  ``find_reference()`` looks for the
install first.  Used by tests/, tests/golden/make_golden.py and bench.py's CPU
baseline / reference arm; never by the product package.
"""
from __future__ import annotations

import importlib
import os
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]

# accelerated entry points of runtime_backends/__init__.py:1-28 and what the
# "unavailable" stub returns for each
_OPS = ("exact_block_score", "exact_block_materialize", "gfst_block_commit", "gfst_heev",
        "gfst_reference_block_average", "gfst_reference_global_sketch", "gfst_local_qr",
        "gfst_global_sketch", "gfst_canonical_summary_from_eigpairs", "gfst_summary_from_sketch",
        "gfst_summary_from_sketch_batched", "load_sm120_extension", "load_mathdx_extension",
        "mathdx_extension_dependency_report", "mathdx_runtime_dependency_report", "mpuc_recurrent_scan",
        "segmented_logsumexp_occurrence", "segmented_max_by_group")
_FLAGS = ("exact_readout_score_available", "experimental_canonical_summary_enabled",
          "mathdx_extension_available", "mpuc_recurrent_scan_available", "segmented_reduction_available",
          "sm120_exact_math_kernels_available")


def find_reference() -> Path | None:
    """Directory of the ``gfst_hmb_mpuc`` package: ``baseline/_ref`` (the offline
    install) or ``$GFST_REFERENCE_SRC`` (a source checkout's ``src`` directory
    or its root).  None when neither exists."""
    cand = [REPO / "baseline" / "_ref" / "gfst_hmb_mpuc"]
    env = os.environ.get("GFST_REFERENCE_SRC")
    if env:
        p = Path(env)
        cand += [p / "gfst_hmb_mpuc", p / "src" / "gfst_hmb_mpuc"]
    for c in cand:
        if (c / "gfst.py").is_file():
            return c
    return None


def _stub_backend() -> types.ModuleType:
    sm = types.ModuleType("gfst_hmb_mpuc.runtime_backends.sm120")

    def _none(*args, **kwargs):
        return None

    def _false(*args, **kwargs):
        return False

    for name in _OPS:
        setattr(sm, name, _none)
    for name in _FLAGS:
        setattr(sm, name, _false)
    return sm


def install(pkg_dir: Path | str, backend: types.ModuleType | None = None):
    """Register ``gfst_hmb_mpuc`` (namespace packages over ``pkg_dir``) with the
    given sm120 backend and return ``importlib`` for convenience.  Replaces any
    earlier registration (modules of an earlier one are dropped)."""
    pkg_dir = Path(pkg_dir)
    for name in [m for m in sys.modules if m == "gfst_hmb_mpuc" or m.startswith("gfst_hmb_mpuc.")]:
        del sys.modules[name]
    pkg = types.ModuleType("gfst_hmb_mpuc")
    pkg.__path__ = [str(pkg_dir)]
    sys.modules["gfst_hmb_mpuc"] = pkg
    for sub in ("diagnostics", "training"):
        m = types.ModuleType(f"gfst_hmb_mpuc.{sub}")
        m.__path__ = [str(pkg_dir / sub)]
        sys.modules[f"gfst_hmb_mpuc.{sub}"] = m
    sm = _stub_backend()
    if backend is not None:
        for name in _OPS + _FLAGS:
            if hasattr(backend, name):
                setattr(sm, name, getattr(backend, name))
    rb = types.ModuleType("gfst_hmb_mpuc.runtime_backends")
    rb.__path__ = [str(pkg_dir / "runtime_backends")]
    sys.modules["gfst_hmb_mpuc.runtime_backends.sm120"] = sm
    for name in _OPS + _FLAGS:
        setattr(rb, name, getattr(sm, name))
    rb.sm120 = sm
    sys.modules["gfst_hmb_mpuc.runtime_backends"] = rb
    return importlib


def load(module: str, pkg_dir: Path | str | None = None, backend: types.ModuleType | None = None):
    """Import ``gfst_hmb_mpuc.<module>`` from the reference (``find_reference()``
    unless ``pkg_dir`` is given).  Raises FileNotFoundError when no copy exists."""
    pkg_dir = pkg_dir if pkg_dir is not None else find_reference()
    if pkg_dir is None:
        raise FileNotFoundError("no copy of the reference package (baseline/_ref or $GFST_REFERENCE_SRC)")
    install(pkg_dir, backend)
    return importlib.import_module(f"gfst_hmb_mpuc.{module}")


def reference_mpuc_cell(modeling, hidden: int, seed: int):
    """A reference MpucGfstHmbBlock that holds only its recurrent cell: the
    submodules that _forward_sequence / _forward_sequence_tensors use
    (modeling.py:4417-4476), built with the reference's own constructors and
    sizes (MpucGfstHmbBlock.__init__, modeling.py:4259-4315: fast = H/2,
    mid = H/4, slow = the rest, cross and semantic rank max(64, H/16),
    boundary hidden max(8, H/16), branch specs (3, 1), (5, 2), (9, 4)), with
    nn.Linear's default initialisation under torch.manual_seed(seed).  The
    GFST sublayer is left out (the cell never touches it)."""
    import torch

    nn = torch.nn
    cls = modeling.MpucGfstHmbBlock
    torch.manual_seed(seed)
    blk = cls.__new__(cls)
    nn.Module.__init__(blk)
    H = int(hidden)
    blk.hidden_size = H
    blk.fast_dim, blk.mid_dim = H // 2, H // 4
    blk.slow_dim = H - blk.fast_dim - blk.mid_dim
    blk.cross_rank = max(64, H // 16)
    blk.semantic_rank = max(64, H // 16)
    F, M, S, C = blk.fast_dim, blk.mid_dim, blk.slow_dim, blk.cross_rank
    br = modeling._CausalDepthwiseBranch
    blk.fast_branch = br(H, F, kernel_size=3, dilation=1)
    blk.mid_branch = br(H, M, kernel_size=5, dilation=2)
    blk.slow_branch = br(H, S, kernel_size=9, dilation=4)
    lr = modeling._LowRankBridge
    blk.fast_from_mid, blk.fast_from_slow = lr(M, F, C), lr(S, F, C)
    blk.mid_from_fast, blk.mid_from_slow = lr(F, M, C), lr(S, M, C)
    blk.slow_from_fast, blk.slow_from_mid = lr(F, S, C), lr(M, S, C)
    blk.fast_gate_proj, blk.fast_cand_proj = nn.Linear(F, F), nn.Linear(F, F)
    blk.mid_gate_proj, blk.mid_cand_proj = nn.Linear(M, M), nn.Linear(M, M)
    blk.slow_gate_proj, blk.slow_cand_proj = nn.Linear(S, S), nn.Linear(S, S)
    bh = max(8, H // 16)
    blk.boundary_mlp = nn.Sequential(nn.Linear(4, bh), nn.SiLU(), nn.Linear(bh, 1))
    blk.semantic_in = nn.Linear(H, blk.semantic_rank, bias=False)
    blk.semantic_cond = nn.Linear(M + S, blk.semantic_rank, bias=False)
    blk.semantic_out = nn.Linear(blk.semantic_rank, H, bias=False)
    blk.fusion_proj = nn.Linear(H, H, bias=False)
    blk.recurrent_kernel_backend = "native"
    blk.recurrent_compile_mode = "max-autotune-no-cudagraphs"
    blk.runtime_profiler_mode = "off"
    blk._runtime_profile_recorder = None
    blk._compiled_forward_sequence_impl = None
    blk.last_forward_stats = None
    blk.last_boundary_logits = None
    return blk
