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
