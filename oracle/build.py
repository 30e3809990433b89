"""Build the C restatement ``oracle/_build/libgfst_oracle.so`` with gcc.

TEST INFRASTRUCTURE ONLY: the library is a checker for the tests; nothing in
the product package loads it.  Compiled with -ffp-contract=off to mirror the
reference's --fmad=false build of the kernel it restates.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "householder.c"
OUT_DIR = ORACLE_DIR / "_build"
LIB = OUT_DIR / "libgfst_oracle.so"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(LIB), str(SRC), "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        fn = lib.gfst_oracle_qr_fixed_order
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                       ctypes.c_float, ctypes.c_int]
        _lib = lib
    return _lib


def qr_fixed_order(matrices: np.ndarray, eps_sign: float = 1e-8, sign_mode: int = 0) -> np.ndarray:
    """Fixed-order fp32 Householder thin Q of [..., m, n] matrices, sign-fixed."""
    a = np.ascontiguousarray(matrices, dtype=np.float32)
    m, n = a.shape[-2], a.shape[-1]
    batch = int(np.prod(a.shape[:-2])) if a.ndim > 2 else 1
    out = np.empty_like(a)
    rc = load().gfst_oracle_qr_fixed_order(a.ctypes.data, out.ctypes.data, batch, m, n, float(eps_sign),
                                           int(sign_mode))
    if rc != 0:
        raise ValueError(f"gfst_oracle_qr_fixed_order rejected shape {a.shape}")
    return out


if __name__ == "__main__":
    print(build(force=True))
