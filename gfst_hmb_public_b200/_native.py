"""ctypes binding of ``libgfst_b200.so`` (the C ABI declared in include/gfst_b200.h).

The library is loaded from this package directory.  There is no fallback: if it
is missing or fails to load, every op raises ``RuntimeError``.  Tensors are
passed as raw device pointers together with the current CUDA stream of their
device; non-zero status codes become ``RuntimeError`` with the library's
detail text.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_NAME = "libgfst_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

GFST_OK = 0
SIGN_FIRST_SIGNIFICANT = 0
SIGN_R_DIAG_POSITIVE = 1
DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F64 = 2

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_int64 = ctypes.c_int64
_c_float = ctypes.c_float

# name -> argtypes (every entry point returns int unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "gfst_status_string": [_c_int],
    "gfst_abi_version": [],
    "gfst_last_error": [],
    "gfst_frame_update_qr": [
        _c_void_p, _c_void_p, _c_void_p, _c_float, _c_void_p, _c_int64, _c_int, _c_int, _c_int,
        _c_float, _c_int, _c_void_p,
    ],
    "gfst_frame_stream": [
        _c_void_p, _c_void_p, _c_void_p, _c_float, _c_int64, _c_int, _c_int, _c_int, _c_int,
        _c_float, _c_int, _c_void_p, _c_int, _c_void_p,
    ],
    "gfst_frame_stream_ex": [
        _c_void_p, _c_void_p, _c_void_p, _c_float, _c_int64, _c_int, _c_int, _c_int, _c_int,
        _c_float, _c_int, _c_void_p, _c_int, _c_int, _c_void_p,
    ],
    "gfst_block_commit_mean": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_void_p,
    ],
    "gfst_block_topk": [
        _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,
        _c_void_p, _c_void_p,
    ],
    "gfst_check_device_errors": [_c_int],
    "gfst_block_tracker_stream": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, ctypes.c_double,
        ctypes.c_double, _c_float, _c_int, _c_void_p,
    ],
    "gfst_centroid_cell_commit": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_centroid_readout": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_exact_readout_collapse": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_global_features": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int,
        _c_void_p, _c_int, _c_float, ctypes.c_double, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_block_commit_eig": [
        _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_void_p, _c_int, ctypes.c_double,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_local_tracker_stream": [
        _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
        ctypes.c_double, ctypes.c_double, _c_float, _c_int, _c_void_p, _c_void_p,
    ],
    "gfst_topk_merge": [_c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p],
    "gfst_exact_readout": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_open_block_readout": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_int64, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_exact_topk_workspace_bytes": [_c_int64, _c_int],
    "gfst_exact_topk": [
        _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
        ctypes.c_size_t, _c_void_p,
    ],
    "gfst_exact_topk_noalloc": [
        _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_segmented_max": [_c_void_p, _c_void_p, _c_int64, _c_int64, _c_void_p, _c_void_p],
    "gfst_segmented_logsumexp_occurrence": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int64, _c_void_p, _c_void_p, _c_void_p,
        _c_void_p,
    ],
    "gfst_debug_bounded_wait": [_c_int64, _c_void_p],
    "gfst_exact_block_materialize": [_c_void_p, _c_int64, _c_int, _c_int64, _c_int64, _c_void_p, _c_void_p],
    "gfst_heev": [_c_void_p, _c_int64, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "gfst_exact_block_score": [
        _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
    ],
    "gfst_block_commit_i8": [_c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int, _c_void_p],
    "gfst_exact_readout_i8": [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
    ],
    "gfst_mpuc_scan_workspace_bytes": [_c_int64, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_size_t)],
    "gfst_mpuc_recurrent_scan": [
        _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int64, _c_int,
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p,
    ],
}
_RESTYPES = {
    "gfst_exact_topk_workspace_bytes": ctypes.c_size_t,
    "gfst_status_string": ctypes.c_char_p,
    "gfst_last_error": ctypes.c_char_p,
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def exported_symbols() -> list[str]:
    """Names this binding expects the library to export."""
    return list(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Load the library once (thread safe) and attach the ctypes signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_NAME} is not built ({LIB_PATH}); run `python -m gfst_hmb_public_b200.build` "
                "(the GFST-HMB B200 ops have no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        missing = [name for name in _SIGNATURES if not hasattr(lib, name)]
        if missing:
            raise RuntimeError(f"{LIB_PATH} does not export {missing}; rebuild the library")
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != GFST_OK:
        lib = load()
        text = lib.gfst_status_string(int(status)).decode()
        detail = lib.gfst_last_error().decode()
        raise RuntimeError(f"{what} failed: {text} (status {status}): {detail}")


def call(name: str, *args) -> None:
    """Invoke entry point ``name`` and raise on a non-OK status."""
    fn = getattr(load(), name)
    check(fn(*args), name)


def check_device_errors(clear: bool = True) -> None:
    """Raise RuntimeError when a kernel recorded a device-side failure since
    the last check: a bounded in-kernel wait that gave up (GFST_ERR_TIMEOUT) or
    an eigensolver that did not converge (GFST_ERR_NUMERIC).  Synchronises the
    current device first, so work enqueued on any stream before the call is
    covered; the recorded status is cleared unless ``clear`` is False.  Call it
    at a point where the host waits anyway (the end of a pass, before results
    are used); outputs of a launch that recorded a failure are not valid."""
    status = int(load().gfst_check_device_errors(1 if clear else 0))
    if status != GFST_OK:
        lib = load()
        raise RuntimeError(f"device-side failure: {lib.gfst_status_string(status).decode()} (status {status}): "
                           f"{lib.gfst_last_error().decode()}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else int(t.data_ptr())


def stream_of(t: torch.Tensor) -> int:
    return int(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors: torch.Tensor | None, what: str) -> torch.device:
    """All given tensors must be CUDA tensors on one device (no CPU fallback)."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{what}: expected a torch.Tensor, got {type(t).__name__}")
        if t.device.type != "cuda":
            raise RuntimeError(f"{what} requires CUDA tensors (got a tensor on {t.device}); there is no CPU path")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError(f"{what}: tensors on different devices ({device} and {t.device})")
    if device is None:
        raise RuntimeError(f"{what}: no tensor given")
    return device


def dtype_code(dtype: torch.dtype, what: str) -> int:
    if dtype == torch.float32:
        return DTYPE_F32
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise RuntimeError(f"{what}: unsupported dtype {dtype} (float32 or bfloat16)")
