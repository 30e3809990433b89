"""Build the sm_100a shared library ``libgfst_b200.so`` in-tree.

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel), then
nvcc links them into ``gfst_hmb_public_b200/libgfst_b200.so``.  An object is
rebuilt when its source or any header under ``csrc/`` or ``include/`` changed.

    python -m gfst_hmb_public_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "gfst_b200"
LIB_PATH = PKG_DIR / "libgfst_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE_DIR}",
    "-Xptxas",
    "-v",
]


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _headers_digest() -> str:
    h = hashlib.sha256()
    for path in sorted(list(CSRC_DIR.glob("*.cuh")) + list(CSRC_DIR.glob("*.h")) + list(INCLUDE_DIR.glob("*.h"))):
        h.update(path.name.encode())
        h.update(path.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def _compile(src: Path, obj: Path, stamp: Path, digest: str, nvcc: str) -> tuple[Path, str]:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    stamp.write_text(digest)
    return obj, proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile every CUDA source and link the shared library; returns its path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers_digest()
    sources = sorted(CSRC_DIR.glob("*.cu"))
    todo = []
    objects = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        stamp = BUILD_DIR / (src.stem + ".stamp")
        digest = hashlib.sha256((headers + hashlib.sha256(src.read_bytes()).hexdigest()).encode()).hexdigest()
        objects.append(obj)
        if force or not obj.exists() or not stamp.exists() or stamp.read_text() != digest:
            todo.append((src, obj, stamp, digest))
    if todo:
        workers = jobs or max(1, min(len(todo), os.cpu_count() or 1))
        with ThreadPoolExecutor(max_workers=workers) as pool:
            for obj, log in pool.map(lambda a: _compile(*a, nvcc), todo):
                if verbose:
                    sys.stderr.write(log)
    link_needed = force or bool(todo) or not LIB_PATH.exists()
    if not link_needed:
        lib_mtime = LIB_PATH.stat().st_mtime
        link_needed = any(obj.stat().st_mtime > lib_mtime for obj in objects)
    if link_needed:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        # cudart is linked statically; driver entry points (tensor-map encoding)
        # are fetched at run time with cudaGetDriverEntryPoint, so the library
        # loads on a machine without a GPU driver.
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register / spill reports")
    args = parser.parse_args()
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
