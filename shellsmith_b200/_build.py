"""Builds libshellcache.so (the C ABI) in-tree with nvcc for sm_100a only."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libshellcache.so"
SOURCES = ("status.cu", "gdn_decode.cu", "gdn_front.cu", "gdn_chunk.cu", "paged_kv.cu",
           "paged_attention.cu", "paged_q8.cu", "exchange.cu")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build shellcache")
    return found


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [CSRC / name for name in SOURCES] + list(CSRC.glob("*.cuh"))
    inputs.append(PACKAGE.parent / "include" / "shellcache.h")
    return any(p.stat().st_mtime > built for p in inputs if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel source into one shared library next to this file."""
    if not force and not _stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-o", str(tmp),
        *[str(CSRC / name) for name in SOURCES],
    ]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True, verbose=True))
