"""Build the native library ``latefuse_b200/lib/liblatefuse_b200.so`` for sm_100a.

The library is compiled in-tree with ``nvcc`` (no JIT cache): every ``.cu``
file under ``latefuse_b200/csrc`` is compiled for ``sm_100a`` and linked into
one shared object exposing the C ABI declared in ``include/latefuse_b200.h``.
``nvcc`` cross-compiles, so this runs on a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "liblatefuse_b200.so"
HEADER = REPO_DIR / "include" / "latefuse_b200.h"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; install the CUDA toolkit or set NVCC")


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = sources() + sorted(CSRC_DIR.glob("*.h")) + sorted(CSRC_DIR.glob("*.cuh")) + [HEADER]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the native library if any source is newer than it. Returns its path."""
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{REPO_DIR / 'include'}", *map(str, sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
