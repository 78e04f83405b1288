"""Build recipe for the in-tree native library ``_lib/libfds_b200.so``.

One nvcc invocation, sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
static cudart, no torch headers: the library is a plain C ABI
(``include/fds_b200.h``) that any FFI can load. The built ``.so`` lives inside
the package directory so that it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libfds_b200.so"
INCLUDE_DIR = REPO_DIR / "include"

SOURCES = ["fds_capi.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA 12.8+ toolkit required to build the sm_100a library)")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh"))
    files += sorted(INCLUDE_DIR.glob("*.h"))
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > mtime for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it (or ``force``)."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
        "-I", str(INCLUDE_DIR),
        "-o", str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
