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

SOURCES = ["fds_capi.cu", "fds_rope_static.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

# The attention kernels split their register file with setmaxnreg
# (csrc/attn_kernel.cuh RegSplit: 2 x 128 softmax threads at 224 or 208, 128
# control threads at 56 or 88). That
# split assumes the CTA is launched with exactly this many registers per
# thread; a different count could make the increase wait forever, so the build
# refuses to produce a library in that case.
ATTN_KERNEL_MARK = "attn_fwd_kernel"
ATTN_LAUNCH_REGS = 168


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
        nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xptxas=-v",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
        "-I", str(INCLUDE_DIR),
        "-o", str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    check_launch_registers(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def check_launch_registers(ptxas_log: str) -> None:
    """Every attention kernel entry must report ATTN_LAUNCH_REGS registers."""
    current, seen = None, 0
    for line in ptxas_log.splitlines():
        if "Compiling entry function" in line:
            current = line
        elif current and "Used" in line and "registers" in line:
            if ATTN_KERNEL_MARK in current:
                regs = int(line.split("Used")[1].split("registers")[0])
                if regs != ATTN_LAUNCH_REGS:
                    raise RuntimeError(f"attention kernel launches with {regs} registers per thread, expected "
                                       f"{ATTN_LAUNCH_REGS} (the setmaxnreg split depends on it): {current}")
                seen += 1
            current = None
    if seen == 0:
        raise RuntimeError("no attention kernel found in the ptxas report")


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
