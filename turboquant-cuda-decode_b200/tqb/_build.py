"""Build recipe for ``libtqb.so`` (the sm_100a kernels behind the C ABI).

The library is compiled in-tree with ``nvcc`` for ``sm_100a`` only and
links the CUDA runtime statically, so the ``.so`` has no torch dependency and
travels with the source tree.  ``python -m tqb._build`` (with the package
directory on ``sys.path``) or ``__graft_entry__.build()`` runs it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parent.parent / "include"
LIB_PATH = PKG_DIR / "libtqb.so"

SOURCES = ["tqb_api.cu", "tqb_stage1.cu", "tqb_stage1_ring.cu", "tqb_stage2.cu", "tqb_store.cu", "tqb_noalloc.cu",
           "tqb_rotate.cu", "tqb_p2p.cu"]
HEADERS = ["tqb_common.cuh", "tqb_internal.h", "tqb_merge_row.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "tqb.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile ``libtqb.so`` if it is missing or older than its sources."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []),
           f"-I{INCLUDE}", "-shared", "-o", str(tmp),
           *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
