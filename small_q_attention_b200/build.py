"""Build the in-tree native library ``_lib/libsqa_b200.so`` with nvcc for sm_100a.

The library is a plain C-ABI shared object (``include/small_q_attention.h``):
no torch types cross it, so it builds without torch and is loaded with
ctypes.  ``python -m small_q_attention_b200.build`` (or
``__graft_entry__.build()``) rebuilds it when a source is newer than the
library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libsqa_b200.so"
SOURCES = ["sqa_split_kv.cu", "sqa_split_kv_tc.cu", "sqa_merge.cu", "sqa_api.cu", "sqa_noalloc.cu",
           "sqa_append.cu"]
HEADERS = ["sqa_internal.h", "sqa_ptx.cuh", "sqa_schedule.cuh", "sqa_merge_row.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-cudart", "static", "--threads", "0",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _inputs():
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [
        ROOT / "include" / "small_q_attention.h", Path(__file__)]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    """Compile the native library if missing or stale; return its path."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []),
           "-I", str(ROOT / "include"), *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
