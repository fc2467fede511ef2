"""Build the in-tree native libraries for sm_100a.

* ``_lib/libsqa_b200.so`` (nvcc): every kernel and the plain C ABI
  (``include/small_q_attention.h``); no torch types cross it, so it builds
  without torch and is loaded with ctypes.
* ``_lib/_sqa_torch<ext>`` (g++ against torch's headers): the torch extension
  over that C ABI -- the ``torch.ops.sqa_b200`` operators and the direct entry
  the Python operator calls.  It computes nothing itself and links
  ``libsqa_b200.so`` from its own directory.

``python -m small_q_attention_b200.build`` (or ``__graft_entry__.build()``)
rebuilds each one when a source is newer than it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libsqa_b200.so"
SOURCES = ["sqa_split_kv.cu", "sqa_split_kv_tc.cu", "sqa_merge.cu", "sqa_api.cu", "sqa_noalloc.cu",
           "sqa_append.cu", "sqa_exchange.cu"]
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


def shared_runtime_cxx() -> str:
    """A C++ compiler that links the shared libstdc++ (the one torch uses).

    A compiler that only finds libstdc++.a would put a private copy of the C++
    runtime into the extension; C++ exceptions thrown there and rethrown by
    torch's error translation then cross two runtimes, which is undefined
    behaviour (it crashed in the unwinder on a CUDA host).  $CXX is taken when
    it qualifies, else the first g++ / c++ on PATH that does."""
    seen = []
    for cand in (os.environ.get("CXX"), "g++", "c++", "/usr/bin/g++"):
        exe = shutil.which(cand) if cand else None
        if not exe or exe in seen:
            continue
        seen.append(exe)
        res = subprocess.run([exe, "-print-file-name=libstdc++.so"], capture_output=True, text=True)
        found = res.stdout.strip()
        if res.returncode == 0 and os.path.isabs(found) and Path(found).exists():
            return exe
    raise RuntimeError(f"no C++ compiler on this host links the shared libstdc++ (tried {seen})")


TORCH_EXT_SOURCE = CSRC / "sqa_torch_op.cpp"
TORCH_EXT_PATH = LIB_DIR / ("_sqa_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def torch_ext_is_stale() -> bool:
    if not TORCH_EXT_PATH.exists():
        return True
    built = TORCH_EXT_PATH.stat().st_mtime
    deps = [TORCH_EXT_SOURCE, ROOT / "include" / "small_q_attention.h", Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch extension (host code only) if missing or stale; return its path."""
    if not force and not torch_ext_is_stale():
        return TORCH_EXT_PATH
    import torch
    from torch.utils import cpp_extension as ce

    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    includes = [Path(torch.__file__).resolve().parent / "include",
                Path(torch.__file__).resolve().parent / "include" / "torch" / "csrc" / "api" / "include",
                Path(cuda_home) / "include", Path(sysconfig.get_paths()["include"])]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_EXT_PATH.with_name(TORCH_EXT_PATH.name + ".tmp")
    cmd = [shared_runtime_cxx(), "-std=c++17", "-O2", "-g", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_sqa_torch",
           *[f"-I{p}" for p in includes], "-I", str(ROOT / "include"), str(TORCH_EXT_SOURCE), "-o", str(tmp),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           f"-L{Path(cuda_home) / 'lib64'}", "-lcudart", f"-L{LIB_DIR}", "-lsqa_b200",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_EXT_PATH)
    return TORCH_EXT_PATH


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


def build_all(force: bool = False, verbose: bool = False) -> list[Path]:
    """Both libraries: the kernels' C ABI first, then the torch extension that links it."""
    return [build(force=force, verbose=verbose), build_torch_ext(force=force, verbose=verbose)]


if __name__ == "__main__":
    for path in build_all(force="--force" in sys.argv, verbose=True):
        print(path)
