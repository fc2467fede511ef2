"""Build recipe for the upstream's own CUDA extension, as a same-box GPU comparator.

TEST AND MEASUREMENT INFRASTRUCTURE ONLY.  Compiles the upstream translation
unit ``csrc/small_q_attention_ext.cu`` (kernels v0-v5 and the split-KV merge,
bound as ``forward``, ``forward_v1`` ... ``forward_v5``, ``ext.cu:1380-1390``)
unmodified, where it lies in the upstream tree, for sm_100a, with the upstream's
own flags (``-O3 --use_fast_math``, ``src/small_q_attention/cuda.py:34``), into
``oracle/_ref/`` (git-ignored; the built module travels to the GPU box with the
working tree).  Nothing in the product package imports it: ``tests/`` check it
against the CPU oracle and ``bench.py --impl reference`` times its v3 path
beside the CPU reference.

    python oracle/build_ref_gpu.py --reference <upstream checkout>

or ``SQA_REFERENCE_ROOT=<upstream checkout> python oracle/build_ref_gpu.py`` (default:
a ``reference`` checkout beside this repository).
The build needs only nvcc and torch's headers (no GPU); without the upstream
tree it does nothing.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
NAME = "small_q_attention_ext_ref"
DEFAULT_REFERENCE = HERE.parent.parent / "reference"  # an upstream checkout beside this repository


def reference_root(path: str | None = None) -> Path:
    return Path(path or os.environ.get("SQA_REFERENCE_ROOT") or DEFAULT_REFERENCE)


def built_module_path() -> Path | None:
    found = sorted(OUT_DIR.glob(f"{NAME}*.so"))
    return found[0] if found else None


def build(reference: str | None = None, verbose: bool = False) -> Path | None:
    """Compile the upstream extension if the upstream tree is present and the
    module is missing or older than its source; return the module path (or None)."""
    src = reference_root(reference) / "csrc" / "small_q_attention_ext.cu"
    if not src.exists():
        return built_module_path()
    existing = built_module_path()
    if existing is not None and existing.stat().st_mtime >= src.stat().st_mtime:
        return existing
    from torch.utils.cpp_extension import load

    sys.path.insert(0, str(HERE.parent))
    from small_q_attention_b200.build import shared_runtime_cxx

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    saved = os.environ.get("CXX")
    os.environ["CXX"] = shared_runtime_cxx()  # link the shared C++ runtime torch uses
    try:
        # an explicit -gencode makes torch add no arch flags of its own (no GPU is needed to build)
        load(name=NAME, sources=[str(src)], build_directory=str(OUT_DIR),
             extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode=arch=compute_100a,code=sm_100a"],
             verbose=verbose, is_python_module=True)
    finally:
        if saved is None:
            os.environ.pop("CXX", None)
        else:
            os.environ["CXX"] = saved
    return built_module_path()


def load_module():
    """Import the built upstream extension (raises if it was not built)."""
    path = built_module_path()
    if path is None:
        raise RuntimeError("the upstream extension is not built (python oracle/build_ref_gpu.py)")
    import torch  # noqa: F401  (the module links torch's libraries)

    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=None, help="upstream checkout (default: $SQA_REFERENCE_ROOT)")
    a = ap.parse_args()
    print(build(a.reference, verbose=True) or "upstream tree not found: nothing built", file=sys.stderr)
