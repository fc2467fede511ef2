"""ctypes binding of the C ABI in ``include/small_q_attention.h``.

The shared library is the only compute path: if it is missing or fails to
load, every operator raises ``RuntimeError``; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

# SQA_LIB_PATH selects another build of the library (for example one compiled
# with -DSQA_DEBUG_CHECKS); the default is the in-tree release build.
LIB_PATH = Path(os.environ.get("SQA_LIB_PATH") or Path(__file__).resolve().parent / "_lib" / "libsqa_b200.so")

# status codes (sqa_status)
SQA_OK = 0
SQA_ERR_INVALID_ARGUMENT = 1
SQA_ERR_UNSUPPORTED = 2
SQA_ERR_WORKSPACE_TOO_SMALL = 3
SQA_ERR_CUDA = 4
SQA_ERR_DEVICE = 5

# element types (SQA_DTYPE_*)
DTYPE_F16 = 0
DTYPE_BF16 = 1

# cache layouts (SQA_KV_*)
KV_NHD = 0
KV_HND = 1

# cache element types (SQA_KV_SAME / SQA_KV_FP8_E4M3)
KV_SAME = 0
KV_FP8_E4M3 = 1

# device status bits (SQA_DEV_*)
DEV_TIMEOUT = 1
DEV_SEQ_TOO_LONG = 2
DEV_SEQ_TOO_SHORT = 4
DEV_BAD_PAGE = 8
DEV_CHECK = 16

EXPORTED_SYMBOLS = (
    "sqa_workspace_bytes",
    "sqa_forward",
    "sqa_forward_timed",
    "sqa_forward_noalloc",
    "sqa_noalloc_read_device_status",
    "sqa_merge_partials",
    "sqa_read_device_status",
    "sqa_workspace_init",
    "sqa_status_string",
    "sqa_abi_version",
    "sqa_selected_kernel",
    "sqa_cache_append",
    "sqa_lc_handle_bytes",
    "sqa_lc_create",
    "sqa_lc_connect",
    "sqa_lc_exchange",
    "sqa_lc_read_status",
    "sqa_lc_disconnect",
    "sqa_lc_destroy",
)


class SqaAppendArgs(ctypes.Structure):
    """Mirror of ``struct sqa_append_args``."""

    _fields_ = [
        ("new_keys", ctypes.c_void_p),
        ("new_values", ctypes.c_void_p),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("max_pages", ctypes.c_int32),
        ("kv_layout", ctypes.c_int32),
        ("page_stride", ctypes.c_int64),
        ("kv_dtype", ctypes.c_int32),
    ]


class SqaArgs(ctypes.Structure):
    """Mirror of ``struct sqa_args``."""

    _fields_ = [
        ("query", ctypes.c_void_p),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("mask_lens", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_partial", ctypes.c_void_p),
        ("out_lse", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("max_pages", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("num_ctas", ctypes.c_int32),
        ("min_pages_per_cta", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("kv_layout", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("out_scale", ctypes.c_float),
        ("page_stride", ctypes.c_int64),
        ("kv_dtype", ctypes.c_int32),
        ("min_seq_len", ctypes.c_int32),
        ("cluster", ctypes.c_int32),
    ]


_lib = None
# Reentrant: torch_ext() holds it while it loads the C library through library().
_lock = threading.RLock()


def library(path: Path | None = None):
    """Load (once) and return the native library; raise if it is unavailable."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"native library {p} is missing; build it with "
                "`python -m small_q_attention_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(p))
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        lib.sqa_workspace_bytes.argtypes = [ctypes.POINTER(SqaArgs), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        lib.sqa_workspace_bytes.restype = sz
        lib.sqa_forward.argtypes = [ctypes.POINTER(SqaArgs), vp, sz, vp]
        lib.sqa_forward.restype = ctypes.c_int
        lib.sqa_forward_timed.argtypes = [ctypes.POINTER(SqaArgs), vp, sz, vp, vp, vp]
        lib.sqa_forward_timed.restype = ctypes.c_int
        lib.sqa_forward_noalloc.argtypes = [ctypes.POINTER(SqaArgs), vp]
        lib.sqa_forward_noalloc.restype = ctypes.c_int
        lib.sqa_noalloc_read_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, vp]
        lib.sqa_noalloc_read_device_status.restype = ctypes.c_int
        lib.sqa_merge_partials.argtypes = [vp, vp, i32, i64, vp, vp, vp, vp]
        lib.sqa_merge_partials.restype = ctypes.c_int
        lib.sqa_read_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, vp]
        lib.sqa_read_device_status.restype = ctypes.c_int
        lib.sqa_workspace_init.argtypes = [vp, sz, vp]
        lib.sqa_workspace_init.restype = ctypes.c_int
        lib.sqa_status_string.argtypes = [ctypes.c_int]
        lib.sqa_status_string.restype = ctypes.c_char_p
        lib.sqa_abi_version.argtypes = []
        lib.sqa_abi_version.restype = ctypes.c_int
        lib.sqa_selected_kernel.argtypes = [ctypes.POINTER(SqaArgs), ctypes.c_int]
        lib.sqa_selected_kernel.restype = ctypes.c_int
        lib.sqa_cache_append.argtypes = [ctypes.POINTER(SqaAppendArgs), vp]
        lib.sqa_cache_append.restype = ctypes.c_int
        lib.sqa_lc_handle_bytes.argtypes = []
        lib.sqa_lc_handle_bytes.restype = sz
        lib.sqa_lc_create.argtypes = [i32, i32, i64, ctypes.POINTER(vp), vp]
        lib.sqa_lc_create.restype = ctypes.c_int
        lib.sqa_lc_connect.argtypes = [vp, vp]
        lib.sqa_lc_connect.restype = ctypes.c_int
        lib.sqa_lc_exchange.argtypes = [vp, vp, vp, vp, i32, vp]
        lib.sqa_lc_exchange.restype = ctypes.c_int
        lib.sqa_lc_read_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, vp]
        lib.sqa_lc_read_status.restype = ctypes.c_int
        lib.sqa_lc_disconnect.argtypes = [vp]
        lib.sqa_lc_disconnect.restype = ctypes.c_int
        lib.sqa_lc_destroy.argtypes = [vp]
        lib.sqa_lc_destroy.restype = ctypes.c_int
        if path is None:
            _lib = lib
        return lib


_ext = None


def torch_ext():
    """Load (once) and return the torch extension module ``_sqa_torch`` (the direct
    entry of the Python operator, and the ``torch.ops.sqa_b200`` operators); it
    links the same ``libsqa_b200.so``.  Raises if it is missing: no fallback."""
    global _ext
    if _ext is not None:
        return _ext
    with _lock:
        if _ext is None:
            import importlib.util
            import sysconfig

            import torch  # noqa: F401  (the extension needs torch's libraries loaded first)

            path = LIB_PATH.parent / ("_sqa_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
            if not path.exists():
                raise RuntimeError(f"torch extension {path} is missing; build it with "
                                   "`python -m small_q_attention_b200.build`")
            library()  # the C ABI it calls (same file, loaded once)
            spec = importlib.util.spec_from_file_location("_sqa_torch", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _ext = mod
    return _ext


def status_string(code: int) -> str:
    return library().sqa_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    """Map a C status code to the Python exception the upstream would raise."""
    if code == SQA_OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code in (SQA_ERR_INVALID_ARGUMENT, SQA_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)
