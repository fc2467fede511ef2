"""Public operator: causal paged MTP attention on B200 through the C ABI.

``small_q_attention(query, key_cache, value_cache, block_tables, seq_lens,
page_size, max_seq_len=0)`` keeps the positional contract of the upstream
``small_q_attention.cuda.forward_v3`` (``src/small_q_attention/cuda.py:177-214``)
and its error behaviour: ``RuntimeError`` without CUDA, ``ValueError`` for a
tensor that is not on CUDA, not contiguous, of the wrong dtype or outside the
shape contract (``cuda.py:197-211``).  It launches on the current torch
stream (the upstream launches on the legacy default stream,
``csrc/small_q_attention_ext.cu:1187``), never synchronises the host, and
reuses one workspace per (device, stream) instead of allocating fp32 scratch
on every call (``ext.cu:1183-1185``).

The operator itself runs through the torch extension (``csrc/sqa_torch_op.cpp``):
its contract checks, argument packing, workspace lookup and launches are C++,
so a call costs a few microseconds of host time; the same code is registered as
``torch.ops.sqa_b200.small_q_attention`` / ``small_q_attention_partial`` for
``torch.compile``.  The ctypes helpers below (``_check_inputs``,
``_fill_args``) serve the C-ABI-level entry points (plan/run wrapper, merge,
tests).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native

HEAD_DIM = 128
PAGE_SIZE = 16
GQA_GROUP = 4
MAX_Q_LEN = 16

_DTYPES = (torch.float16, torch.bfloat16)
_FP8 = getattr(torch, "float8_e4m3fn", None)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_cuda_ok: bool | None = None


def _stream_handle(device: torch.device) -> int:
    """cudaStream_t of torch's current stream on ``device`` (the raw handle lookup
    avoids building a Stream object on every call)."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _cuda_available() -> bool:
    global _cuda_ok
    if _cuda_ok is None:
        _cuda_ok = torch.cuda.is_available()
    return _cuda_ok


class _on_device:
    """``torch.cuda.device(device)`` only when it is not already current (the
    context manager costs several microseconds per call)."""

    __slots__ = ("index", "prev")

    def __init__(self, device: torch.device):
        self.index = device.index

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.index:
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev != self.index:
            torch.cuda.set_device(self.prev)
        return False


_LAYOUTS = {"NHD": 0, "HND": 1}


def _layout_code(kv_layout: str) -> int:
    code = _LAYOUTS.get(kv_layout)
    if code is None:
        raise ValueError('kv_layout must be "NHD" ([pages, 16, Hkv, 128]) or "HND" ([pages, Hkv, 16, 128])')
    return code


def _cache_page_stride(key_cache, value_cache) -> int:
    """Elements from one page to the next (0 = contiguous caches).

    The caches may be views with a larger page stride, e.g. ``kv[:, 0]`` / ``kv[:, 1]``
    of a ``[pages, 2, ...]`` pool or one layer of a multi-layer pool: every dim but
    the page dim must be packed, the page stride a multiple of 8 elements, and K
    and V must have the same strides.
    """
    if key_cache.dim() != 4:
        raise ValueError("key_cache must be 4-D")
    if key_cache.is_contiguous() and value_cache.is_contiguous():
        return 0
    st = key_cache.stride()
    inner = key_cache.shape[1] * key_cache.shape[2] * key_cache.shape[3]
    packed = (key_cache.shape[2] * key_cache.shape[3], key_cache.shape[3], 1)
    align = 16 // key_cache.element_size()  # 16-byte aligned pages
    if value_cache.stride() != st or tuple(st[1:]) != packed or st[0] < inner or st[0] % align:
        raise ValueError("key_cache / value_cache must be packed within a page, with one page stride "
                         "(16-byte aligned) shared by K and V")
    return int(st[0])


def _check_inputs(query, key_cache, value_cache, block_tables, seq_lens, page_size, mask_lens=None,
                  kv_layout: str = "NHD"):
    if not _cuda_available():
        raise RuntimeError("CUDA is required for the small-q attention kernel")
    tensors = (query, key_cache, value_cache, block_tables, seq_lens) + ((mask_lens,) if mask_lens is not None else ())
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        raise ValueError("all inputs must be CUDA tensors")
    dev = query.device
    if dev.type != "cuda":
        raise ValueError("all inputs must be CUDA tensors")
    for i, t in enumerate(tensors):
        if t.device != dev:
            raise ValueError("all inputs must be CUDA tensors on the same device")
        if i not in (1, 2) and not t.is_contiguous():
            raise ValueError("all inputs must be contiguous")
    _cache_page_stride(key_cache, value_cache)
    qd = query.dtype
    kd = key_cache.dtype
    if qd not in _DTYPES or value_cache.dtype != kd or not (kd == qd or (kd == _FP8 and _FP8 is not None)):
        raise ValueError("the kernel requires FP16 (or BF16) Q/K/V of one type, or FP16/BF16 Q with FP8-E4M3 K/V")
    for t in tensors[3:]:
        if t.dtype != torch.int32:
            raise ValueError("block_tables, seq_lens and mask_lens must be int32")
    if query.dim() != 4 or key_cache.dim() != 4:
        raise ValueError("query and key_cache must be 4-D")
    kshape = key_cache.shape
    if value_cache.shape != kshape:
        raise ValueError("value_cache shape mismatch")
    batch, q_len, hq, head_dim = query.shape
    if _layout_code(kv_layout):
        _, hkv, cache_page, cache_dim = kshape
    else:
        _, cache_page, hkv, cache_dim = kshape
    if not (1 <= q_len <= MAX_Q_LEN):
        raise ValueError(f"q_len must be in [1, {MAX_Q_LEN}]")
    if head_dim != HEAD_DIM or cache_dim != HEAD_DIM:
        raise ValueError("the kernel supports head_dim 128")
    if hq % hkv != 0 or hq // hkv != GQA_GROUP:
        raise ValueError("the kernel requires a GQA group size of exactly 4 (Hq/Hkv = 32/8)")
    if int(page_size) != cache_page or cache_page != PAGE_SIZE:
        raise ValueError("page_size must be 16 and match the cache's page dimension")
    if block_tables.dim() != 2 or block_tables.shape[0] != batch or seq_lens.numel() != batch:
        raise ValueError("invalid metadata: block_tables must be [batch, max_pages], seq_lens [batch]")
    if mask_lens is not None and mask_lens.numel() != batch:
        raise ValueError("mask_lens must have one entry per sequence")
    if kshape[0] == 0 or block_tables.shape[1] == 0:
        raise ValueError("empty KV cache is not supported")


def _fill_args(query, key_cache, value_cache, block_tables, seq_lens, mask_lens, max_seq_len,
               num_ctas, min_pages_per_cta, kernel: int = 0, kv_layout: str = "NHD", sm_scale=None,
               out_scale: float = 1.0) -> _native.SqaArgs:
    batch, q_len, hq, head_dim = query.shape
    layout = _layout_code(kv_layout)
    if layout:
        num_pages, hkv, page_size, _ = key_cache.shape
    else:
        num_pages, page_size, hkv, _ = key_cache.shape
    return _native.SqaArgs(
        query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_tables.data_ptr(),
        seq_lens.data_ptr(), mask_lens.data_ptr() if mask_lens is not None else None, None, None, None,
        batch, q_len, hq, hkv, head_dim, page_size, num_pages, block_tables.shape[1], int(max_seq_len),
        int(num_ctas), int(min_pages_per_cta), int(kernel),
        _native.DTYPE_BF16 if query.dtype == torch.bfloat16 else _native.DTYPE_F16, layout,
        0.0 if sm_scale is None else float(sm_scale), float(out_scale),
        _cache_page_stride(key_cache, value_cache),
        _native.KV_FP8_E4M3 if key_cache.dtype == _FP8 else _native.KV_SAME)


def selected_kernel(query, key_cache, value_cache, block_tables, seq_lens, page_size,
                    max_seq_len: int = 0, *, num_ctas: int = 0, min_pages_per_cta: int = 0,
                    kernel: int = 0, kv_layout: str = "NHD", min_seq_len: int = 0, cluster: int = 0) -> int:
    """The kernel a call with these shapes launches: 1 = warp-level mma.sync,
    2 = tcgen05, 2 + 100 * C = tcgen05 in clusters of C CTAs (``kernel=0`` and
    ``cluster=0`` resolved the way ``small_q_attention`` resolves them)."""
    _check_inputs(query, key_cache, value_cache, block_tables, seq_lens, page_size, kv_layout=kv_layout)
    args = _fill_args(query, key_cache, value_cache, block_tables, seq_lens, None, max_seq_len,
                      num_ctas, min_pages_per_cta, kernel, kv_layout)
    args.min_seq_len, args.cluster = int(min_seq_len), int(cluster)
    code = _native.library().sqa_selected_kernel(ctypes.byref(args), query.device.index)
    if code < 0:
        _native.check(-code, "sqa_selected_kernel")
    return int(code)


def workspace_bytes(query, key_cache, value_cache, block_tables, seq_lens, page_size,
                    max_seq_len: int = 0, *, num_ctas: int = 0, min_pages_per_cta: int = 0,
                    kernel: int = 0, kv_layout: str = "NHD") -> int:
    """Bytes of workspace ``small_q_attention`` needs for these shapes."""
    _check_inputs(query, key_cache, value_cache, block_tables, seq_lens, page_size, kv_layout=kv_layout)
    args = _fill_args(query, key_cache, value_cache, block_tables, seq_lens, None, max_seq_len,
                      num_ctas, min_pages_per_cta, kernel, kv_layout)
    st = ctypes.c_int(0)
    need = _native.library().sqa_workspace_bytes(ctypes.byref(args), query.device.index, ctypes.byref(st))
    _native.check(st.value, "sqa_workspace_bytes")
    return int(need)


def read_device_status(workspace_ptr: int, clear: bool = True, device=None) -> int:
    """Synchronise and return the sticky SQA_DEV_* bits of a workspace."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    bits = ctypes.c_uint32(0)
    code = _native.library().sqa_read_device_status(
        ctypes.c_void_p(workspace_ptr), ctypes.byref(bits), int(clear), ctypes.c_void_p(_stream_handle(dev)))
    if code not in (_native.SQA_OK, _native.SQA_ERR_DEVICE):
        _native.check(code, "sqa_read_device_status")
    return int(bits.value)


def _raise_device_bits(bits: int) -> None:
    if bits & _native.DEV_SEQ_TOO_SHORT:
        raise ValueError("seq_lens must be at least q_len for MTP attention")
    if bits & _native.DEV_SEQ_TOO_LONG:
        raise ValueError("seq_lens exceeds page_size * block_tables.shape[1]")
    if bits & _native.DEV_BAD_PAGE:
        raise IndexError("block_tables holds a page id outside the cache")
    if bits & _native.DEV_TIMEOUT:
        raise RuntimeError("a bounded device wait timed out; the output is not valid")


def small_q_attention(query, key_cache, value_cache, block_tables, seq_lens, page_size: int,
                      max_seq_len: int = 0, *, out=None, workspace=None, num_ctas: int = 0,
                      min_pages_per_cta: int = 0, kernel: int = 0, check: bool = False,
                      kv_layout: str = "NHD", sm_scale: float | None = None, out_scale: float = 1.0,
                      min_seq_len: int = 0, cluster: int = 0):
    """Causal paged MTP attention; returns ``[batch, q_len, Hq, 128]`` in the input type.

    Q/K/V are FP16 (the upstream contract) or BF16 (all three of one type;
    accumulation is FP32 either way), or FP16/BF16 Q with FP8-E4M3 K/V (tcgen05
    kernel, read as fp8 by the tensor core; Q and the probabilities enter as
    two e4m3 parts each; pass the caches' dequantisation scales as
    ``sm_scale = k_scale / sqrt(128)`` and ``out_scale = v_scale``).

    ``seq_lens[b]`` is the KV length including the ``q_len`` draft tokens and
    draft row ``qi`` sees tokens ``< seq_lens[b] - q_len + qi + 1``
    (``src/small_q_attention/reference.py:63``).  ``max_seq_len`` is an
    optional upper bound of ``seq_lens`` that only sizes the launch (0: use the
    page-table width); unlike the upstream (``ext.cu:1173-1176``) it is never
    measured with a device-to-host copy.  ``check=True`` synchronises and
    raises the exception the upstream CPU reference would raise for bad
    metadata (``seq_lens < q_len``, page ids outside the pool).  ``kernel``
    selects the implementation: 0 auto, 1 warp-level mma.sync, 2 tcgen05 with
    tensor memory (same operator).  ``kv_layout`` "HND" takes caches as
    ``[pages, Hkv, 16, 128]``; ``sm_scale`` (default ``128**-0.5``) scales q.k and
    ``out_scale`` every output row (FlashInfer's ``bmm1_scale`` / ``bmm2_scale``).
    ``min_seq_len`` (a lower bound of ``seq_lens``, 0 = unknown) lets the launch
    split each (sequence, KV head) over a thread-block cluster when lengths are
    near-uniform; ``cluster`` forces that mode (2/4/8/16 CTAs) or turns it off (1).
    Both only steer the launch: the result is the same operator.
    """
    if not _cuda_available():
        raise RuntimeError("CUDA is required for the small-q attention kernel")
    try:
        return _native.torch_ext().forward(
            query, key_cache, value_cache, block_tables, seq_lens, page_size, max_seq_len, out, workspace,
            num_ctas, min_pages_per_cta, kernel, check, _layout_code(kv_layout),
            0.0 if sm_scale is None else sm_scale, out_scale, min_seq_len, cluster)
    except TypeError as e:  # a non-tensor where a tensor belongs (pybind11's argument check)
        raise ValueError(f"all inputs must be CUDA tensors ({e})") from None


def small_q_attention_partial(query, key_cache, value_cache, block_tables, seq_lens, page_size: int,
                              mask_lens=None, max_seq_len: int = 0, *, out=None, out_lse=None,
                              workspace=None, num_ctas: int = 0, min_pages_per_cta: int = 0,
                              kernel: int = 0, check: bool = False, kv_layout: str = "NHD",
                              sm_scale: float | None = None, out_scale: float = 1.0, min_seq_len: int = 0,
                              cluster: int = 0):
    """Attention over the tokens this call holds; returns ``(O fp32, LSE fp32)``.

    The shard form of the operator for splitting one sequence's KV range:
    the cache/page table hold tokens ``[offset, offset + seq_lens[b])`` of a
    sequence whose whole length minus ``offset`` is ``mask_lens[b]`` (default
    ``seq_lens``).  ``O`` is the normalised output ``[B, q_len, Hq, 128]`` and
    ``LSE`` the natural-log log-sum-exp ``[B, q_len, Hq]`` (-inf for a row
    that sees no key here).  Combine shards with :func:`merge_partials`.
    """
    if not _cuda_available():
        raise RuntimeError("CUDA is required for the small-q attention kernel")
    try:
        return _native.torch_ext().forward_partial(
            query, key_cache, value_cache, block_tables, seq_lens, page_size, mask_lens, max_seq_len, out, out_lse,
            workspace, num_ctas, min_pages_per_cta, kernel, check, _layout_code(kv_layout),
            0.0 if sm_scale is None else sm_scale, out_scale, min_seq_len, cluster)
    except TypeError as e:
        raise ValueError(f"all inputs must be CUDA tensors ({e})") from None


def merge_partials(parts_o, parts_lse, *, out=None, out_dtype=torch.float16, return_lse: bool = False):
    """Log-sum-exp merge of stacked partials ``[n, ..., 128]`` / ``[n, ...]``.

    Returns the merged output in ``out_dtype`` (fp16, bf16 or fp32) and, with
    ``return_lse``, the merged LSE.  Same arithmetic as the upstream split-KV
    merge (``csrc/small_q_attention_ext.cu:339-366``).  BF16 output is merged in
    fp32 and rounded once (``sqa_merge_partials`` writes fp16 or fp32).
    """
    if not (parts_o.is_cuda and parts_lse.is_cuda):
        raise ValueError("partials must be CUDA tensors")
    if parts_o.dtype != torch.float32 or parts_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    if not (parts_o.is_contiguous() and parts_lse.is_contiguous()):
        raise ValueError("partials must be contiguous")
    if parts_o.shape[-1] != HEAD_DIM or parts_o.shape[:-1] != parts_lse.shape:
        raise ValueError("parts_o must be [n, ..., 128] and parts_lse [n, ...]")
    n = int(parts_o.shape[0])
    rows = parts_lse[0].numel() if n else 0
    shape = parts_o.shape[1:]
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=parts_o.device)
    if out.dtype not in (torch.float16, torch.bfloat16, torch.float32) or out.shape != shape:
        raise ValueError("out must be fp16, bf16 or fp32 and shaped like one part")
    if out.dtype == torch.bfloat16:
        merged = merge_partials(parts_o, parts_lse, out_dtype=torch.float32, return_lse=return_lse)
        o32, lse = merged if return_lse else (merged, None)
        out.copy_(o32)
        return (out, lse) if return_lse else out
    lse = torch.empty(parts_lse.shape[1:], dtype=torch.float32, device=parts_o.device) if return_lse else None
    o16 = out.data_ptr() if out.dtype == torch.float16 else None
    o32 = out.data_ptr() if out.dtype == torch.float32 else None
    with _on_device(parts_o.device):
        code = _native.library().sqa_merge_partials(
            ctypes.c_void_p(parts_o.data_ptr()), ctypes.c_void_p(parts_lse.data_ptr()), n, rows,
            ctypes.c_void_p(o16), ctypes.c_void_p(o32),
            ctypes.c_void_p(lse.data_ptr() if lse is not None else None),
            ctypes.c_void_p(_stream_handle(parts_o.device)))
    _native.check(code, "sqa_merge_partials")
    return (out, lse) if return_lse else out
