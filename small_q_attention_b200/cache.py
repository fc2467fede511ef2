"""The cache-append step before MTP attention.

``cache_append(new_keys, new_values, key_cache, value_cache, block_tables,
seq_lens)`` writes the K/V of the ``q_len`` new (draft) tokens of every
sequence into their page slots, in place: token ``qi`` of sequence ``b`` is
position ``t = seq_lens[b] - q_len + qi`` (``seq_lens`` is the length after the
append, as the attention takes it: ``src/small_q_attention/reference.py:25``),
stored in page ``block_tables[b, t // 16]``, slot ``t % 16``.  The upstream
leaves this step to its caller.  One CUDA kernel (``sqa_cache_append``), a pure
copy; a following ``small_q_attention`` on the same stream sees the new K/V.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _native
from .attention import (HEAD_DIM, PAGE_SIZE, _cache_page_stride, _cuda_available, _layout_code, _on_device,
                        _raise_device_bits, _stream_handle, read_device_status)

_status_lock = threading.Lock()
_status_words: dict[tuple[int, int], torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    key = (device.index, _stream_handle(device))
    with _status_lock:
        w = _status_words.get(key)
        if w is None:
            w = torch.zeros(256, dtype=torch.uint8, device=device)
            _status_words[key] = w
    return w


def cache_append(new_keys, new_values, key_cache, value_cache, block_tables, seq_lens, *,
                 check: bool = False, kv_layout: str = "NHD"):
    """Write ``new_keys`` / ``new_values`` ``[batch, q_len, Hkv, 128]`` into the
    paged caches ``[num_pages, 16, Hkv, 128]`` (``kv_layout="HND"``:
    ``[num_pages, Hkv, 16, 128]``) in place; returns the caches.

    Errors of the contract (dtype, device, shape, contiguity) raise ``ValueError``
    before launch.  With ``check=True`` the call synchronises and raises
    ``ValueError`` for ``seq_lens < q_len`` or lengths beyond the page table and
    ``IndexError`` for a page id outside the cache (those tokens are not written).
    """
    if not _cuda_available():
        raise RuntimeError("CUDA is required for the cache-append kernel")
    tensors = [new_keys, new_values, key_cache, value_cache, block_tables, seq_lens]
    if any(not isinstance(t, torch.Tensor) or not t.is_cuda for t in tensors):
        raise ValueError("all inputs must be CUDA tensors")
    if any(t.device != key_cache.device for t in tensors):
        raise ValueError("all inputs must be on the same CUDA device")
    if any(not t.is_contiguous() for t in (new_keys, new_values, block_tables, seq_lens)):
        raise ValueError("all inputs must be contiguous")
    fp8 = getattr(torch, "float8_e4m3fn", None)
    if new_keys.dtype not in (torch.float16, torch.bfloat16, fp8) or any(t.dtype != new_keys.dtype
                                                                          for t in tensors[1:4]):
        raise ValueError("new K/V and the caches must be FP16, BF16 or FP8-E4M3, all of one type")
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("block_tables and seq_lens must be int32")
    if new_keys.dim() != 4 or new_values.shape != new_keys.shape:
        raise ValueError("new_keys / new_values must be [batch, q_len, Hkv, 128]")
    if key_cache.dim() != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("key_cache / value_cache must be 4-D and of one shape")
    layout = _layout_code(kv_layout)
    batch, q_len, hkv, dim = new_keys.shape
    cache_page, cache_heads = (key_cache.shape[2], key_cache.shape[1]) if layout else key_cache.shape[1:3]
    if dim != HEAD_DIM or key_cache.shape[3] != HEAD_DIM:
        raise ValueError("the kernel supports head_dim 128")
    if cache_page != PAGE_SIZE:
        raise ValueError("page_size must be 16")
    if cache_heads != hkv:
        raise ValueError("new K/V and the caches disagree on the number of KV heads")
    if q_len < 1:
        raise ValueError("q_len must be at least 1")
    if block_tables.dim() != 2 or block_tables.shape[0] != batch or seq_lens.numel() != batch:
        raise ValueError("invalid metadata: block_tables must be [batch, max_pages], seq_lens [batch]")
    if key_cache.shape[0] == 0 or block_tables.shape[1] == 0:
        raise ValueError("empty KV cache is not supported")
    if batch == 0:
        return key_cache, value_cache

    device = key_cache.device
    status = _status_word(device)
    a = _native.SqaAppendArgs()
    a.new_keys, a.new_values = new_keys.data_ptr(), new_values.data_ptr()
    a.key_cache, a.value_cache = key_cache.data_ptr(), value_cache.data_ptr()
    a.block_tables, a.seq_lens = block_tables.data_ptr(), seq_lens.data_ptr()
    a.status = status.data_ptr()
    a.batch, a.q_len, a.num_kv_heads = batch, q_len, hkv
    a.head_dim, a.page_size = HEAD_DIM, PAGE_SIZE
    a.num_pages, a.max_pages = int(key_cache.shape[0]), int(block_tables.shape[1])
    a.kv_layout = layout
    a.page_stride = _cache_page_stride(key_cache, value_cache)
    a.kv_dtype = _native.KV_FP8_E4M3 if key_cache.element_size() == 1 else _native.KV_SAME
    with _on_device(device):
        code = _native.library().sqa_cache_append(ctypes.byref(a), ctypes.c_void_p(_stream_handle(device)))
        _native.check(code, "sqa_cache_append")
        if check:
            _raise_device_bits(read_device_status(status.data_ptr(), clear=True, device=device))
    return key_cache, value_cache
