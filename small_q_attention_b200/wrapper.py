"""Plan once, run many: a persistent-workspace, CUDA-graph-capturable wrapper.

``small_q_attention`` already reuses a workspace per (device, stream), but it
looks the workspace up (and may grow it) on every call.  A serving loop wants
the FlashInfer-style split of the decode wrapper instead: ``plan`` once per
batch shape (allocates and zeroes the workspace, fixes the launch plan and the
kernel), then ``run`` every step with no allocation, no host synchronisation
and no shape-dependent host work beyond filling one argument struct, so that
``run`` can be captured in a CUDA graph and replayed.  ``run`` can also append
the step's new K/V to the cache first (``cache_append``), on the same stream.

The operator contract is that of ``small_q_attention`` (the upstream
``forward_v3``, ``src/small_q_attention/cuda.py:177-214``); this wrapper adds no
arithmetic of its own.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native
from .attention import (GQA_GROUP, HEAD_DIM, MAX_Q_LEN, PAGE_SIZE, _check_inputs, _fill_args, _layout_code,
                        _on_device, _raise_device_bits, _stream_handle, read_device_status)
from .cache import cache_append


class PagedMTPAttention:
    """Causal paged MTP attention with a planned launch.

    >>> attn = PagedMTPAttention(torch.device("cuda", 0))
    >>> attn.plan(batch=4, q_len=4, num_kv_heads=8, num_pages=3072, max_pages=512, max_seq_len=8192)
    >>> out = attn.run(q, k_cache, v_cache, block_tables, seq_lens, out=out)   # graph-capturable

    ``plan`` may be called again for another shape; it reallocates only when the
    new plan needs a larger workspace.
    """

    def __init__(self, device: torch.device | int | None = None, *, kernel: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is required for the small-q attention kernel")
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if kernel not in (0, 1, 2):
            raise ValueError("kernel must be 0 (auto), 1 (warp-level) or 2 (tcgen05)")
        self._kernel = kernel
        self._workspace: torch.Tensor | None = None
        self._shape = None
        self.selected_kernel = None

    # ------------------------------------------------------------------ plan
    def plan(self, batch: int, q_len: int, num_kv_heads: int, num_pages: int, max_pages: int,
             max_seq_len: int = 0, *, page_size: int = PAGE_SIZE, head_dim: int = HEAD_DIM,
             num_ctas: int = 0, min_pages_per_cta: int = 0, kv_layout: str = "NHD",
             sm_scale: float | None = None, out_scale: float = 1.0,
             cache_dtype: torch.dtype | None = None, min_seq_len: int = 0,
             cluster: int = 0) -> "PagedMTPAttention":
        """Fix the shapes of the following ``run`` calls and size the workspace.

        ``max_seq_len`` bounds ``seq_lens`` for the launch size (0: the page-table
        width); a ``run`` with longer sequences than planned is clamped to the
        table like ``small_q_attention``.  ``min_seq_len`` (a lower bound of the
        runs' ``seq_lens``, 0 = unknown) and ``cluster`` steer the launch as in
        ``small_q_attention``: with both bounds within 15% of each other, batches
        of few sequences run the tcgen05 kernel in thread-block clusters or with
        every segment split evenly over several CTAs (``selected_kernel`` reports
        ``2 + 100 * C`` or ``2 + 10000 * k``); a run whose lengths fall outside the
        bounds still gives the right result.
        """
        if not (1 <= q_len <= MAX_Q_LEN):
            raise ValueError(f"q_len must be in [1, {MAX_Q_LEN}]")
        if head_dim != HEAD_DIM or page_size != PAGE_SIZE:
            raise ValueError("the kernel supports head_dim 128 and page_size 16")
        if batch < 0 or num_kv_heads <= 0 or num_pages <= 0 or max_pages <= 0 or max_seq_len < 0:
            raise ValueError("invalid plan shape")
        if min_seq_len < 0 or cluster not in (0, 1, 2, 4, 8, 16):
            raise ValueError("min_seq_len must be >= 0 and cluster one of 0, 1, 2, 4, 8, 16")
        a = _native.SqaArgs()
        a.batch, a.q_len, a.num_q_heads, a.head_dim = batch, q_len, GQA_GROUP * num_kv_heads, head_dim
        a.num_kv_heads, a.page_size, a.num_pages, a.max_pages = num_kv_heads, page_size, num_pages, max_pages
        a.max_seq_len, a.num_ctas, a.min_pages_per_cta, a.kernel = max_seq_len, num_ctas, min_pages_per_cta, self._kernel
        a.kv_layout = _layout_code(kv_layout)
        a.min_seq_len, a.cluster = min_seq_len, cluster
        if cache_dtype is not None and cache_dtype == getattr(torch, "float8_e4m3fn", None):
            a.kv_dtype = _native.KV_FP8_E4M3  # fp8 caches run on the tcgen05 kernel
        lib = _native.library()
        st = ctypes.c_int(0)
        need = int(lib.sqa_workspace_bytes(ctypes.byref(a), self.device.index, ctypes.byref(st)))
        _native.check(st.value, "sqa_workspace_bytes")
        picked = lib.sqa_selected_kernel(ctypes.byref(a), self.device.index)
        if picked < 0:
            _native.check(-picked, "sqa_selected_kernel")
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.zeros(max(need, 1 << 16), dtype=torch.uint8, device=self.device)
        self._shape = (batch, q_len, num_kv_heads, num_pages, max_pages)
        self._max_seq_len, self._num_ctas, self._min_pages = max_seq_len, num_ctas, min_pages_per_cta
        self._kv_layout, self._sm_scale, self._out_scale = kv_layout, sm_scale, out_scale
        self._min_seq_len, self._cluster = min_seq_len, cluster
        self.selected_kernel = int(picked)
        return self

    @property
    def workspace(self) -> torch.Tensor:
        if self._workspace is None:
            raise RuntimeError("plan() has not been called")
        return self._workspace

    # ------------------------------------------------------------------ run
    def run(self, query, key_cache, value_cache, block_tables, seq_lens, *, out=None,
            append_keys=None, append_values=None, check: bool = False):
        """One step: optionally append ``append_keys/values`` ``[batch, q_len, Hkv, 128]``
        to the cache, then attend.  Returns ``out`` (allocated when not given; give
        it when capturing a CUDA graph)."""
        if self._shape is None:
            raise RuntimeError("plan() has not been called")
        _check_inputs(query, key_cache, value_cache, block_tables, seq_lens, PAGE_SIZE, kv_layout=self._kv_layout)
        hkv = key_cache.shape[1] if self._kv_layout == "HND" else key_cache.shape[2]
        shape = (int(query.shape[0]), int(query.shape[1]), int(hkv), int(key_cache.shape[0]),
                 int(block_tables.shape[1]))
        if shape != self._shape:
            raise ValueError(f"run() shapes {shape} differ from the planned {self._shape} "
                             "(batch, q_len, Hkv, num_pages, max_pages): plan() again")
        if query.device != self.device:
            raise ValueError("inputs are not on the planned device")
        if out is None:
            out = torch.empty_like(query)
        elif out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous() or out.device != query.device:
            raise ValueError("out must be a contiguous tensor shaped and typed like query")
        if (append_keys is None) != (append_values is None):
            raise ValueError("append_keys and append_values go together")
        if append_keys is not None:
            cache_append(append_keys, append_values, key_cache, value_cache, block_tables, seq_lens,
                         kv_layout=self._kv_layout)
        a = _fill_args(query, key_cache, value_cache, block_tables, seq_lens, None, self._max_seq_len,
                       self._num_ctas, self._min_pages, self._kernel, self._kv_layout, self._sm_scale,
                       self._out_scale)
        a.min_seq_len, a.cluster = self._min_seq_len, self._cluster
        a.out = out.data_ptr()
        ws = self._workspace
        with _on_device(self.device):
            code = _native.library().sqa_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()),
                                                ctypes.c_size_t(ws.numel()),
                                                ctypes.c_void_p(_stream_handle(self.device)))
            _native.check(code, "sqa_forward")
            if check:
                _raise_device_bits(read_device_status(ws.data_ptr(), clear=True, device=self.device))
        return out
