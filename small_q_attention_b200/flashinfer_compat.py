"""FlashInfer-compatible entry point for speculative-decoding (MTP) attention.

``trtllm_batch_decode_with_kv_cache`` mirrors the signature of FlashInfer's
``flashinfer.decode.trtllm_batch_decode_with_kv_cache`` (FlashInfer 0.6) —
the paged decode call that takes ``q_len_per_req`` draft tokens per request —
and runs it on this library's kernels, so a serving stack that calls FlashInfer
for MTP decode can switch by changing one import.  The formats are the same as
this path's: a ``[batch, max_pages]`` int32 page table, per-request KV lengths
that include the ``q_len_per_req`` new tokens, and a paged cache in ``HND``
(``[pages, Hkv, page_size, 128]``, FlashInfer's default) or ``NHD``
(``[pages, page_size, Hkv, 128]``, the upstream's) layout, given either as a
``(k_cache, v_cache)`` tuple or as one ``[pages, 2, ...]`` tensor (both are read
in place through the page stride).  ``bmm1_scale`` is the full softmax scale on
q.k (FlashInfer folds ``1/sqrt(head_dim)`` into it) and ``bmm2_scale`` scales
the output.

Supported subset (anything else raises ``ValueError``): uniform
``q_len_per_req`` in 1..16, page size 16, head dim 128, GQA group 4, fp16 or
bf16 query and output, a cache of the query's type or fp8-e4m3 (its
dequantisation scales folded into ``bmm1_scale`` / ``bmm2_scale``, as FlashInfer
does), float scales, ``window_left=-1``, no sinks, no custom mask, no variable
query lengths, no nvfp4 scale-factor tensors, one shared page table for K and V.  ``backend`` and ``enable_pdl`` are
accepted and ignored (the kernels always use programmatic dependent launch).
"""

from __future__ import annotations

import torch

from .attention import small_q_attention

__all__ = ["trtllm_batch_decode_with_kv_cache"]


def _unsupported(what: str):
    raise ValueError(f"trtllm_batch_decode_with_kv_cache: {what} is not supported by small_q_attention_b200")


def trtllm_batch_decode_with_kv_cache(
    query,
    kv_cache,
    workspace_buffer,
    block_tables,
    seq_lens,
    max_seq_len: int,
    bmm1_scale=1.0,
    bmm2_scale=1.0,
    window_left: int = -1,
    out=None,
    out_dtype=None,
    o_sf_scale=None,
    o_sf_vec_size=None,
    sinks=None,
    kv_layout: str = "HND",
    enable_pdl=None,
    backend: str = "auto",
    q_len_per_req: int | None = 1,
    o_scale: float | None = 1.0,
    mask=None,
    max_q_len=None,
    cum_seq_lens_q=None,
    skip_softmax_threshold_scale_factor=None,
    kv_cache_sf=None,
    uses_shared_paged_kv_idx: bool = True,
):
    """Paged MTP decode attention with FlashInfer's argument conventions.

    ``query`` is ``[batch * q_len_per_req, num_heads, 128]``; returns the same shape.
    """
    if not isinstance(bmm1_scale, (int, float)) or not isinstance(bmm2_scale, (int, float)):
        _unsupported("a tensor bmm1_scale / bmm2_scale (pass floats)")
    if window_left != -1:
        _unsupported("a sliding window")
    if sinks is not None:
        _unsupported("attention sinks")
    if mask is not None:
        _unsupported("a custom mask (the causal draft-token rule is built in)")
    if max_q_len is not None or cum_seq_lens_q is not None:
        _unsupported("variable query lengths")
    if o_sf_scale is not None or o_sf_vec_size is not None or kv_cache_sf is not None:
        _unsupported("fp4 / scale-factor tensors")
    if o_scale not in (None, 1.0):
        _unsupported("o_scale (fp8 output)")
    if not uses_shared_paged_kv_idx:
        _unsupported("separate K and V page tables")
    if backend not in ("auto", "trtllm-gen", "xqa"):
        raise ValueError(f"unknown backend {backend!r}")
    if kv_layout not in ("HND", "NHD"):
        raise ValueError(f"unknown kv_layout {kv_layout!r}")
    q_len = int(q_len_per_req or 1)
    if query.dim() != 3 or query.shape[0] % q_len:
        raise ValueError("query must be [batch * q_len_per_req, num_heads, head_dim]")
    if out_dtype is not None and out_dtype != query.dtype:
        _unsupported("an output type other than the query's")

    if isinstance(kv_cache, (tuple, list)):
        if len(kv_cache) != 2:
            raise ValueError("kv_cache must be a (k_cache, v_cache) tuple or one [pages, 2, ...] tensor")
        k_cache, v_cache = kv_cache
    else:
        if kv_cache.dim() != 5 or kv_cache.shape[1] != 2:
            _unsupported("a kv_cache tensor that is not [pages, 2, ...]")
        k_cache, v_cache = kv_cache[:, 0], kv_cache[:, 1]

    if seq_lens.dtype == torch.uint32:
        seq_lens = seq_lens.view(torch.int32)  # lengths < 2^31: same bits
    batch = query.shape[0] // q_len
    q4 = query.view(batch, q_len, query.shape[1], query.shape[2])
    if out is not None:
        if out.shape != query.shape or out.dtype != query.dtype:
            raise ValueError("out must be shaped and typed like query")
        out4 = out.view(batch, q_len, out.shape[1], out.shape[2])
    else:
        out4 = None
    ws = workspace_buffer if workspace_buffer is not None and workspace_buffer.dtype == torch.uint8 else None
    res = small_q_attention(q4, k_cache, v_cache, block_tables, seq_lens, 16, max_seq_len, out=out4, workspace=ws,
                            kv_layout=kv_layout, sm_scale=float(bmm1_scale), out_scale=float(bmm2_scale))
    return res.view(query.shape)
