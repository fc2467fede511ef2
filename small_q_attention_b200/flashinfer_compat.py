"""FlashInfer-compatible entry points for speculative-decoding (MTP) attention.

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

``BatchDecodeWithPagedKVCacheWrapper`` mirrors FlashInfer's decode wrapper
(``flashinfer.decode.BatchDecodeWithPagedKVCacheWrapper``, 0.6 / 0.7) as the
upstream drives it for MTP (``scripts/compare_flashinfer_paths.py:104-121``,
``docs/pr3859_comment_draft.md:19-23``): ``plan(indptr, indices, last_page_len,
..., q_len_per_req=q)`` once per batch, then ``run(q, paged_kv_cache)`` per
step.  The CSR page layout (``indptr`` [batch + 1], ``indices`` the pages of
every request back to back, ``last_page_len`` [batch] in 1..page_size) is
turned into this path's padded page table and lengths once, in ``plan``; the
draft rows follow the same causal rule (row ``qi`` of a request sees the
tokens before ``kv_len - q_len + qi + 1``).  Same supported subset as above;
``pos_encoding_mode`` must be "NONE", no logits soft cap, no rope scaling, no
``return_lse``.
"""

from __future__ import annotations

import torch

from .attention import small_q_attention

__all__ = ["trtllm_batch_decode_with_kv_cache", "BatchDecodeWithPagedKVCacheWrapper", "csr_to_block_table"]


def _unsupported(what: str):
    raise ValueError(f"{what} is not supported by small_q_attention_b200's FlashInfer-compatible entry points")


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


def csr_to_block_table(indptr, indices, last_page_len, page_size: int = 16):
    """FlashInfer's CSR page layout -> ``(block_tables [batch, max_pages] int32,
    seq_lens [batch] int32)`` on the indices' device.  A request with ``n > 0``
    pages holds ``(n - 1) * page_size + last_page_len`` tokens; one with none, 0.
    Table entries past a request's pages are 0 (never read: the kernels stop at
    the length)."""
    indptr = indptr.to(device=indices.device, dtype=torch.int64)
    last = last_page_len.to(device=indices.device, dtype=torch.int64)
    counts = indptr[1:] - indptr[:-1]
    if (counts < 0).any():
        raise ValueError("indptr must be non-decreasing")
    batch = counts.numel()
    max_pages = max(int(counts.max()) if batch else 0, 1)
    j = torch.arange(max_pages, device=indices.device, dtype=torch.int64)
    valid = j[None, :] < counts[:, None]
    idx = (indptr[:-1, None] + j[None, :]).clamp(max=max(indices.numel() - 1, 0))
    table = torch.where(valid, indices.to(torch.int64)[idx] if indices.numel() else torch.zeros_like(idx),
                        torch.zeros_like(idx))
    lens = torch.where(counts > 0, (counts - 1) * page_size + last, torch.zeros_like(counts))
    if ((counts > 0) & ((last < 1) | (last > page_size))).any():
        raise ValueError("last_page_len must be in [1, page_size] for a request with pages")
    return table.to(torch.int32).contiguous(), lens.to(torch.int32).contiguous()


class BatchDecodeWithPagedKVCacheWrapper:
    """FlashInfer's paged decode wrapper, for MTP decode on this library's kernels.

    >>> w = BatchDecodeWithPagedKVCacheWrapper(workspace, "NHD", use_tensor_cores=True)
    >>> w.plan(indptr, indices, last_page_len, 32, 8, 128, 16, q_data_type=torch.float16,
    ...        q_len_per_req=4)
    >>> out = w.run(q, kv_cache)        # q [batch * 4, 32, 128]; kv_cache [pages, 2, 16, 8, 128]
    """

    def __init__(self, float_workspace_buffer, kv_layout: str = "NHD", use_cuda_graph: bool = False,
                 use_tensor_cores: bool = False, paged_kv_indptr_buffer=None, paged_kv_indices_buffer=None,
                 paged_kv_last_page_len_buffer=None, backend: str = "auto", jit_args=None):
        if kv_layout not in ("NHD", "HND"):
            raise ValueError(f"unknown kv_layout {kv_layout!r}")
        if jit_args is not None:
            _unsupported("jit_args")
        ws = float_workspace_buffer
        self._workspace = ws.view(torch.uint8) if ws is not None and ws.is_contiguous() else None
        self._kv_layout = kv_layout
        self._plan = None

    def plan(self, indptr, indices, last_page_len, num_qo_heads: int, num_kv_heads: int, head_dim: int,
             page_size: int, pos_encoding_mode: str = "NONE", window_left: int = -1, logits_soft_cap=None,
             q_data_type="float16", kv_data_type=None, data_type=None, sm_scale=None, rope_scale=None,
             rope_theta=None, non_blocking: bool = True, block_tables=None, seq_lens=None,
             fixed_split_size=None, disable_split_kv: bool = False, q_len_per_req: int = 1, **unused):
        """Fix the batch: page layout, heads, types, scale and draft tokens per request."""
        if pos_encoding_mode != "NONE":
            _unsupported(f"pos_encoding_mode={pos_encoding_mode!r}")
        if window_left != -1:
            _unsupported("a sliding window")
        if logits_soft_cap not in (None, 0, 0.0):
            _unsupported("a logits soft cap")
        if rope_scale is not None or rope_theta is not None:
            _unsupported("rope")
        if head_dim != 128 or page_size != 16 or num_qo_heads != 4 * num_kv_heads:
            _unsupported(f"head_dim {head_dim}, page_size {page_size}, heads {num_qo_heads}/{num_kv_heads}")
        q_len = int(q_len_per_req or 1)
        if not 1 <= q_len <= 16:
            _unsupported(f"q_len_per_req={q_len}")
        q_dt = getattr(torch, q_data_type) if isinstance(q_data_type, str) else q_data_type
        if data_type is not None:  # older name of the query/KV type
            q_dt = getattr(torch, data_type) if isinstance(data_type, str) else data_type
        kv_dt = kv_data_type if kv_data_type is not None else q_dt
        kv_dt = getattr(torch, kv_dt) if isinstance(kv_dt, str) else kv_dt
        if q_dt not in (torch.float16, torch.bfloat16):
            _unsupported(f"query type {q_dt}")
        if kv_dt not in (q_dt, getattr(torch, "float8_e4m3fn", None)):
            _unsupported(f"KV type {kv_dt}")
        if block_tables is not None and seq_lens is not None:
            table, lens = block_tables.to(torch.int32).contiguous(), seq_lens.to(torch.int32).contiguous()
        else:
            table, lens = csr_to_block_table(indptr, indices, last_page_len, page_size)
        # both length bounds, read once here as FlashInfer's plan reads its host-side layout:
        # they steer the launch (cluster mode or the segment-aligned split for near-uniform
        # batches of few requests), never the result
        self._plan = dict(table=table, lens=lens, q_len=q_len, hq=num_qo_heads, hkv=num_kv_heads,
                          q_dtype=q_dt, kv_dtype=kv_dt, max_seq_len=int(lens.max()) if lens.numel() else 0,
                          min_seq_len=int(lens.min()) if lens.numel() else 0,
                          sm_scale=float(sm_scale) if sm_scale is not None else 128 ** -0.5)

    begin_forward = plan

    def run(self, q, paged_kv_cache, *args, q_scale=None, k_scale=None, v_scale=None, out=None, lse=None,
            return_lse: bool = False, window_left=None, enable_pdl=None):
        """Attention of ``q`` ``[batch * q_len_per_req, num_qo_heads, 128]`` over the planned pages;
        ``paged_kv_cache`` is ``(k_cache, v_cache)`` or one ``[pages, 2, ...]`` tensor."""
        p = self._plan
        if p is None:
            raise RuntimeError("plan() has not been called")
        if return_lse or lse is not None:
            _unsupported("return_lse")
        if window_left not in (None, -1):
            _unsupported("a sliding window")
        if q.dim() != 3 or q.shape[0] != p["table"].shape[0] * p["q_len"] or q.shape[1] != p["hq"]:
            raise ValueError("q must be [batch * q_len_per_req, num_qo_heads, head_dim] as planned")
        if q.dtype != p["q_dtype"]:
            raise ValueError(f"q is {q.dtype}, planned {p['q_dtype']}")
        if isinstance(paged_kv_cache, (tuple, list)):
            k_cache, v_cache = paged_kv_cache
        else:
            if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2:
                _unsupported("a paged_kv_cache tensor that is not [pages, 2, ...]")
            k_cache, v_cache = paged_kv_cache[:, 0], paged_kv_cache[:, 1]
        scale = p["sm_scale"] * (float(q_scale) if q_scale is not None else 1.0) * (
            float(k_scale) if k_scale is not None else 1.0)
        out_scale = float(v_scale) if v_scale is not None else 1.0
        batch = p["table"].shape[0]
        q4 = q.view(batch, p["q_len"], q.shape[1], q.shape[2])
        out4 = None
        if out is not None:
            if out.shape != q.shape or out.dtype != q.dtype:
                raise ValueError("out must be shaped and typed like q")
            out4 = out.view(q4.shape)
        res = small_q_attention(q4, k_cache, v_cache, p["table"], p["lens"], 16, p["max_seq_len"], out=out4,
                                workspace=self._workspace, kv_layout=self._kv_layout, sm_scale=scale,
                                out_scale=out_scale, min_seq_len=p["min_seq_len"])
        return res.view(q.shape)

    forward = run
