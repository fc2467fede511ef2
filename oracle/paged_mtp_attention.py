"""CPU oracle for causal paged multi-token-prediction (MTP) attention.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against; it is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the CPU-baseline legs of ``bench.py``.  The
product package (``small_q_attention_b200``) never imports it and has no CPU
fallback.

It restates, in float32 numpy, the algorithm of the upstream reference
``paged_mtp_attention_reference`` (``src/small_q_attention/reference.py:10-74``
of zz774ever/small_q_attention):

* contract checks and their ``ValueError`` messages (``reference.py:34-44``,
  ``:52-53``);
* the page gather ``page_ids = block_tables[b, :ceil(len/page_size)]`` and the
  truncation of the gathered keys/values to ``len`` tokens (``reference.py:54-59``);
* the spec-dec causal rule ``valid_kv = total_len - q_len + qi + 1``
  (``reference.py:63``);
* GQA grouping ``kvh = qh // (Hq/Hkv)`` (``reference.py:67``);
* ``softmax((K[:valid] @ q) * head_dim**-0.5) @ V[:valid]`` in float32
  (``reference.py:68-70``).

All reference parity code feeds the reference float32 upcasts of the fp16 GPU
inputs and casts the result back to fp16 (``scripts/run_gpu_matrix.py:162-165``,
``scripts/build_and_test_v3.py:32-40``); with float32 inputs the reference's
``probs.to(query.dtype)`` (``reference.py:69``) is a no-op.  This oracle always
computes in float32 for the same reason.

Pinning: ``tests/golden/make_golden.py`` runs the upstream reference itself
(imported from the read-only reference tree) on seeded inputs and stores the
inputs and outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this oracle against every stored vector, and ``tests/test_oracle_known.py``
restates the reference's own unit tests (``tests/test_reference.py``,
``tests/test_reference_edges.py``, with the two broken fixtures fixed).

Vectorisation: the reference loops over (qi, qh) and does one mat-vec per pair.
Here the loop is over (b, kvh) and the ``group * q_len`` query rows of one KV
head are handled as one matrix, with the causal rule applied as a mask.  The
masked positions get probability exactly 0, so the result is the same softmax
up to float32 summation order.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "paged_mtp_attention_reference",
    "paged_mtp_attention_partial",
    "merge_partials",
]


def _as_f32(x) -> np.ndarray:
    """Return a float32 numpy view/copy of a numpy array or a CPU torch tensor."""
    if hasattr(x, "detach"):  # torch tensor: the tests may pass either kind
        x = x.detach().cpu().float().numpy()
    return np.asarray(x, dtype=np.float32)


def _as_array(x) -> np.ndarray:
    """numpy array in the tensor's own dtype (the caches are upcast per sequence,
    after the page gather, so a multi-GB fp16 pool is never converted whole)."""
    if hasattr(x, "detach"):
        x = x.detach().cpu()
        if str(x.dtype) == "torch.bfloat16":
            x = x.float()
        x = x.numpy()
    return np.asarray(x)


def _as_i64(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x).astype(np.int64)


def _check_contract(query, key_cache, value_cache, block_tables, seq_lens, page_size, num_kv_heads):
    """Shape checks, same order and messages as ``reference.py:34-44``."""
    if query.ndim != 4:
        raise ValueError("query must have shape [batch, q_len, heads, head_dim]")
    batch, q_len, num_query_heads, head_dim = query.shape
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if tuple(key_cache.shape[1:]) != (page_size, num_kv_heads, head_dim):
        raise ValueError("key_cache shape does not match page/head contract")
    if tuple(value_cache.shape) != tuple(key_cache.shape):
        raise ValueError("key_cache and value_cache must have the same shape")
    if block_tables.shape[0] != batch or seq_lens.size != batch:
        raise ValueError("batch metadata shape mismatch")
    return batch, q_len, num_query_heads, head_dim


def _gather_sequence(cache, table_row, total_len, page_size, num_kv_heads, head_dim):
    """``index_select`` of the sequence's pages, then truncation (``reference.py:54-59``)."""
    num_pages = (total_len + page_size - 1) // page_size
    page_ids = table_row[:num_pages]
    if num_pages and (page_ids.min() < 0 or page_ids.max() >= cache.shape[0]):
        # torch.index_select raises on an out-of-range index; so does the oracle.
        raise IndexError("block_tables holds a page id outside the cache")
    return cache[page_ids].reshape(-1, num_kv_heads, head_dim)[:total_len].astype(np.float32)


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    """Row softmax in float32; rows that are entirely -inf give all-zero probabilities."""
    row_max = scores.max(axis=-1, keepdims=True)
    row_max = np.where(np.isfinite(row_max), row_max, np.float32(0.0))
    e = np.exp(scores - row_max, dtype=np.float32)
    denom = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    safe = np.where(denom > 0, denom, np.float32(1.0))
    return (e / safe).astype(np.float32), denom, row_max


def paged_mtp_attention_reference(
    query,
    key_cache,
    value_cache,
    block_tables,
    seq_lens,
    page_size: int,
    num_kv_heads: int,
) -> np.ndarray:
    """Causal paged MTP attention, float32 result ``[batch, q_len, Hq, head_dim]``.

    Same signature and argument meaning as the upstream
    ``paged_mtp_attention_reference`` (``reference.py:10-31``): ``seq_lens[b]`` is
    the total KV length *including* the ``q_len`` draft tokens, and draft row
    ``qi`` attends to KV positions ``< seq_lens[b] - q_len + qi + 1``.
    """
    q = _as_f32(query)
    kc = _as_array(key_cache)
    vc = _as_array(value_cache)
    tables = _as_i64(block_tables)
    lens = _as_i64(seq_lens).reshape(-1)
    batch, q_len, num_query_heads, head_dim = _check_contract(
        q, kc, vc, tables, lens, page_size, num_kv_heads
    )

    scale = np.float32(head_dim ** -0.5)  # reference.py:46
    group = num_query_heads // num_kv_heads  # reference.py:47
    out = np.zeros((batch, q_len, num_query_heads, head_dim), dtype=np.float32)
    qi_of_row = np.repeat(np.arange(q_len), group)  # row r = qi * group + g
    for b in range(batch):
        total_len = int(lens[b])
        if total_len < q_len:  # reference.py:52-53
            raise ValueError("seq_lens must be at least q_len for MTP attention")
        keys = _gather_sequence(kc, tables[b], total_len, page_size, num_kv_heads, head_dim)
        values = _gather_sequence(vc, tables[b], total_len, page_size, num_kv_heads, head_dim)
        valid = total_len - q_len + qi_of_row + 1  # reference.py:63, one entry per row
        mask = np.arange(total_len)[None, :] >= valid[:, None]
        for kvh in range(num_kv_heads):
            # rows of this KV head: (qi, qh) for qh in [kvh*group, (kvh+1)*group)
            rows = q[b, :, kvh * group:(kvh + 1) * group, :].reshape(q_len * group, head_dim)
            scores = (rows @ keys[:, kvh, :].T) * scale  # reference.py:68
            scores = np.where(mask, np.float32(-np.inf), scores).astype(np.float32)
            probs, _, _ = _softmax_rows(scores)  # reference.py:69
            o = probs @ values[:, kvh, :]  # reference.py:70
            out[b, :, kvh * group:(kvh + 1) * group, :] = o.reshape(q_len, group, head_dim)
    return out


def paged_mtp_attention_partial(
    query,
    key_cache,
    value_cache,
    block_tables,
    seq_lens,
    mask_lens,
    page_size: int,
    num_kv_heads: int,
):
    """Attention over a slice of each sequence's keys; returns ``(O, LSE)``.

    This is the per-shard step of splitting one sequence's KV range across
    devices.  The shard holds ``seq_lens[b]`` tokens, which are tokens
    ``[offset, offset + seq_lens[b])`` of the whole sequence; ``mask_lens[b]``
    is the whole sequence's length minus ``offset``, so the spec-dec rule of
    ``reference.py:63`` reads ``t < mask_lens[b] - q_len + qi + 1`` in shard
    coordinates.  With ``mask_lens == seq_lens`` this is the full operator.

    Returns the normalised float32 output ``O`` ``[B, q_len, Hq, D]`` and the
    natural-log ``LSE`` ``[B, q_len, Hq]`` of the scaled scores; a row with no
    visible key gets ``O = 0`` and ``LSE = -inf``.
    """
    q = _as_f32(query)
    kc = _as_array(key_cache)
    vc = _as_array(value_cache)
    tables = _as_i64(block_tables)
    lens = _as_i64(seq_lens).reshape(-1)
    mlens = _as_i64(mask_lens).reshape(-1)
    batch, q_len, num_query_heads, head_dim = _check_contract(
        q, kc, vc, tables, lens, page_size, num_kv_heads
    )
    scale = np.float32(head_dim ** -0.5)
    group = num_query_heads // num_kv_heads
    out = np.zeros((batch, q_len, num_query_heads, head_dim), dtype=np.float32)
    lse = np.full((batch, q_len, num_query_heads), -np.inf, dtype=np.float32)
    qi_of_row = np.repeat(np.arange(q_len), group)
    for b in range(batch):
        n = int(lens[b])
        if n <= 0:
            continue
        keys = _gather_sequence(kc, tables[b], n, page_size, num_kv_heads, head_dim)
        values = _gather_sequence(vc, tables[b], n, page_size, num_kv_heads, head_dim)
        valid = np.minimum(int(mlens[b]) - q_len + qi_of_row + 1, n)
        mask = np.arange(n)[None, :] >= valid[:, None]
        for kvh in range(num_kv_heads):
            rows = q[b, :, kvh * group:(kvh + 1) * group, :].reshape(q_len * group, head_dim)
            scores = (rows @ keys[:, kvh, :].T) * scale
            scores = np.where(mask, np.float32(-np.inf), scores).astype(np.float32)
            probs, denom, row_max = _softmax_rows(scores)
            o = probs @ values[:, kvh, :]
            row_lse = np.where(denom[:, 0] > 0, row_max[:, 0] + np.log(np.maximum(denom[:, 0], 1e-38)), -np.inf)
            out[b, :, kvh * group:(kvh + 1) * group, :] = o.reshape(q_len, group, head_dim)
            lse[b, :, kvh * group:(kvh + 1) * group] = row_lse.reshape(q_len, group)
    return out, lse


def merge_partials(parts_o, parts_lse):
    """Log-sum-exp merge of partial attention results over their first axis.

    Restates the split-KV merge of the upstream kernel
    (``csrc/small_q_attention_ext.cu:339-366``): global max of the per-chunk
    statistics, rescale each chunk by ``exp(stat - max)``, sum, divide; a row
    whose total weight is 0 yields 0.  Here each part is already normalised,
    so its weight is ``exp(lse_i - LSE)`` with ``LSE = logsumexp(lse_i)``.
    Returns ``(O, LSE)``.
    """
    o = np.asarray(parts_o, dtype=np.float32)
    l = np.asarray(parts_lse, dtype=np.float32)
    gmax = l.max(axis=0)
    base = np.where(np.isfinite(gmax), gmax, np.float32(0.0))
    w = np.exp(l - base[None], dtype=np.float32)
    w = np.where(np.isfinite(l), w, np.float32(0.0))
    total = w.sum(axis=0)
    safe = np.where(total > 0, total, np.float32(1.0))
    merged = (o * (w / safe[None])[..., None]).sum(axis=0)
    merged = np.where((total > 0)[..., None], merged, np.float32(0.0)).astype(np.float32)
    merged_lse = np.where(total > 0, base + np.log(safe), -np.inf).astype(np.float32)
    return merged, merged_lse
