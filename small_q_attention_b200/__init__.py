"""B200-native (sm_100a) small-q paged-KV attention for MTP / speculative decoding.

Public API:
  small_q_attention(query, key_cache, value_cache, block_tables, seq_lens, page_size, max_seq_len=0)
  small_q_attention_partial(...) -> (O, LSE)   shard form for a split sequence
  merge_partials(parts_o, parts_lse)           log-sum-exp merge of shards
  cache_append(new_k, new_v, k_cache, v_cache, block_tables, seq_lens)
                                               write the draft tokens' K/V into their pages
  PagedMTPAttention(device).plan(...).run(...)  planned, CUDA-graph-capturable step
  cuda.forward_v0 ... forward_v5               upstream-compatible entry points

All compute runs in the in-tree C-ABI library ``_lib/libsqa_b200.so``; there is
no CPU fallback.
"""

from .cache import cache_append  # noqa: F401
from .wrapper import PagedMTPAttention  # noqa: F401
from .attention import (  # noqa: F401
    merge_partials,
    read_device_status,
    selected_kernel,
    small_q_attention,
    small_q_attention_partial,
    workspace_bytes,
)

__all__ = [
    "small_q_attention",
    "small_q_attention_partial",
    "merge_partials",
    "workspace_bytes",
    "read_device_status",
    "selected_kernel",
    "cache_append",
    "PagedMTPAttention",
]
