"""Drop-in replacements for the upstream ``small_q_attention.cuda`` wrappers.

The upstream module (``src/small_q_attention/cuda.py:16-336``) JIT-compiles one
extension per kernel revision (v0-v5) and exposes ``forward_v0`` ...
``forward_v5`` and ``load_v0`` ... ``load_v5``.  Here every revision maps to
the single B200 kernel: the arguments keep their names, positions and
validation (``ValueError`` for a non-positive ``chunk_keys`` or a
``token_group`` outside {2, 4}), and the results are the same operator.
``chunk_keys`` and ``token_group`` only tuned the upstream launch; the B200
split is sized from the SM count and the sequence lengths, so they do not
change the output.  q_len may be 1-16 (the upstream CUDA path accepted 2, 4,
8; ``cuda.py:206-207``).
"""

from __future__ import annotations

from . import _native
from .attention import small_q_attention


def _load(verbose: bool = False):
    lib = _native.library()
    if verbose:
        print(f"small_q_attention_b200: loaded {_native.LIB_PATH} (ABI {lib.sqa_abi_version()})")
    return lib


load_v0 = load_v1 = load_v2 = load_v3 = load_v4 = load_v5 = _load


def _check_chunk(chunk_keys):
    if int(chunk_keys) <= 0:
        raise ValueError("chunk_keys must be positive")


def _fp16_only(query, key_cache, value_cache):
    # the upstream wrappers accept FP16 only (cuda.py:197-211); small_q_attention also takes BF16
    import torch

    if any(isinstance(t, torch.Tensor) and t.dtype != torch.float16 for t in (query, key_cache, value_cache)):
        raise ValueError("the kernel requires FP16 Q/K/V")


def forward_v0(query, key_cache, value_cache, block_tables, seq_lens, page_size: int, verbose: bool = False):
    _load(verbose)
    _fp16_only(query, key_cache, value_cache)
    return small_q_attention(query, key_cache, value_cache, block_tables, seq_lens, page_size)


forward_v1 = forward_v0


def forward_v2(query, key_cache, value_cache, block_tables, seq_lens, page_size: int,
               chunk_keys: int = 512, verbose: bool = False):
    _check_chunk(chunk_keys)
    _load(verbose)
    _fp16_only(query, key_cache, value_cache)
    return small_q_attention(query, key_cache, value_cache, block_tables, seq_lens, page_size)


def forward_v3(query, key_cache, value_cache, block_tables, seq_lens, page_size: int,
               chunk_keys: int = 512, max_seq_len: int = 0, verbose: bool = False):
    _check_chunk(chunk_keys)
    _load(verbose)
    _fp16_only(query, key_cache, value_cache)
    return small_q_attention(query, key_cache, value_cache, block_tables, seq_lens, page_size,
                             max_seq_len=max_seq_len)


forward_v4 = forward_v3


def forward_v5(query, key_cache, value_cache, block_tables, seq_lens, page_size: int,
               chunk_keys: int = 512, token_group: int = 2, max_seq_len: int = 0, verbose: bool = False):
    if token_group not in (2, 4):
        raise ValueError("v5 token_group must be 2 or 4")
    return forward_v3(query, key_cache, value_cache, block_tables, seq_lens, page_size,
                      chunk_keys, max_seq_len, verbose)
