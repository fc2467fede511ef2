"""Generate the golden vectors under ``tests/golden/`` from the upstream reference.

Run once in a container that has the upstream repository checked out (its
``src/`` directory must contain the ``small_q_attention`` package)::

    python tests/golden/make_golden.py --reference-src <upstream>/src

Each case draws seeded fp16 inputs, runs the upstream
``paged_mtp_attention_reference`` (``src/small_q_attention/reference.py:10-74``)
on float32 upcasts of them -- exactly as the upstream parity scripts do
(``scripts/run_gpu_matrix.py:162-165``) -- and writes inputs plus the float32
output to ``<case>.npz``.  The GPU box never runs this script; the tests read
only the ``.npz`` files.

The first three cases are the upstream unit-test fixtures
(``tests/test_reference.py:9-45``, ``tests/test_reference_edges.py:17-38``) in
their general (non-kernel) shapes; they pin the CPU oracle.  The remaining
cases use the kernel contract (head_dim 128, page 16, GQA group 4) with 2 or 8
KV heads and exercise: a length that is not a multiple of 16, ``seq_len ==
q_len``, a one-page sequence, ragged batches, a reversed page table, random
pages from an oversized pool, q_len 1 and 16, and K scaled by 4 on a random
subset of tokens.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _contract_case(torch, seed, batch, q_len, lens, num_kv_heads, pool_factor=2.0,
                   table="random", k_scale_frac=0.0):
    page_size, head_dim, group = 16, 128, 4
    g = torch.Generator().manual_seed(seed)
    pages = [(n + page_size - 1) // page_size for n in lens]
    max_pages = max(pages)
    needed = sum(pages)
    pool = max(needed, int(np.ceil(needed * pool_factor)))
    query = torch.randn(batch, q_len, num_kv_heads * group, head_dim, generator=g).half()
    key_cache = torch.randn(pool, page_size, num_kv_heads, head_dim, generator=g)
    value_cache = torch.randn(pool, page_size, num_kv_heads, head_dim, generator=g).half()
    if k_scale_frac > 0:
        hit = torch.rand(pool, page_size, generator=g) < k_scale_frac
        key_cache[hit] *= 4.0
    key_cache = key_cache.half()
    if table == "reversed":
        ids = torch.arange(pool - 1, -1, -1, dtype=torch.int32)
    else:
        ids = torch.randperm(pool, generator=g).to(torch.int32)
    block_tables = torch.full((batch, max_pages), -1, dtype=torch.int32)
    cursor = 0
    for b, n in enumerate(pages):
        block_tables[b, :n] = ids[cursor:cursor + n]
        cursor += n
    # slots past a sequence's last page hold a poison id the kernel must never read
    block_tables[block_tables < 0] = 0x7FFFFFFF
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    return dict(query=query, key_cache=key_cache, value_cache=value_cache,
                block_tables=block_tables, seq_lens=seq_lens, page_size=page_size,
                num_kv_heads=num_kv_heads)


def _cases(torch):
    cases = {}
    # tests/test_reference.py:9-33 (manual single-head recompute, page_size 2)
    torch.manual_seed(0)
    cases["upstream_manual_single_head"] = dict(
        query=torch.randn(1, 2, 2, 4), key_cache=torch.randn(2, 2, 1, 4),
        value_cache=torch.randn(2, 2, 1, 4),
        block_tables=torch.tensor([[0, 1]], dtype=torch.int32),
        seq_lens=torch.tensor([4], dtype=torch.int32), page_size=2, num_kv_heads=1)
    # tests/test_reference.py:35-45 (GQA grouping, page_size 4)
    torch.manual_seed(1)
    cases["upstream_gqa_grouping"] = dict(
        query=torch.randn(1, 2, 4, 8), key_cache=torch.randn(2, 4, 2, 8),
        value_cache=torch.randn(2, 4, 2, 8),
        block_tables=torch.tensor([[0, 1]], dtype=torch.int32),
        seq_lens=torch.tensor([5], dtype=torch.int32), page_size=4, num_kv_heads=2)
    # tests/test_reference_edges.py:17-38 (physical page order [2, 0, 1]); seeded here
    torch.manual_seed(2)
    cases["upstream_physical_order"] = dict(
        query=torch.randn(1, 2, 2, 4), key_cache=torch.randn(3, 2, 1, 4),
        value_cache=torch.randn(3, 2, 1, 4),
        block_tables=torch.tensor([[2, 0, 1]], dtype=torch.int32),
        seq_lens=torch.tensor([5], dtype=torch.int32), page_size=2, num_kv_heads=1)

    cases["q2_len33_b2_random"] = _contract_case(torch, 11, 2, 2, [33, 33], 2)
    cases["q4_ragged_b3"] = _contract_case(torch, 12, 3, 4, [4, 16, 45], 2)
    cases["q8_len100_reversed"] = _contract_case(torch, 13, 1, 8, [100], 2, 1.0, "reversed")
    cases["q16_kscaled_b2"] = _contract_case(torch, 14, 2, 16, [16, 40], 2, 1.5, k_scale_frac=0.05)
    cases["q1_decode_b2"] = _contract_case(torch, 15, 2, 1, [1, 17], 2)
    cases["q2_hkv8_len24"] = _contract_case(torch, 16, 1, 2, [24], 8)
    cases["q4_hkv8_b2_ragged"] = _contract_case(torch, 17, 2, 4, [64, 31], 8)
    return cases


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", required=True,
                        help="the upstream repository's src/ directory")
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    import torch
    from small_q_attention import paged_mtp_attention_reference  # the upstream oracle

    for name, c in _cases(torch).items():
        expected = paged_mtp_attention_reference(
            c["query"].float(), c["key_cache"].float(), c["value_cache"].float(),
            c["block_tables"], c["seq_lens"], c["page_size"], c["num_kv_heads"])
        np.savez_compressed(
            HERE / f"{name}.npz",
            query=c["query"].numpy(), key_cache=c["key_cache"].numpy(),
            value_cache=c["value_cache"].numpy(),
            block_tables=c["block_tables"].numpy(), seq_lens=c["seq_lens"].numpy(),
            page_size=np.int32(c["page_size"]), num_kv_heads=np.int32(c["num_kv_heads"]),
            expected=expected.float().numpy())
        print(f"{name}: q{tuple(c['query'].shape)} cache{tuple(c['key_cache'].shape)} "
              f"lens={c['seq_lens'].tolist()}")


if __name__ == "__main__":
    main()
