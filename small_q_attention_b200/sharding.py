"""Single-box partitioning of the operator over 1/2/4/8 GPUs (one process per GPU).

The upstream has no distributed code at all (no NCCL, MPI or P2P call site);
these are the three ways its operator shards:

* batch sharding — sequences are independent: rank r runs the operator on its own
  sequences; no collective on the hot path.  :func:`lpt_batch_shards` balances
  ranks by total tokens (longest-processing-time greedy), since cost is linear in
  the tokens streamed.
* KV-head sharding — KV heads are independent: rank r owns KV heads
  ``[lo, hi)`` (its cache holds only those heads) and query heads
  ``[4 lo, 4 hi)``; no collective on the hot path.  :func:`kv_head_range`.
* long-context split — one sequence's pages are cut into contiguous ranges, one
  per rank (each rank holds its range in its own HBM); every rank computes the
  shard form of the operator (normalised O and LSE over the tokens it holds,
  with the causal rule in whole-sequence coordinates), the partials are
  all-gathered over NCCL and merged with the log-sum-exp merge kernel.
  :func:`page_split`, :func:`shard_lengths`, :func:`long_context_attention`.

Every collective here goes through ``torch.distributed`` (NCCL on GPUs, gloo in
the CPU tests); every bulk load in the kernels reads this GPU's own memory.
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

PAGE = 16


def lpt_batch_shards(lens, world: int) -> list[list[int]]:
    """Assign sequence indices to ``world`` ranks, balancing total tokens.

    Longest first, each to the currently least-loaded rank (ties: lowest rank);
    each rank's list is returned in increasing index order.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    return [sorted(s) for s in shards]


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous KV heads of ``rank``; ``num_kv_heads`` must divide evenly."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def page_split(num_pages: int, world: int, rank: int) -> tuple[int, int]:
    """Near-equal contiguous page range ``[lo, hi)`` of ``rank`` (may be empty)."""
    base, extra = divmod(num_pages, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_lengths(total_len: int, page_lo: int, page_hi: int, page_size: int = PAGE) -> tuple[int, int]:
    """Tokens a shard holding pages ``[page_lo, page_hi)`` of a ``total_len``
    sequence holds, and its mask length (``total_len`` minus the shard offset):
    draft row ``qi`` sees shard token ``t`` iff ``t < held`` and
    ``t < mask_len - q_len + qi + 1`` — the upstream causal rule
    (``src/small_q_attention/reference.py:63``) in shard coordinates."""
    held = max(0, min(total_len, page_hi * page_size) - page_lo * page_size)
    return held, total_len - page_lo * page_size


def gather_partials(o: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather per-rank partials: returns ``([world, *o.shape], [world, *lse.shape])``.
    Without an initialised process group there is one rank."""
    if not dist.is_initialized():
        return o[None], lse[None]
    world = dist.get_world_size(group)
    # flat buffers: NCCL and gloo both gather 1-D tensors into a 1-D output
    parts_o = torch.empty(world * o.numel(), dtype=o.dtype, device=o.device)
    parts_lse = torch.empty(world * lse.numel(), dtype=lse.dtype, device=lse.device)
    dist.all_gather_into_tensor(parts_o, o.contiguous().view(-1), group=group)
    dist.all_gather_into_tensor(parts_lse, lse.contiguous().view(-1), group=group)
    return parts_o.view(world, *o.shape), parts_lse.view(world, *lse.shape)


def long_context_attention(query, key_cache, value_cache, block_tables, held_lens, mask_lens,
                           page_size: int = PAGE, group=None, *, out=None, workspace=None):
    """Attention over sequences whose pages are split across the ranks of ``group``.

    Each rank passes the full ``query`` and its own shard: ``key_cache`` /
    ``value_cache`` pool on this GPU, ``block_tables`` of the pages it holds,
    ``held_lens`` (tokens held per sequence) and ``mask_lens`` (whole length
    minus this shard's token offset), as given by :func:`shard_lengths`.
    Returns the merged fp16 output on every rank.
    """
    from .attention import merge_partials, small_q_attention_partial

    o, lse = small_q_attention_partial(query, key_cache, value_cache, block_tables, held_lens, page_size,
                                       mask_lens=mask_lens, workspace=workspace)
    parts_o, parts_lse = gather_partials(o, lse, group)
    return merge_partials(parts_o, parts_lse, out=out)


def shard_sequence_pages(block_tables_row, total_len: int, world: int, rank: int, page_size: int = PAGE):
    """Page ids, held length and mask length of ``rank``'s part of one sequence."""
    n_pages = (total_len + page_size - 1) // page_size
    lo, hi = page_split(n_pages, world, rank)
    held, mask_len = shard_lengths(total_len, lo, hi, page_size)
    return block_tables_row[lo:hi], held, mask_len
