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
  with the causal rule in whole-sequence coordinates) and the partials are
  merged.  :class:`LongContextGroup` does the exchange in the library's own
  kernels: each rank stores its partial into rank 0's memory with peer stores
  over NVLink and sets a flag, rank 0 waits for the flags (bounded) and merges
  (result on rank 0).  :func:`long_context_attention` without a group
  all-gathers the partials over ``torch.distributed`` and merges on every rank
  (any backend; the CPU tests use gloo).  :func:`page_split`,
  :func:`shard_lengths`.

Set-up collectives (handle exchange, barriers) go through ``torch.distributed``;
every bulk load in the kernels reads this GPU's own memory, and the exchange
uses plain peer stores (no multicast).
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


class LongContextGroup:
    """The exchange step of the long-context split, over NVLink peer memory.

    Collective construction (every rank of the process group, each with its own
    GPU current): each rank allocates its exchange block (``sqa_lc_create``), the
    IPC handles are all-gathered over ``torch.distributed`` and every rank maps
    the others' blocks (``sqa_lc_connect``).  ``rows`` is ``batch * q_len * Hq``
    of the merged output.  Then :meth:`exchange` once per step on every rank, in
    the same order: rank r's fp32 (O, LSE) goes into its slot on rank 0 with peer
    stores, rank 0 merges into ``out`` (fp16 or bf16).  No allocation, no host
    synchronisation and no collective library on the step; capturable in a CUDA
    graph.  Waits are bounded (about a second): a rank that stops shows up as
    ``SQA_DEV_TIMEOUT`` in :meth:`device_status`.  :meth:`close` (collective)
    unmaps and frees.
    """

    def __init__(self, rows: int, group=None, device=None):
        import ctypes

        from . import _native

        self._lib = _native.library()
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rows = int(rows)
        self._group = group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        n = int(self._lib.sqa_lc_handle_bytes())
        handle = (ctypes.c_uint8 * n)()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            code = self._lib.sqa_lc_create(self.rank, self.world, self.rows, ctypes.byref(ptr), handle)
            _native.check(code, "sqa_lc_create")
            self._ptr = ptr
            handles = [bytes(handle)]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
            joined = (ctypes.c_uint8 * (n * self.world)).from_buffer_copy(b"".join(handles))
            _native.check(self._lib.sqa_lc_connect(self._ptr, joined), "sqa_lc_connect")
            if self.world > 1:
                dist.barrier(group=group)  # every block is mapped before the first exchange

    def exchange(self, o: torch.Tensor, lse: torch.Tensor, out: torch.Tensor | None = None):
        """Send this rank's partial; on rank 0 return the merged output (``out`` or a
        new fp16 tensor shaped like ``o``), on the other ranks None."""
        import ctypes

        from . import _native
        from .attention import _stream_handle

        if o.dtype != torch.float32 or lse.dtype != torch.float32 or not (o.is_contiguous() and lse.is_contiguous()):
            raise ValueError("o and lse must be contiguous fp32 tensors")
        if o.numel() != self.rows * 128 or lse.numel() != self.rows or o.device != self.device:
            raise ValueError(f"o must hold {self.rows} rows of 128 and lse {self.rows} entries on {self.device}")
        if self.rank == 0:
            if out is None:
                out = torch.empty(o.shape, dtype=torch.float16, device=o.device)
            if out.dtype not in (torch.float16, torch.bfloat16) or out.numel() != o.numel() or not out.is_contiguous():
                raise ValueError("out must be a contiguous fp16 or bf16 tensor shaped like o")
        code = self._lib.sqa_lc_exchange(self._ptr, ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(lse.data_ptr()),
                                         ctypes.c_void_p(out.data_ptr() if self.rank == 0 else None),
                                         int(self.rank == 0 and out.dtype == torch.bfloat16),
                                         ctypes.c_void_p(_stream_handle(self.device)))
        _native.check(code, "sqa_lc_exchange")
        return out if self.rank == 0 else None

    def device_status(self, clear: bool = True) -> int:
        """Synchronise and return the SQA_DEV_* bits of this rank's exchange block."""
        import ctypes

        from .attention import _stream_handle

        bits = ctypes.c_uint32(0)
        self._lib.sqa_lc_read_status(self._ptr, ctypes.byref(bits), int(clear),
                                     ctypes.c_void_p(_stream_handle(self.device)))
        return int(bits.value)

    def close(self):
        """Collective: unmap and free once no rank has an exchange in flight."""
        from . import _native

        if self._ptr is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self._group)  # no rank has an exchange in flight
        _native.check(self._lib.sqa_lc_disconnect(self._ptr), "sqa_lc_disconnect")
        if self.world > 1:
            dist.barrier(group=self._group)  # no rank maps another's block any more
        _native.check(self._lib.sqa_lc_destroy(self._ptr), "sqa_lc_destroy")
        self._ptr = None


def long_context_attention(query, key_cache, value_cache, block_tables, held_lens, mask_lens,
                           page_size: int = PAGE, group=None, *, out=None, workspace=None,
                           exchange: LongContextGroup | None = None):
    """Attention over sequences whose pages are split across the ranks of ``group``.

    Each rank passes the full ``query`` and its own shard: ``key_cache`` /
    ``value_cache`` pool on this GPU, ``block_tables`` of the pages it holds,
    ``held_lens`` (tokens held per sequence) and ``mask_lens`` (whole length
    minus this shard's token offset), as given by :func:`shard_lengths`.
    With ``exchange`` (a :class:`LongContextGroup` of the same ranks) the merged
    fp16 output is returned on rank 0 and None elsewhere; without it the
    partials are all-gathered and the merged output is returned on every rank.
    """
    from .attention import merge_partials, small_q_attention_partial

    o, lse = small_q_attention_partial(query, key_cache, value_cache, block_tables, held_lens, page_size,
                                       mask_lens=mask_lens, workspace=workspace)
    if exchange is not None:
        return exchange.exchange(o, lse, out=out)
    parts_o, parts_lse = gather_partials(o, lse, group)
    return merge_partials(parts_o, parts_lse, out=out)


def shard_sequence_pages(block_tables_row, total_len: int, world: int, rank: int, page_size: int = PAGE):
    """Page ids, held length and mask length of ``rank``'s part of one sequence."""
    n_pages = (total_len + page_size - 1) // page_size
    lo, hi = page_split(n_pages, world, rank)
    held, mask_len = shard_lengths(total_len, lo, hi, page_size)
    return block_tables_row[lo:hi], held, mask_len
