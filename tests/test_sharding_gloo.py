"""Multi-rank partitioning on CPU ranks (gloo, world size 2).

The three single-box modes — batch sharding, KV-head sharding and the
long-context page split with an (O, LSE) all-gather — are exercised with the
product's planning functions and collective helper
(``small_q_attention_b200.sharding``); each rank computes its shard with the
CPU oracle, and the reassembled result must equal the unsharded oracle.  The
GPU kernels' shard form and merge are covered in ``tests/test_gpu_parity.py``.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from small_q_attention_b200.sharding import (
    gather_partials,
    kv_head_range,
    lpt_batch_shards,
    page_split,
    shard_lengths,
    shard_sequence_pages,
)

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed, batch, q_len, lens, hkv=2):
    rng = np.random.default_rng(seed)
    pages = [(n + 15) // 16 for n in lens]
    pool = sum(pages) + 3
    ids = rng.permutation(pool).astype(np.int32)
    table = np.zeros((batch, max(pages)), np.int32)
    cur = 0
    for b, n in enumerate(pages):
        table[b, :n] = ids[cur:cur + n]
        cur += n
    q = rng.standard_normal((batch, q_len, 4 * hkv, 128)).astype(np.float16)
    kc = rng.standard_normal((pool, 16, hkv, 128)).astype(np.float16)
    vc = rng.standard_normal((pool, 16, hkv, 128)).astype(np.float16)
    return q, kc, vc, table, np.array(lens, np.int32)


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)


def _long_context_rank(rank, port, result):
    from oracle import merge_partials, paged_mtp_attention_partial, paged_mtp_attention_reference

    _init(rank, port)
    try:
        q, kc, vc, table, lens = _case(3, 2, 16, [1000, 37])
        rows, held, mlen = [], [], []
        for b in range(len(lens)):
            ids, h, m = shard_sequence_pages(table[b], int(lens[b]), WORLD, rank)
            rows.append(ids)
            held.append(h)
            mlen.append(m)
        width = max(1, max(len(r) for r in rows))
        shard_table = np.zeros((len(lens), width), np.int32)
        for b, r in enumerate(rows):
            shard_table[b, :len(r)] = r
        o, lse = paged_mtp_attention_partial(q, kc, vc, shard_table, np.array(held), np.array(mlen), 16, 2)
        parts_o, parts_lse = gather_partials(torch.from_numpy(o), torch.from_numpy(lse))
        merged, _ = merge_partials(parts_o.numpy(), parts_lse.numpy())
        whole = paged_mtp_attention_reference(q, kc, vc, table, lens, 16, 2)
        result[rank] = float(np.abs(merged - whole).max())
    finally:
        dist.destroy_process_group()


def _batch_rank(rank, port, result):
    from oracle import paged_mtp_attention_reference

    _init(rank, port)
    try:
        lens = [4000, 33, 700, 1600, 16, 2500]
        q, kc, vc, table, lens_np = _case(4, len(lens), 4, lens)
        mine = lpt_batch_shards(lens, WORLD)[rank]
        out = paged_mtp_attention_reference(q[mine], kc, vc, table[mine], lens_np[mine], 16, 2)
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (mine, out))
        full = np.zeros(q.shape, np.float32)
        for idx, o in gathered:
            full[idx] = o
        whole = paged_mtp_attention_reference(q, kc, vc, table, lens_np, 16, 2)
        result[rank] = float(np.abs(full - whole).max())
    finally:
        dist.destroy_process_group()


def _heads_rank(rank, port, result):
    from oracle import paged_mtp_attention_reference

    _init(rank, port)
    try:
        hkv = 4
        q, kc, vc, table, lens = _case(5, 3, 8, [300, 1200, 8], hkv=hkv)
        lo, hi = kv_head_range(hkv, WORLD, rank)
        out = paged_mtp_attention_reference(q[:, :, 4 * lo:4 * hi], kc[:, :, lo:hi], vc[:, :, lo:hi], table,
                                            lens, 16, hi - lo)
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (lo, hi, out))
        full = np.zeros(q.shape, np.float32)
        for a, b, o in gathered:
            full[:, :, 4 * a:4 * b] = o
        whole = paged_mtp_attention_reference(q, kc, vc, table, lens, 16, hkv)
        result[rank] = float(np.abs(full - whole).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fn", [_long_context_rank, _batch_rank, _heads_rank],
                         ids=["long_context", "batch", "kv_heads"])
def test_two_gloo_ranks(fn):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        mp.start_processes(fn, args=(_free_port(), result), nprocs=WORLD, start_method="spawn")
        assert sorted(result.keys()) == list(range(WORLD))
        for r in range(WORLD):
            assert result[r] < 1e-4, (r, result[r])


def test_lpt_balances_and_covers():
    rng = np.random.default_rng(0)
    lens = [int(x) for x in rng.integers(512, 32768, 64)]
    for world in (1, 2, 4, 8):
        shards = lpt_batch_shards(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))
        loads = [sum(lens[i] for i in s) for s in shards]
        # LPT bound: max load <= optimal + largest item <= mean + max
        assert max(loads) <= sum(lens) / world + max(lens)


def test_head_and_page_partitions():
    for world in (1, 2, 4, 8):
        heads = [kv_head_range(8, world, r) for r in range(world)]
        assert heads[0][0] == 0 and heads[-1][1] == 8
        assert all(heads[i][1] == heads[i + 1][0] for i in range(world - 1))
        for n in (1, 7, 16384):
            ranges = [page_split(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1
    with pytest.raises(ValueError):
        kv_head_range(8, 3, 0)


def test_shard_lengths():
    # 100 tokens = 7 pages; shard of pages [4, 7) holds tokens 64..99
    assert shard_lengths(100, 4, 7) == (36, 36)
    assert shard_lengths(100, 0, 4) == (64, 100)
    assert shard_lengths(100, 7, 7) == (0, -12)
