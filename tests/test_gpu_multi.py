"""Sharded operator on 2 GPUs: long-context split, batch and KV-head shards.

Each rank holds the same seeded pool (generated on the host) and runs its
shard through the C ABI; the reassembled output must match the single-GPU
operator and the oracle.  The long-context split is checked with both
exchanges: the NCCL all-gather and the library's NVLink peer-store exchange
(three steps in a row, then a captured CUDA graph replayed twice, then a step
that rank 1 skips, which rank 0's bounded wait must report as a timeout).
NVLS is off (NCCL_NVLS_ENABLE=0); the exchange uses plain peer stores.
Skipped on hosts with fewer than 2 GPUs.
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, result):
    import datetime

    import torch.distributed as dist

    from oracle import paged_mtp_attention_reference
    from small_q_attention_b200 import small_q_attention, small_q_attention_partial
    from small_q_attention_b200.sharding import (kv_head_range, long_context_attention, lpt_batch_shards,
                                                 shard_sequence_pages)
    from small_q_attention_b200.workloads import make_case

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    dev = torch.device("cuda", rank)
    errs = {}
    try:
        # long-context: two sequences, pages split over the ranks
        c = make_case(2, 16, [5000, 700], hkv=8, pool_factor=1.0, seed=41, device=dev, gen_device="cpu")
        rows, held, mlen = [], [], []
        for b, n in enumerate(c["lens"]):
            ids, h, m = shard_sequence_pages(c["block_tables"][b], n, WORLD, rank)
            rows.append(ids)
            held.append(h)
            mlen.append(m)
        width = max(1, max(len(r) for r in rows))
        table = torch.zeros(2, width, dtype=torch.int32, device=dev)
        for b, r in enumerate(rows):
            table[b, :len(r)] = r
        out = long_context_attention(c["query"], c["key_cache"], c["value_cache"], table,
                                     torch.tensor(held, dtype=torch.int32, device=dev),
                                     torch.tensor(mlen, dtype=torch.int32, device=dev))
        whole = small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                                  16, check=True)
        ref = paged_mtp_attention_reference(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                            c["seq_lens"], 16, 8)
        errs["long_vs_whole"] = float((out.float() - whole.float()).abs().max())
        errs["long_vs_oracle"] = float(np.abs(out.float().cpu().numpy() - ref).max())

        # the same split through the NVLink exchange: the merged output lands on rank 0
        from small_q_attention_b200.sharding import LongContextGroup

        held_t = torch.tensor(held, dtype=torch.int32, device=dev)
        mlen_t = torch.tensor(mlen, dtype=torch.int32, device=dev)
        grp = LongContextGroup(rows=2 * 16 * 32)
        for _ in range(3):
            p2p = long_context_attention(c["query"], c["key_cache"], c["value_cache"], table, held_t, mlen_t,
                                         exchange=grp)
        torch.cuda.synchronize()
        if rank == 0:
            errs["p2p_vs_whole"] = float((p2p.float() - whole.float()).abs().max())
        else:
            errs["p2p_vs_whole"] = 0.0 if p2p is None else 1.0
        o, lse = small_q_attention_partial(c["query"], c["key_cache"], c["value_cache"], table, held_t, 16,
                                           mask_lens=mlen_t)
        gout = torch.empty(c["query"].shape, dtype=torch.float16, device=dev)
        s_ = torch.cuda.Stream(dev)
        s_.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s_):
            grp.exchange(o, lse, out=gout)
        for _ in range(2):
            gout.zero_()
            g.replay()
        torch.cuda.synchronize()
        del g
        if rank == 0:
            errs["graph_vs_whole"] = float((gout.float() - whole.float()).abs().max())
        errs["p2p_status"] = grp.device_status()
        dist.barrier()
        if rank == 0:  # rank 1 skips this step: the bounded wait gives up and says so
            grp.exchange(o, lse, out=gout)
            errs["skip_status"] = grp.device_status()
        dist.barrier()
        grp.close()

        # batch shards (LPT), gathered for checking only
        lens = [3000, 40, 900, 5000, 17]
        c = make_case(5, 4, lens, hkv=8, pool_factor=1.2, seed=42, device=dev, gen_device="cpu")
        mine = lpt_batch_shards(lens, WORLD)[rank]
        idx = torch.tensor(mine, device=dev)
        part = small_q_attention(c["query"][idx].contiguous(), c["key_cache"], c["value_cache"],
                                 c["block_tables"][idx].contiguous(), c["seq_lens"][idx].contiguous(), 16, check=True)
        got = [None] * WORLD
        dist.all_gather_object(got, (mine, part.cpu()))
        full = torch.zeros_like(c["query"], device="cpu")
        for m_, p_ in got:
            full[m_] = p_
        ref = paged_mtp_attention_reference(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                            c["seq_lens"], 16, 8)
        errs["batch_vs_oracle"] = float(np.abs(full.float().numpy() - ref).max())

        # KV-head shards: each rank keeps its heads' cache only
        c = make_case(3, 8, [1500, 64, 4000], hkv=8, pool_factor=1.0, seed=43, device=dev, gen_device="cpu")
        lo, hi = kv_head_range(8, WORLD, rank)
        part = small_q_attention(c["query"][:, :, 4 * lo:4 * hi].contiguous(),
                                 c["key_cache"][:, :, lo:hi].contiguous(), c["value_cache"][:, :, lo:hi].contiguous(),
                                 c["block_tables"], c["seq_lens"], 16, check=True)
        got = [None] * WORLD
        dist.all_gather_object(got, (lo, hi, part.cpu()))
        full = torch.zeros_like(c["query"], device="cpu")
        for a, b, p_ in got:
            full[:, :, 4 * a:4 * b] = p_
        ref = paged_mtp_attention_reference(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                            c["seq_lens"], 16, 8)
        errs["heads_vs_oracle"] = float(np.abs(full.float().numpy() - ref).max())
        result[rank] = errs
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharding():
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        mp.start_processes(_rank, args=(_free_port(), result), nprocs=WORLD, start_method="spawn")
        for r in range(WORLD):
            errs = result[r]
            assert errs["long_vs_whole"] < 2e-3, errs
            assert errs["p2p_vs_whole"] < 2e-3 and errs["p2p_status"] == 0, errs
            if r == 0:
                assert errs["graph_vs_whole"] < 2e-3, errs
                assert errs["skip_status"] & 1, errs  # SQA_DEV_TIMEOUT
            for k in ("long_vs_oracle", "batch_vs_oracle", "heads_vs_oracle"):
                assert errs[k] < 2e-2, (k, errs)
