"""Seeded synthetic workloads: the five named configurations and the 36-case matrix.

The upstream measured no public dataset; all of its inputs are synthetic
(``scripts/run_gpu_matrix.py:34-60``).  The shapes here follow the benchmark
contract (``configs/core_matrix.json``: fp16, head_dim 128, page 16, 32 query /
8 KV heads) and the five named configurations:

* ``cfg1``  B=1,  q=2,  kv=1024,   pool 2x the needed pages, random permutation
* ``cfg2``  B=4,  q=4,  kv=8192,   pool 1.5x
* ``cfg3``  B=16, q=8,  kv=32768,  pool 1x
* ``cfg4``  B=64, q=4,  kv ~ U[512, 32768] rounded up to 16, K x4 on 1% of tokens, pool 1.25x
* ``cfg5``  B=1,  q=16, kv=262144, pool 1x

Page tables give each sequence distinct pages drawn from a seeded permutation
of the pool ("random"), or the upstream's reversed-contiguous layouts
("unique": request r owns pages [r*n, (r+1)*n) in reverse order; "shared":
every request uses the same reversed pages, ``run_gpu_matrix.py:42-48``).
"""

from __future__ import annotations

import itertools
import math

import torch

HQ, HKV, HEAD_DIM, PAGE = 32, 8, 128, 16

CONFIGS = {
    "cfg1": dict(batch=1, q_len=2, kv_len=1024, pool_factor=2.0),
    "cfg2": dict(batch=4, q_len=4, kv_len=8192, pool_factor=1.5),
    "cfg3": dict(batch=16, q_len=8, kv_len=32768, pool_factor=1.0),
    "cfg4": dict(batch=64, q_len=4, kv_len=(512, 32768), pool_factor=1.25, k_outlier_frac=0.01),
    "cfg5": dict(batch=1, q_len=16, kv_len=262144, pool_factor=1.0),
}

MATRIX_Q = (2, 4, 8, 16)
MATRIX_KV = (1024, 8192, 32768)
MATRIX_B = (1, 4, 16)


def matrix_cases():
    """The 36 (q_len, kv_len, batch) cells of ``configs/core_matrix.json``."""
    return [dict(q_len=q, kv_len=kv, batch=b) for q, kv, b in itertools.product(MATRIX_Q, MATRIX_KV, MATRIX_B)]


def config_lens(name: str, seed: int = 0) -> list[int]:
    c = CONFIGS[name]
    if isinstance(c["kv_len"], tuple):
        lo, hi = c["kv_len"]
        g = torch.Generator().manual_seed(4000 + seed)
        raw = torch.randint(lo, hi + 1, (c["batch"],), generator=g)
        return [int(math.ceil(int(x) / PAGE) * PAGE) for x in raw]
    return [c["kv_len"]] * c["batch"]


def algorithmic_bytes(batch: int, q_len: int, lens, hq: int = HQ, hkv: int = HKV, kv_bytes: int = 2) -> int:
    """Bytes the operator must move at least once: K and V of every visible
    token of every KV head (``kv_bytes`` per element: 2 for fp16/bf16, 1 for
    fp8), Q in, O out (2 bytes each), the used page-table entries and the
    lengths."""
    kv = sum(int(n) for n in lens) * hkv * HEAD_DIM * 2 * kv_bytes
    qo = 2 * batch * q_len * hq * HEAD_DIM * 2
    table = sum((int(n) + PAGE - 1) // PAGE for n in lens) * 4
    return kv + qo + table + 4 * batch


def make_case(batch: int, q_len: int, lens, *, hkv: int = HKV, pool_factor: float = 1.0,
              page_mode: str = "random", seed: int = 0, device="cuda", k_outlier_frac: float = 0.0,
              gen_device=None, max_pages: int | None = None, dtype=torch.float16):
    """Seeded fp16 Q/K/V caches, int32 page table and lengths on ``device``.

    ``gen_device`` is where the random numbers are drawn ("cpu" for
    bit-reproducible small cases; the target device for multi-GB ones).
    """
    lens = [int(n) for n in lens]
    device = torch.device(device)
    gen_device = torch.device(gen_device) if gen_device is not None else device
    pages = [(n + PAGE - 1) // PAGE for n in lens]
    needed = sum(pages)
    width = max(max(pages), 1) if max_pages is None else max_pages
    if page_mode == "shared":
        pool = max(pages)
    else:
        pool = max(needed, int(math.ceil(needed * pool_factor)), 1)
    g = torch.Generator(device=gen_device).manual_seed(seed)
    hq = 4 * hkv
    query = torch.randn(batch, q_len, hq, HEAD_DIM, generator=g, device=gen_device, dtype=torch.float16).to(dtype)
    key_cache = torch.randn(pool, PAGE, hkv, HEAD_DIM, generator=g, device=gen_device, dtype=torch.float16).to(dtype)
    value_cache = torch.randn(pool, PAGE, hkv, HEAD_DIM, generator=g, device=gen_device,
                              dtype=torch.float16).to(dtype)
    if k_outlier_frac > 0:
        hit = torch.rand(pool, PAGE, generator=g, device=gen_device) < k_outlier_frac
        key_cache[hit] *= 4
    table = torch.full((batch, width), 0, dtype=torch.int32)
    if page_mode == "random":
        perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32)
        cursor = 0
        for b, n in enumerate(pages):
            table[b, :n] = perm[cursor:cursor + n]
            cursor += n
    elif page_mode == "unique":
        cursor = 0
        for b, n in enumerate(pages):
            table[b, :n] = torch.arange(cursor + n - 1, cursor - 1, -1, dtype=torch.int32)
            cursor += n
    elif page_mode == "shared":
        for b, n in enumerate(pages):
            table[b, :n] = torch.arange(n - 1, -1, -1, dtype=torch.int32)
    else:
        raise ValueError(f"unknown page_mode {page_mode}")
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    return dict(
        query=query.to(device), key_cache=key_cache.to(device), value_cache=value_cache.to(device),
        block_tables=table.to(device), seq_lens=seq_lens.to(device), page_size=PAGE,
        num_kv_heads=hkv, lens=lens)


def make_config(name: str, *, seed: int = 0, device="cuda", gen_device=None, hkv: int = HKV):
    c = CONFIGS[name]
    lens = config_lens(name, seed)
    return make_case(c["batch"], c["q_len"], lens, hkv=hkv, pool_factor=c["pool_factor"], seed=seed,
                     device=device, gen_device=gen_device, k_outlier_frac=c.get("k_outlier_frac", 0.0))
