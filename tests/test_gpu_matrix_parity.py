"""Oracle parity on every benchmark case: the 36-cell matrix, the five named
configurations (cfg5 also with FP8-E4M3 caches), and the sharded forms of
cfg3 / cfg4 / cfg5 computed rank by rank on one GPU.

The upstream checks every matrix case against its CPU reference
(``scripts/run_gpu_matrix.py:159-169`` with ``src/small_q_attention/reference.py:10-74``);
so does this file, for both kernels and for the automatic choice.  Inputs are the
benchmark's own seeded workloads (``small_q_attention_b200.workloads``), drawn on
the GPU.  The whole batch is computed; the oracle checks a fixed sample of its
sequences (all of them up to batch 4; first, middle and last at batch 16; first,
last, longest and shortest of the ragged cfg4), each with its whole KV range, so
multi-GB cases stay within seconds of numpy.  cfg5 (one 262,144-token q16
sequence, split over every CTA of the GPU and merged) is checked whole.

Tolerance: ``|out - ref| <= 2e-2 + 1e-2 |ref|`` element-wise and max-abs 2e-2
(the operator contract), via ``tests.test_gpu_parity.assert_close``; the device
status word must stay clean (``check=True``).
"""

import math
import re

import pytest
import torch

from oracle import merge_partials as oracle_merge
from oracle import paged_mtp_attention_reference
from tests.test_gpu_parity import assert_close

pytestmark = pytest.mark.gpu
F8 = getattr(torch, "float8_e4m3fn", None)


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m
    from small_q_attention_b200 import _native

    _native.library()  # fail loudly if the native library is missing
    return m


def _cases():
    from small_q_attention_b200.workloads import CONFIGS, matrix_cases

    names = [f"q{c['q_len']}_kv{c['kv_len']}_b{c['batch']}" for c in matrix_cases()]
    return names + list(CONFIGS) + ["cfg5_fp8"]


CASES = _cases()
# kernel "h": the automatic choice given both length hints (min and max of seq_lens), as the
# benchmark passes them: cluster mode or the segment-aligned split where they apply
PARAMS = [(name, k) for name in CASES for k in ((0, 2, "h") if name.endswith("fp8") else (0, 1, 2, "h"))]


def _make(name):
    from small_q_attention_b200.workloads import make_case, make_config

    if name.startswith("cfg"):
        base = name.split("_")[0]
        c = make_config(base, seed=11, device="cuda")
        if name.endswith("fp8"):
            c = dict(c, key_cache=c["key_cache"].to(F8), value_cache=c["value_cache"].to(F8))
        return c
    q, kv, b = (int(x) for x in re.fullmatch(r"q(\d+)_kv(\d+)_b(\d+)", name).groups())
    seed = 1000 * q + b + kv // 1024
    return make_case(b, q, [kv] * b, pool_factor=1.0, seed=seed, device="cuda")


def _sample(lens):
    """Indices of the sequences the oracle checks."""
    n = len(lens)
    if n <= 4:
        return list(range(n))
    if n <= 16:
        return [0, n // 2, n - 1]
    longest = max(range(n), key=lambda i: (lens[i], -i))
    shortest = min(range(n), key=lambda i: (lens[i], i))
    return sorted({0, n - 1, longest, shortest})


def sub_case(c, idx):
    """The sequences ``idx`` of a case with only their pages, in a compact host pool
    (same values, same per-sequence page order): the oracle input for them."""
    lens = [int(c["lens"][b]) for b in idx]
    npg = [(n + 15) // 16 for n in lens]
    ids = torch.cat([c["block_tables"][b, :n].long() for b, n in zip(idx, npg)])

    def gather(cache):
        if cache.dtype == F8:  # e4m3 values are exact in fp16
            return cache.view(torch.uint8).index_select(0, ids).view(F8).to(torch.float16).cpu()
        return cache.index_select(0, ids).cpu()

    table = torch.zeros(len(idx), max(npg), dtype=torch.int32)
    cursor = 0
    for i, n in enumerate(npg):
        table[i, :n] = torch.arange(cursor, cursor + n, dtype=torch.int32)
        cursor += n
    return dict(query=c["query"][idx].cpu(), key_cache=gather(c["key_cache"]), value_cache=gather(c["value_cache"]),
                block_tables=table, seq_lens=torch.tensor(lens, dtype=torch.int32), num_kv_heads=c["num_kv_heads"],
                lens=lens)


def oracle_of(s):
    return paged_mtp_attention_reference(s["query"], s["key_cache"], s["value_cache"], s["block_tables"],
                                         s["seq_lens"], 16, s["num_kv_heads"])


_last = {}


def case_and_ref(name):
    """One case at a time is kept (inputs on the GPU, the oracle's answer on the host)."""
    if _last.get("name") != name:
        _last.clear()
        torch.cuda.empty_cache()
        c = _make(name)
        idx = _sample(c["lens"])
        _last.update(name=name, c=c, idx=idx, ref=oracle_of(sub_case(c, idx)))
    return _last["c"], _last["idx"], _last["ref"]


@pytest.mark.parametrize("name,kernel", PARAMS, ids=[f"{n}-k{k}" for n, k in PARAMS])
def test_matrix_case_vs_oracle(sqa, name, kernel):
    c, idx, ref = case_and_ref(name)
    hints = dict(kernel=0, min_seq_len=min(c["lens"])) if kernel == "h" else dict(kernel=kernel)
    out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                max(c["lens"]), check=True, **hints)
    assert out.dtype == torch.float16
    assert_close(out[idx], ref)


# ---------------------------------------------------------------- sharded configurations, one rank at a time
SHARDED = [(cfg, w) for cfg in ("cfg3", "cfg4", "cfg5") for w in (2, 4, 8)]


@pytest.mark.parametrize("cfg,world", SHARDED, ids=[f"{c}-x{w}" for c, w in SHARDED])
def test_sharded_config_vs_oracle(sqa, cfg, world):
    """What every rank of ``bench.py --gpus N --workload cfgX`` computes, run rank by
    rank on this GPU, then combined the way the ranks combine it (cfg3 / cfg4: each
    rank's output is its slice of the whole; cfg5: the (O, LSE) partials are merged).
    Each rank passes the bounds of its own lengths, as the bench does, so the launch
    shapes are the bench's (the segment-aligned split for cfg5's shards and for cfg3 at
    8 ranks)."""
    from small_q_attention_b200.sharding import kv_head_range, lpt_batch_shards, page_split, shard_lengths

    c, idx, ref = case_and_ref(cfg)
    kc, vc, q, bt, sl = c["key_cache"], c["value_cache"], c["query"], c["block_tables"], c["seq_lens"]
    if cfg == "cfg3":  # rank r owns KV heads [lo, hi) and query heads [4 lo, 4 hi)
        out = torch.empty_like(q)
        for r in range(world):
            lo, hi = kv_head_range(8, world, r)
            out[:, :, 4 * lo:4 * hi] = sqa.small_q_attention(
                q[:, :, 4 * lo:4 * hi].contiguous(), kc[:, :, lo:hi].contiguous(), vc[:, :, lo:hi].contiguous(),
                bt, sl, 16, max(c["lens"]), min_seq_len=min(c["lens"]), check=True)
        assert_close(out[idx], ref)
    elif cfg == "cfg4":  # rank r owns the sequences LPT gives it (same pool)
        out = torch.empty_like(q)
        for mine in lpt_batch_shards(c["lens"], world):
            sel = torch.tensor(mine, dtype=torch.long, device="cuda")
            my_lens = [c["lens"][i] for i in mine]
            out[sel] = sqa.small_q_attention(q[sel].contiguous(), kc, vc, bt[sel].contiguous(), sl[sel].contiguous(),
                                             16, max(my_lens), min_seq_len=min(my_lens), check=True)
        assert_close(out[idx], ref)
    else:  # cfg5: rank r holds pages [lo, hi) of the one sequence; partials merged
        total = c["lens"][0]
        parts_o, parts_lse = [], []
        for r in range(world):
            lo, hi = page_split(math.ceil(total / 16), world, r)
            held, mlen = shard_lengths(total, lo, hi)
            o, lse = sqa.small_q_attention_partial(
                q, kc, vc, bt[:, lo:hi].contiguous(), torch.tensor([held], dtype=torch.int32, device="cuda"), 16,
                mask_lens=torch.tensor([mlen], dtype=torch.int32, device="cuda"), max_seq_len=held, min_seq_len=held,
                check=True)
            parts_o.append(o)
            parts_lse.append(lse)
        merged = sqa.merge_partials(torch.stack(parts_o), torch.stack(parts_lse))
        assert_close(merged, ref)
        ro, _ = oracle_merge([p.cpu().numpy() for p in parts_o], [p.cpu().numpy() for p in parts_lse])
        assert_close(merged, ro)
