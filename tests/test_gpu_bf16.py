"""BF16 Q/K/V (the second KV dtype of the path): GPU parity with the oracle for both
kernels, BF16 cache append, BF16 shard + merge, and the upstream aliases still
FP16-only.

Tolerance: the FP16 bar (``|err| <= 2e-2 + 1e-2 |ref|`` element-wise) and a max-abs
bar of 2e-2 plus one BF16 rounding of the largest output (2^-8 relative), since the
output itself is rounded to BF16's 8-bit mantissa.
"""

import numpy as np
import pytest
import torch

from oracle import cache_append_reference, paged_mtp_attention_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m

    return m


def case_bf16(q_len, lens, *, hkv=8, seed=0, k_outlier_frac=0.0):
    from small_q_attention_b200.workloads import make_case

    return make_case(len(lens), q_len, lens, hkv=hkv, pool_factor=1.5, seed=seed, device="cuda", gen_device="cpu",
                     k_outlier_frac=k_outlier_frac, dtype=torch.bfloat16)


def oracle(c):
    return paged_mtp_attention_reference(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                         c["seq_lens"], 16, c["num_kv_heads"])


def assert_close_bf16(out, ref):
    out = out.float().cpu().numpy()
    assert out.shape == ref.shape and np.isfinite(out).all()
    err = np.abs(out - ref)
    bad = err > 2e-2 + 1e-2 * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance; max err {err.max():.3e}"
    assert err.max() <= 2e-2 + 2.0 ** -8 * np.abs(ref).max(), f"max abs err {err.max():.3e}"


CASES = [
    (1, [1, 2, 17, 500], 4),
    (2, [33, 1024], 8),
    (3, [3, 100, 257], 8),
    (4, [4, 16, 17, 1000], 8),
    (4, [8192] * 4, 8),
    (8, [2048, 8, 9, 300], 2),
    (12, [12, 200, 777], 2),
    (16, [16, 17, 31, 4096], 8),
]


@pytest.mark.parametrize("kernel", [1, 2])
@pytest.mark.parametrize("q_len,lens,hkv", CASES, ids=[f"q{q}-n{len(l)}-kv{max(l)}" for q, l, _ in CASES])
def test_bf16_parity(sqa, kernel, q_len, lens, hkv):
    c = case_bf16(q_len, lens, hkv=hkv, seed=q_len * 13 + len(lens))
    out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                kernel=kernel, check=True)
    assert out.dtype == torch.bfloat16
    assert_close_bf16(out, oracle(c))


@pytest.mark.parametrize("kernel", [1, 2])
def test_bf16_forced_splits_and_outliers(sqa, kernel):
    c = case_bf16(8, [40, 700, 16, 1500, 8], hkv=2, seed=7, k_outlier_frac=0.05)
    ref = oracle(c)
    for n in (3, 64, 296):
        out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                                    16, kernel=kernel, num_ctas=n, min_pages_per_cta=1, check=True)
        assert_close_bf16(out, ref)


def test_bf16_kernels_agree(sqa):
    c = case_bf16(4, [3000, 517, 9000], seed=11)
    args = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)
    a = sqa.small_q_attention(*args, kernel=1).float()
    b = sqa.small_q_attention(*args, kernel=2).float()
    assert (a - b).abs().max().item() <= 2 * 2.0 ** -8 * max(a.abs().max().item(), 1.0)


def test_bf16_shards_merge_to_whole(sqa):
    q_len, n = 16, 5000
    c = case_bf16(q_len, [n], seed=21)
    table = c["block_tables"]
    cut = 150  # pages [0, 150) and [150, 313) as two shards
    held = [cut * 16, n - cut * 16]
    parts_o, parts_lse = [], []
    for lo, hi, h in ((0, cut, held[0]), (cut, table.shape[1], held[1])):
        o, lse = sqa.small_q_attention_partial(c["query"], c["key_cache"], c["value_cache"],
                                               table[:, lo:hi].contiguous(),
                                               torch.tensor([h], dtype=torch.int32, device="cuda"), 16,
                                               mask_lens=torch.tensor([n - lo * 16], dtype=torch.int32, device="cuda"),
                                               check=True)
        parts_o.append(o)
        parts_lse.append(lse)
    merged = sqa.merge_partials(torch.stack(parts_o), torch.stack(parts_lse), out_dtype=torch.bfloat16)
    assert merged.dtype == torch.bfloat16
    assert_close_bf16(merged, oracle(c))


def test_bf16_cache_append_bit_exact(sqa):
    c = case_bf16(4, [40, 513, 2048], seed=5)
    gen = torch.Generator().manual_seed(6)
    nk = torch.randn(3, 4, 8, 128, generator=gen).to(torch.bfloat16)
    nv = torch.randn(3, 4, 8, 128, generator=gen).to(torch.bfloat16)
    as16 = lambda t: t.cpu().view(torch.int16).numpy()  # noqa: E731
    ek, ev = cache_append_reference(as16(nk), as16(nv), as16(c["key_cache"]), as16(c["value_cache"]),
                                    c["block_tables"].cpu().numpy(), c["seq_lens"].cpu().numpy())
    sqa.cache_append(nk.cuda(), nv.cuda(), c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                     check=True)
    assert np.array_equal(as16(c["key_cache"]), ek) and np.array_equal(as16(c["value_cache"]), ev)


def test_upstream_aliases_stay_fp16_only(sqa):
    from small_q_attention_b200 import cuda

    c = case_bf16(2, [64], seed=1)
    with pytest.raises(ValueError):
        cuda.forward_v3(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)
    with pytest.raises(ValueError):  # mixed types
        sqa.small_q_attention(c["query"].half(), c["key_cache"], c["value_cache"], c["block_tables"],
                              c["seq_lens"], 16)
