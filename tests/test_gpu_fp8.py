"""FP8-E4M3 K/V caches with FP16 queries (tcgen05 kernel): parity with the oracle on
the same fp8 values, the dequantisation scales folded into sm_scale / out_scale, HND
and interleaved pools, splits, append, and the contract errors.

The tensor core reads the fp8 K/V values unchanged (kind::f8f6f4); the fp16
queries and the probabilities enter as sums of two e4m3 parts (about 8
significant bits).  The FP16 tolerance applies (``|err| <= 2e-2 + 1e-2 |ref|``,
max-abs 2e-2) against the oracle fed the same fp8 values in float32; measured
worst cases use 0.3 of it.
"""

import math

import numpy as np
import pytest
import torch

from oracle import cache_append_reference, paged_mtp_attention_reference
from tests.test_gpu_parity import assert_close, case

pytestmark = pytest.mark.gpu
F8 = getattr(torch, "float8_e4m3fn", None)


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available() or F8 is None:
        pytest.skip("needs a CUDA device and torch.float8_e4m3fn")
    import small_q_attention_b200 as m

    return m


def case_fp8(q_len, lens, *, hkv=8, seed=0, k_outlier_frac=0.0):
    c = case(q_len, lens, hkv=hkv, seed=seed, k_outlier_frac=k_outlier_frac)
    return dict(c, key_cache=c["key_cache"].to(F8), value_cache=c["value_cache"].to(F8))


def oracle(c, k_scale=1.0, v_scale=1.0):
    ref = paged_mtp_attention_reference(c["query"], c["key_cache"].float() * k_scale,
                                        c["value_cache"].float() * v_scale, c["block_tables"], c["seq_lens"], 16,
                                        c["num_kv_heads"])
    return ref


CASES = [(1, [1, 17, 500], 4), (2, [33, 1024], 8), (4, [4, 16, 17, 1000], 8), (4, [8192] * 4, 8),
         (8, [2048, 8, 9, 300], 2), (12, [12, 200, 777], 2), (16, [16, 31, 4096], 8)]


@pytest.mark.parametrize("q_len,lens,hkv", CASES, ids=[f"q{q}-n{len(l)}-kv{max(l)}" for q, l, _ in CASES])
def test_fp8_parity(sqa, q_len, lens, hkv):
    c = case_fp8(q_len, lens, hkv=hkv, seed=q_len * 17 + len(lens))
    out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                check=True)
    assert out.dtype == torch.float16
    assert_close(out, oracle(c))


def test_fp8_splits_outliers_and_scales(sqa):
    c = case_fp8(8, [40, 700, 16, 1500, 8], hkv=2, seed=7, k_outlier_frac=0.05)
    k_scale, v_scale = 0.25, 3.0  # dequantised K = fp8 * 0.25, V = fp8 * 3
    ref = oracle(c, k_scale, v_scale)
    for n in (3, 64, 296):
        out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                                    16, num_ctas=n, min_pages_per_cta=1, sm_scale=k_scale / math.sqrt(128),
                                    out_scale=v_scale, check=True)
        assert_close(out, ref)


@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_fp8_layouts_and_pools(sqa, layout):
    c = case_fp8(4, [100, 2000, 5000], seed=12)
    k, v = c["key_cache"], c["value_cache"]
    if layout == "HND":
        k, v = k.permute(0, 2, 1, 3).contiguous(), v.permute(0, 2, 1, 3).contiguous()
    pool = torch.stack([k.view(torch.uint8), v.view(torch.uint8)], dim=1).contiguous().view(F8)
    out = sqa.small_q_attention(c["query"], pool[:, 0], pool[:, 1], c["block_tables"], c["seq_lens"], 16,
                                kv_layout=layout, check=True)
    assert_close(out, oracle(c))


def test_fp8_nan_tail_slots_are_masked(sqa):
    c = case_fp8(12, [37, 50, 16], hkv=2, seed=5)
    ref = oracle(c)
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    table = c["block_tables"].cpu()
    for b, n in enumerate(c["lens"]):
        if n % 16:
            last = int(table[b, (n - 1) // 16])
            kc.view(torch.uint8)[last, n % 16:] = 0x7F  # e4m3 NaN
            vc.view(torch.uint8)[last, n % 16:] = 0x7F
    out = sqa.small_q_attention(c["query"], kc, vc, c["block_tables"], c["seq_lens"], 16, check=True)
    assert_close(out, ref)


def test_fp8_append_bit_exact(sqa):
    c = case_fp8(4, [40, 513, 2048], seed=5)
    gen = torch.Generator().manual_seed(6)
    nk = torch.randn(3, 4, 8, 128, generator=gen).to(F8)
    nv = torch.randn(3, 4, 8, 128, generator=gen).to(F8)
    u8 = lambda t: t.cpu().view(torch.uint8).numpy()  # noqa: E731
    ek, ev = cache_append_reference(u8(nk), u8(nv), u8(c["key_cache"]), u8(c["value_cache"]),
                                    c["block_tables"].cpu().numpy(), c["seq_lens"].cpu().numpy())
    sqa.cache_append(nk.cuda(), nv.cuda(), c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                     check=True)
    assert np.array_equal(u8(c["key_cache"]), ek) and np.array_equal(u8(c["value_cache"]), ev)


def test_fp8_contract(sqa):
    c = case_fp8(2, [64, 80], seed=1)
    args = (c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)
    with pytest.raises(ValueError):  # the warp-level kernel has no fp8 path
        sqa.small_q_attention(c["query"], *args, kernel=1)
    with pytest.raises(ValueError):  # fp32 queries are not a path type
        sqa.small_q_attention(c["query"].float(), *args)
    assert sqa.selected_kernel(c["query"], *args) == 2


@pytest.mark.parametrize("q_len,lens,hkv", [(2, [33, 1024], 8), (8, [2048, 8, 9, 300], 2), (16, [16, 31, 4096], 8)])
def test_fp8_bf16_queries(sqa, q_len, lens, hkv):
    """BF16 queries (and output) with FP8 K/V: a BF16 model with an FP8 cache."""
    c = case_fp8(q_len, lens, hkv=hkv, seed=q_len * 31 + len(lens))
    q = c["query"].to(torch.bfloat16)
    out = sqa.small_q_attention(q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                check=True)
    assert out.dtype == torch.bfloat16
    assert_close(out, oracle(dict(c, query=q.float())))


def test_fp8_flashinfer_entry(sqa):
    """The FlashInfer-compatible entry with an fp8 cache ([pages, 2, Hkv, 16, 128]) and BF16 queries, the
    dequantisation scales folded into bmm1_scale / bmm2_scale."""
    from small_q_attention_b200.flashinfer_compat import trtllm_batch_decode_with_kv_cache

    q_len = 4
    c = case_fp8(q_len, [100, 2000, 8192], seed=13)
    hnd = lambda t: t.view(torch.uint8).permute(0, 2, 1, 3).contiguous()  # noqa: E731
    kv = torch.stack([hnd(c["key_cache"]), hnd(c["value_cache"])], dim=1).contiguous().view(F8)
    b = c["query"].shape[0]
    query = c["query"].to(torch.bfloat16).reshape(b * q_len, 32, 128)
    ws = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
    k_scale, v_scale = 0.5, 2.0
    out = trtllm_batch_decode_with_kv_cache(query, kv, ws, c["block_tables"], c["seq_lens"], max(c["lens"]),
                                            bmm1_scale=k_scale / math.sqrt(128), bmm2_scale=v_scale,
                                            kv_layout="HND", q_len_per_req=q_len)
    assert out.dtype == torch.bfloat16 and out.shape == query.shape
    ref = oracle(dict(c, query=c["query"].to(torch.bfloat16).float()), k_scale, v_scale)
    assert_close(out.view(c["query"].shape), ref)


@pytest.mark.parametrize("q_len", [4, 16])
@pytest.mark.parametrize("num_ctas", [5, 17, 64])
def test_fp8_block_shapes(sqa, q_len, num_ctas):
    """Both fp8 block shapes: 8-page blocks when a CTA's range is long (few CTAs here),
    4-page blocks otherwise; partial blocks and piece boundaries in both."""
    c = case_fp8(q_len, [3000, 5000, 700, 37], hkv=8, seed=q_len + num_ctas)
    out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                num_ctas=num_ctas, min_pages_per_cta=1, check=True)
    assert_close(out, oracle(c))
