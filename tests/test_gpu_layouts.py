"""Cache layouts, page strides and scales on the GPU: HND caches, K/V interleaved per page
(``[pages, 2, ...]``) read in place, the softmax / output scales, and the
FlashInfer-compatible entry point (``small_q_attention_b200.flashinfer_compat``).
Every result is checked against the oracle on the same data in the upstream NHD layout."""

import math

import numpy as np
import pytest
import torch

from oracle import cache_append_reference, paged_mtp_attention_reference
from tests.test_gpu_parity import assert_close, case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m

    return m


def oracle(c, sm_scale=None, out_scale=1.0):
    q = c["query"].float()
    if sm_scale is not None:  # the oracle's scale is 128**-0.5: fold the ratio into q
        q = q * (sm_scale * math.sqrt(128))
    ref = paged_mtp_attention_reference(q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                        c["num_kv_heads"])
    return ref * out_scale


def hnd(x):  # [P, 16, H, D] -> [P, H, 16, D]
    return x.permute(0, 2, 1, 3).contiguous()


def interleaved(k, v):  # -> one [P, 2, ...] pool
    return torch.stack([k, v], dim=1).contiguous()


@pytest.mark.parametrize("kernel", [1, 2])
@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("pool", ["separate", "interleaved"])
def test_layouts_and_page_strides(sqa, kernel, layout, pool):
    c = case(8, [40, 700, 16, 1500, 8], hkv=2, seed=7)
    k, v = c["key_cache"], c["value_cache"]
    if layout == "HND":
        k, v = hnd(k), hnd(v)
    if pool == "interleaved":
        kv = interleaved(k, v)
        k, v = kv[:, 0], kv[:, 1]
        assert not k.is_contiguous()
    out = sqa.small_q_attention(c["query"], k, v, c["block_tables"], c["seq_lens"], 16, kernel=kernel,
                                kv_layout=layout, num_ctas=37, min_pages_per_cta=1, check=True)
    assert_close(out, oracle(c))


@pytest.mark.parametrize("kernel", [1, 2])
def test_softmax_and_output_scales(sqa, kernel):
    c = case(4, [33, 1024, 4000], seed=3)
    out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                kernel=kernel, sm_scale=0.05, out_scale=0.5, check=True)
    assert_close(out, oracle(c, sm_scale=0.05, out_scale=0.5))


def test_append_in_hnd_and_interleaved_pools(sqa):
    q_len, lens = 4, [40, 513, 2048]
    c = case(q_len, lens, seed=8)
    gen = torch.Generator().manual_seed(9)
    nk = torch.randn(3, q_len, 8, 128, generator=gen).half()
    nv = torch.randn(3, q_len, 8, 128, generator=gen).half()
    ek, ev = cache_append_reference(nk, nv, c["key_cache"].cpu(), c["value_cache"].cpu(), c["block_tables"].cpu(),
                                    c["seq_lens"].cpu())
    as16 = lambda t: t.cpu().contiguous().view(torch.int16).numpy()  # noqa: E731
    kv = interleaved(hnd(c["key_cache"]), hnd(c["value_cache"]))
    sqa.cache_append(nk.cuda(), nv.cuda(), kv[:, 0], kv[:, 1], c["block_tables"], c["seq_lens"], kv_layout="HND",
                     check=True)
    back_k = kv[:, 0].permute(0, 2, 1, 3)  # HND -> NHD
    back_v = kv[:, 1].permute(0, 2, 1, 3)
    assert np.array_equal(as16(back_k), ek.view(np.int16)) and np.array_equal(as16(back_v), ev.view(np.int16))


@pytest.mark.parametrize("layout,form", [("HND", "tuple"), ("HND", "pool"), ("NHD", "tuple"), ("NHD", "pool")])
def test_flashinfer_compatible_entry(sqa, layout, form):
    from small_q_attention_b200.flashinfer_compat import trtllm_batch_decode_with_kv_cache

    q_len = 4
    c = case(q_len, [100, 2000, 8192], seed=12)
    k, v = c["key_cache"], c["value_cache"]
    if layout == "HND":
        k, v = hnd(k), hnd(v)
    kv = (k, v) if form == "tuple" else interleaved(k, v)
    b = c["query"].shape[0]
    query = c["query"].reshape(b * q_len, 32, 128)
    ws = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
    seq_lens = c["seq_lens"].view(torch.uint32)
    out = trtllm_batch_decode_with_kv_cache(query, kv, ws, c["block_tables"], seq_lens, max(c["lens"]),
                                            bmm1_scale=1 / math.sqrt(128), bmm2_scale=1.0, kv_layout=layout,
                                            q_len_per_req=q_len)
    assert out.shape == query.shape
    assert_close(out.view(c["query"].shape), oracle(c))
    scaled = trtllm_batch_decode_with_kv_cache(query, kv, ws, c["block_tables"], seq_lens, max(c["lens"]),
                                               bmm1_scale=0.07, bmm2_scale=2.0, kv_layout=layout, q_len_per_req=q_len)
    assert_close(scaled.view(c["query"].shape), oracle(c, sm_scale=0.07, out_scale=2.0))


def test_flashinfer_compatible_entry_rejects_what_it_does_not_do(sqa):
    from small_q_attention_b200.flashinfer_compat import trtllm_batch_decode_with_kv_cache

    c = case(2, [64, 80], seed=1)
    query = c["query"].reshape(4, 32, 128)
    kv = (hnd(c["key_cache"]), hnd(c["value_cache"]))
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    args = (query, kv, ws, c["block_tables"], c["seq_lens"], 80)
    for kw in ({"window_left": 16}, {"sinks": [torch.zeros(1)]}, {"max_q_len": 2},
               {"bmm1_scale": torch.tensor(0.1)}, {"uses_shared_paged_kv_idx": False}, {"q_len_per_req": 3}):
        with pytest.raises(ValueError):
            trtllm_batch_decode_with_kv_cache(*args, q_len_per_req=kw.pop("q_len_per_req", 2), **kw)


@pytest.mark.parametrize("q_len,kv_form", [(2, "pool"), (4, "tuple"), (8, "pool"), (16, "tuple")])
def test_flashinfer_decode_wrapper_with_q_len_per_req(sqa, q_len, kv_form):
    """FlashInfer's decode wrapper as the upstream drives it for MTP
    (scripts/compare_flashinfer_paths.py:104-121): CSR pages, plan(..., q_len_per_req),
    run(q, kv) with the NHD [pages, 2, 16, Hkv, 128] pool or a (k, v) tuple."""
    from small_q_attention_b200.flashinfer_compat import BatchDecodeWithPagedKVCacheWrapper

    lens = [q_len, 700, 4096, 33]
    c = case(q_len, lens, seed=60 + q_len)
    pages = [(n + 15) // 16 for n in lens]
    indices = torch.cat([c["block_tables"][b, :p] for b, p in enumerate(pages)])
    indptr = torch.tensor([0] + list(np.cumsum(pages)), dtype=torch.int32, device="cuda")
    last = torch.tensor([n - (p - 1) * 16 for n, p in zip(lens, pages)], dtype=torch.int32, device="cuda")
    kv = (c["key_cache"], c["value_cache"]) if kv_form == "tuple" else interleaved(c["key_cache"], c["value_cache"])
    w = BatchDecodeWithPagedKVCacheWrapper(torch.zeros(64 << 20, dtype=torch.int8, device="cuda"), "NHD",
                                           use_tensor_cores=True)
    w.plan(indptr=indptr, indices=indices, last_page_len=last, num_qo_heads=32, num_kv_heads=8, head_dim=128,
           page_size=16, pos_encoding_mode="NONE", q_data_type=torch.float16, kv_data_type=torch.float16,
           q_len_per_req=q_len)
    b = len(lens)
    out = w.run(c["query"].reshape(b * q_len, 32, 128), kv)
    assert out.shape == (b * q_len, 32, 128)
    assert_close(out.view(c["query"].shape), oracle(c))
    with pytest.raises(ValueError):
        w.run(c["query"].reshape(b * q_len, 32, 128), kv, return_lse=True)
    with pytest.raises(ValueError):
        w.plan(indptr, indices, last, 32, 8, 128, 16, pos_encoding_mode="ROPE_LLAMA", q_len_per_req=q_len)
