"""The segment-aligned split of the tcgen05 kernel: with near-uniform length hints and
fewer (sequence, KV head) segments than CTAs, every segment is split evenly over
k = CTAs / segments CTAs (no CTA crosses a segment boundary) and the merge kernel
combines the k parts of each segment.

The mode only changes the launch, so every case must match the CPU oracle with the
operator's tolerance (``|err| <= 2e-2 + 1e-2 |ref|``, max-abs 2e-2), including wrong
hints (ragged lengths and empty sequences under a "uniform" hint), the shard (partial)
form with a causal offset, BF16 and FP8 caches; the automatic choice is reported by
``selected_kernel`` as ``2 + 10000 * k``.
"""

import numpy as np
import pytest
import torch

from oracle import paged_mtp_attention_partial
from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m
    from small_q_attention_b200 import _native

    _native.library()
    return m


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def _args(c):
    return (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)


# (q_len, lens, KV heads, kernel): kernel 0 = the automatic choice (the tcgen05 kernel at
# these sizes); q_len 1-2 calls of this size run the warp-level kernel unless the tcgen05
# kernel is requested
ALIGNED = [(4, [8192], 8, 0), (16, [8192], 8, 0), (1, [6000, 6000], 8, 2), (8, [4100, 4000, 3900], 8, 0),
           (2, [20000], 2, 2)]


@pytest.mark.parametrize("q_len,lens,hkv,kernel", ALIGNED,
                         ids=["q4-b1-kv8k", "q16-b1-kv8k", "q1-b2", "q8-b3-ragged", "q2-hkv2-k74"])
def test_aligned_parity_vs_oracle(sqa, q_len, lens, hkv, kernel):
    c = case(q_len, lens, hkv=hkv, seed=500 + q_len + len(lens))
    hint = dict(min_seq_len=min(lens), kernel=kernel)
    segs = len(lens) * hkv
    sel = sqa.selected_kernel(*_args(c), max(lens), **hint)
    assert sel == 2 + 10000 * (_sms() // segs), sel
    out = sqa.small_q_attention(*_args(c), max(lens), check=True, **hint)
    ref = oracle(c)
    assert_close(out, ref)
    # the cost-balanced schedule (no min hint) agrees within the tolerance; repeats are bit-identical
    assert sqa.selected_kernel(*_args(c), max(lens), kernel=kernel) in (1, 2)
    assert_close(sqa.small_q_attention(*_args(c), max(lens), kernel=kernel, check=True), ref)
    for _ in range(2):
        assert torch.equal(out, sqa.small_q_attention(*_args(c), max(lens), **hint))


def test_aligned_wrong_hint_ragged_and_empty_partial(sqa):
    """A "uniform" hint over ragged lengths and an empty sequence: segments of every
    length (0 pages, fewer pages than CTAs, a whole segment in one CTA) in the shard
    form (normalised fp32 O, natural-log LSE) with a causal offset."""
    lens = [9000, 8, 4000, 16]  # 4 x 4 KV heads = 16 segments, 9 CTAs each; the last one page long
    c = case(8, lens, hkv=4, seed=71)
    seq = c["seq_lens"].clone()
    seq[1] = 0
    mlen = seq + torch.tensor([0, 8, 100, 0], dtype=torch.int32, device="cuda")
    sel = sqa.selected_kernel(*_args(c), 9000, min_seq_len=9000)
    assert sel >= 10000, sel
    o, lse = sqa.small_q_attention_partial(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], seq, 16,
                                           mask_lens=mlen, max_seq_len=9000, min_seq_len=9000)
    ro, rl = paged_mtp_attention_partial(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], seq,
                                         mlen, 16, 4)
    assert_close(o, ro)
    got = lse.cpu().numpy()
    assert np.array_equal(np.isneginf(got), np.isneginf(rl))
    fin = np.isfinite(rl)
    np.testing.assert_allclose(got[fin], rl[fin], rtol=1e-4, atol=1e-3)


def test_aligned_wrong_hint_full_output(sqa):
    lens = [12000, 17, 5000]
    c = case(4, lens, hkv=8, seed=72)
    sel = sqa.selected_kernel(*_args(c), 12000, min_seq_len=12000)
    assert sel >= 10000, sel
    assert_close(sqa.small_q_attention(*_args(c), 12000, min_seq_len=12000, check=True), oracle(c))


def test_aligned_bf16_and_fp8(sqa):
    c = case(4, [8192], hkv=8, seed=73)
    bf = dict(c, query=c["query"].bfloat16(), key_cache=c["key_cache"].bfloat16(),
              value_cache=c["value_cache"].bfloat16())
    out = sqa.small_q_attention(*_args(bf), 8192, min_seq_len=8192, check=True)
    assert out.dtype == torch.bfloat16
    assert_close(out.float(), oracle(bf))
    f8 = getattr(torch, "float8_e4m3fn", None)
    if f8 is not None:
        c8 = dict(c, key_cache=c["key_cache"].to(f8), value_cache=c["value_cache"].to(f8))
        from tests.test_gpu_fp8 import oracle as oracle_fp8

        assert sqa.selected_kernel(*_args(c8), 8192, min_seq_len=8192) >= 10000
        assert_close(sqa.small_q_attention(*_args(c8), 8192, min_seq_len=8192, check=True), oracle_fp8(c8))


def test_aligned_not_chosen_where_it_idles_ctas(sqa):
    """Four sequences x 8 KV heads = 32 segments: 4 CTAs each would leave 20 of 148 SMs
    idle, so the cost-balanced schedule stays; short segments (< 16 pages per CTA) too."""
    c = case(4, [8192] * 4, hkv=8, seed=74)
    if _sms() == 148:
        assert sqa.selected_kernel(*_args(c), 8192, min_seq_len=8192) < 10000
    c = case(4, [1024], hkv=8, seed=75)
    assert sqa.selected_kernel(*_args(c), 1024, min_seq_len=1024) < 10000
