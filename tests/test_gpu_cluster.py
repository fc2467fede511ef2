"""Cluster mode of the tcgen05 kernel: every (sequence, KV head) segment split
evenly over a thread-block cluster of C CTAs, the parts reduced through
distributed shared memory.

The mode only changes the launch, so every case must match the CPU oracle with
the operator's tolerance (``|err| <= 2e-2 + 1e-2 |ref|``, max-abs 2e-2) for every
cluster size, including ragged batches (clusters of short sequences hold CTAs
with no pages), empty sequences, the shard (partial) form, BF16 and FP8 caches,
NaN in unused slots and exact indexing; the automatic choice (from the
``min_seq_len`` / ``max_seq_len`` hints) must give the same result as the
cost-balanced schedule.
"""

import numpy as np
import pytest
import torch

from oracle import paged_mtp_attention_partial
from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu
SIZES = (2, 4, 8, 16)


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m
    from small_q_attention_b200 import _native

    _native.library()
    return m


def run(sqa, c, cluster, **kw):
    try:
        return sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                     c["seq_lens"], 16, check=True, cluster=cluster, **kw)
    except ValueError as e:
        if cluster == 16 and "unsupported" in str(e):
            pytest.skip("16-CTA clusters are not available on this device")
        raise


CASES = [(4, [8192] * 4, 8), (1, [1, 2, 15, 16, 17, 500], 4), (8, [2048, 8, 9, 300], 2),
         (16, [16, 17, 31, 4096], 2), (2, [1024], 8), (12, [12, 200, 777], 2)]


@pytest.mark.parametrize("cluster", SIZES)
@pytest.mark.parametrize("q_len,lens,hkv", CASES, ids=[f"q{q}-n{len(l)}-kv{max(l)}-h{h}" for q, l, h in CASES])
def test_cluster_parity_vs_oracle(sqa, q_len, lens, hkv, cluster):
    c = case(q_len, lens, hkv=hkv, seed=300 + q_len + len(lens))
    assert_close(run(sqa, c, cluster), oracle(c))


@pytest.mark.parametrize("cluster", (4, 16))
def test_cluster_partial_mode_and_empty_sequences(sqa, cluster):
    """The shard form (normalised fp32 O and natural-log LSE) with a causal offset,
    and a batch whose middle sequence holds no tokens (every CTA of its clusters
    has an empty range: O = 0, LSE = -inf)."""
    c = case(8, [3000, 8, 700], hkv=8, seed=41)
    seq = c["seq_lens"].clone()
    seq[1] = 0
    mlen = seq + torch.tensor([0, 8, 100], dtype=torch.int32, device="cuda")
    try:
        o, lse = sqa.small_q_attention_partial(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], seq,
                                               16, mask_lens=mlen, cluster=cluster)
    except ValueError as e:
        if cluster == 16 and "unsupported" in str(e):
            pytest.skip("16-CTA clusters are not available on this device")
        raise
    ro, rl = paged_mtp_attention_partial(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], seq,
                                         mlen, 16, 8)
    assert_close(o, ro)
    got = lse.cpu().numpy()
    assert np.array_equal(np.isneginf(got), np.isneginf(rl))
    fin = np.isfinite(rl)
    np.testing.assert_allclose(got[fin], rl[fin], rtol=1e-4, atol=1e-3)


def test_cluster_bf16_fp8_and_nan_tails(sqa):
    c = case(4, [4000, 37, 1500], hkv=8, seed=43)
    ref = oracle(c)
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    table = c["block_tables"].cpu()
    for b, n in enumerate(c["lens"]):
        if n % 16:  # NaN in the unused slots of each sequence's last page
            last = int(table[b, (n - 1) // 16])
            kc[last, n % 16:] = float("nan")
            vc[last, n % 16:] = float("nan")
    nan_case = dict(c, key_cache=kc, value_cache=vc)
    assert_close(run(sqa, nan_case, 4), ref)
    bf = dict(c, query=c["query"].bfloat16(), key_cache=c["key_cache"].bfloat16(),
              value_cache=c["value_cache"].bfloat16())
    out = run(sqa, bf, 8)
    assert out.dtype == torch.bfloat16
    assert_close(out.float(), oracle(bf))
    f8 = getattr(torch, "float8_e4m3fn", None)
    if f8 is not None:
        c8 = dict(c, key_cache=c["key_cache"].to(f8), value_cache=c["value_cache"].to(f8))
        from tests.test_gpu_fp8 import oracle as oracle_fp8

        assert_close(run(sqa, c8, 4), oracle_fp8(c8))


@pytest.mark.parametrize("q_len", [2, 8, 16])
def test_cluster_one_hot_indexing_exact(sqa, q_len):
    from tests.test_oracle_known import one_hot_case

    lens = [q_len, 17, 33, 64, 100, 128]
    q, k, v, table, lens_np, expected = one_hot_case(q_len, lens, num_kv_heads=2, seed=q_len)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    c = dict(query=t(q), key_cache=t(k), value_cache=t(v), block_tables=t(table), seq_lens=t(lens_np))
    out = run(sqa, c, 2)
    np.testing.assert_allclose(out.float().cpu().numpy(), expected, rtol=2e-3, atol=1e-3)


def test_cluster_auto_from_length_hints(sqa):
    """Near-uniform hints select cluster mode; its result equals the cost-balanced
    schedule's within the tolerance, and repeated calls are bit-identical."""
    c = case(4, [8192] * 4, hkv=8, seed=45)
    args = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16, 8192)
    off = sqa.small_q_attention(*args, cluster=1, check=True)
    auto = sqa.small_q_attention(*args, min_seq_len=8192, check=True)
    assert_close(auto, off)
    for _ in range(3):
        assert torch.equal(auto, sqa.small_q_attention(*args, min_seq_len=8192))
    assert_close(auto, oracle(c))


def test_cluster_rejected_for_the_warp_level_kernel(sqa):
    c = case(2, [64], hkv=2, seed=1)
    with pytest.raises(ValueError):
        sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                              kernel=1, cluster=4)
    with pytest.raises(ValueError):
        sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                              cluster=3)
