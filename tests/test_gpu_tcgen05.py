"""GPU parity of the tcgen05 / tensor-memory kernel (``kernel=2``).

Same cases and tolerance as ``test_gpu_parity.py``: the tcgen05 path must match
the CPU oracle and, bit for bit where the schedule is the same, be
deterministic across calls.
"""

import numpy as np
import pytest
import torch

from oracle import paged_mtp_attention_partial, paged_mtp_attention_reference
from tests.test_gpu_parity import PARITY, assert_close, case, oracle

pytestmark = pytest.mark.gpu

TC = 2


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m
    from small_q_attention_b200 import _native

    _native.library()
    return m


def run(sqa, c, **kw):
    return sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                 c["seq_lens"], c["page_size"], check=True, kernel=TC, **kw)


@pytest.mark.parametrize("q_len,lens,hkv,page_mode", PARITY,
                         ids=[f"q{q}-n{len(l)}-kv{max(l)}-h{h}-{m}" for q, l, h, m in PARITY])
def test_tc_parity_vs_oracle(sqa, q_len, lens, hkv, page_mode):
    c = case(q_len, lens, hkv=hkv, page_mode=page_mode, seed=len(lens) * 100 + q_len)
    assert_close(run(sqa, c), oracle(c))


@pytest.mark.parametrize("num_ctas", [1, 3, 64, 296, 1000])
def test_tc_forced_splits(sqa, num_ctas):
    c = case(8, [40, 700, 16, 1500, 8], hkv=2, seed=7)
    assert_close(run(sqa, c, num_ctas=num_ctas, min_pages_per_cta=1), oracle(c))


@pytest.mark.parametrize("q_len", [1, 2, 4, 8, 16])
def test_tc_one_hot_indexing_exact(sqa, q_len):
    from tests.test_oracle_known import one_hot_case

    lens = [q_len, 17, 33, 64, 100, 128]
    q, k, v, table, lens_np, expected = one_hot_case(q_len, lens, num_kv_heads=2, seed=q_len)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = sqa.small_q_attention(t(q), t(k), t(v), t(table), t(lens_np), 16, check=True, kernel=TC)
    np.testing.assert_allclose(out.float().cpu().numpy(), expected, rtol=2e-3, atol=1e-3)


def test_tc_outliers_and_nan_tail(sqa):
    c = case(16, [3000, 517, 9000], seed=11, k_outlier_frac=0.05)
    assert_close(run(sqa, c), oracle(c))
    c = case(12, [37, 50, 16], hkv=2, seed=5)
    ref = oracle(c)
    kc, vc = c["key_cache"].clone(), c["value_cache"].clone()
    table = c["block_tables"].cpu()
    for b, n in enumerate(c["lens"]):
        if n % 16:
            last = int(table[b, (n - 1) // 16])
            kc[last, n % 16:] = float("nan")
            vc[last, n % 16:] = float("nan")
    out = sqa.small_q_attention(c["query"], kc, vc, c["block_tables"], c["seq_lens"], 16, check=True, kernel=TC)
    assert_close(out, ref)


def test_tc_partial_mode(sqa):
    q_len, n, hkv = 16, 5000, 8
    c = case(q_len, [n], hkv=hkv, seed=21, pool_factor=1.0)
    lo, hi = 100, 200
    table = c["block_tables"][:, lo:hi].contiguous()
    seq = torch.tensor([(hi - lo) * 16], dtype=torch.int32, device="cuda")
    mlen = torch.tensor([n - lo * 16], dtype=torch.int32, device="cuda")
    o, lse = sqa.small_q_attention_partial(c["query"], c["key_cache"], c["value_cache"], table, seq, 16,
                                           mask_lens=mlen, check=True, kernel=TC)
    ro, rl = paged_mtp_attention_partial(c["query"], c["key_cache"], c["value_cache"], table, seq, mlen, 16, hkv)
    assert_close(o, ro)
    np.testing.assert_allclose(lse.cpu().numpy(), rl, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("q_len", [5, 8, 16])
def test_tc_large_pool_repeat(sqa, q_len):
    from small_q_attention_b200.workloads import make_case

    c = make_case(16, q_len, [8192] * 16, hkv=8, pool_factor=1.0, seed=77, device="cuda")
    first = run(sqa, c, max_seq_len=8192)
    for _ in range(4):
        assert torch.equal(first, run(sqa, c, max_seq_len=8192))
    kc, vc = c["key_cache"].cpu(), c["value_cache"].cpu()
    for b in (0, 15):
        ref = paged_mtp_attention_reference(c["query"][b:b + 1], kc, vc, c["block_tables"][b:b + 1],
                                            c["seq_lens"][b:b + 1], 16, 8)
        assert_close(first[b:b + 1], ref)


def test_tc_workspace_shared_across_shapes(sqa):
    """One workspace for calls of different shapes, interleaved: the in-kernel
    merge's per-segment counters of one shape are left in place when the next
    shape runs, and the launch generation keeps them apart."""
    cases = [case(4, [3000, 900, 5000, 40], hkv=8, seed=31),
             case(8, [700] * 40, hkv=8, seed=32),               # 320 segments
             case(2, [9000], hkv=2, seed=33)]
    refs = [oracle(c) for c in cases]
    ws = torch.zeros(max(sqa.workspace_bytes(c["query"], c["key_cache"], c["value_cache"], c["block_tables"],
                                             c["seq_lens"], 16, kernel=TC) for c in cases),
                     dtype=torch.uint8, device="cuda")
    for i in (0, 1, 0, 2, 1, 2, 0):
        c = cases[i]
        out = sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                                    16, check=True, kernel=TC, workspace=ws, num_ctas=37, min_pages_per_cta=1)
        assert_close(out, refs[i])


def test_tc_empty_sequences_are_zero(sqa):
    """A sequence with seq_lens 0 has no page to visit: its rows are written as 0."""
    c = case(4, [2000, 16, 1200], hkv=8, seed=41)
    ref = oracle(c)
    lens = c["seq_lens"].clone()
    lens[1] = 0
    out = torch.full_like(c["query"], float("nan"))
    # own workspace: the unchecked call leaves SQA_DEV_SEQ_TOO_SHORT in its status word
    ws = torch.zeros(sqa.workspace_bytes(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], lens, 16,
                                         kernel=TC, num_ctas=20, min_pages_per_cta=1),
                     dtype=torch.uint8, device="cuda")
    sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], lens, 16,
                          out=out, kernel=TC, num_ctas=20, min_pages_per_cta=1, workspace=ws)
    assert torch.count_nonzero(out[1]).item() == 0
    assert_close(out[0:1], ref[0:1])
    assert_close(out[2:3], ref[2:3])
