"""The plan/run wrapper (``PagedMTPAttention``): parity with the oracle, CUDA-graph
capture and replay with new inputs, append + attend in one step, plan checks."""

import numpy as np
import pytest
import torch

from oracle import cache_append_reference
from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m

    return m


def _plan(sqa, c, kernel=0):
    q = c["query"]
    return sqa.PagedMTPAttention(q.device, kernel=kernel).plan(
        q.shape[0], q.shape[1], c["key_cache"].shape[2], c["key_cache"].shape[0], c["block_tables"].shape[1],
        max(c["lens"]))


@pytest.mark.parametrize("kernel", [0, 1, 2])
@pytest.mark.parametrize("q_len,lens", [(2, [33, 1000]), (4, [4096] * 4), (8, [17, 300, 8192]), (16, [2000])])
def test_run_matches_oracle(sqa, kernel, q_len, lens):
    c = case(q_len, lens, seed=q_len + len(lens))
    attn = _plan(sqa, c, kernel)
    assert attn.selected_kernel in (1, 2) and (kernel == 0 or attn.selected_kernel == kernel)
    out = attn.run(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], check=True)
    assert_close(out, oracle(c))


def test_graph_capture_and_replay_with_new_inputs(sqa):
    c = case(4, [5000, 700, 9000], seed=3)
    attn = _plan(sqa, c)
    q = c["query"].clone()
    out = torch.empty_like(q)
    args = (q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"])
    attn.run(*args, out=out)  # warm up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s):
        attn.run(*args, out=out)
    for seed in (11, 12):
        c2 = case(4, [5000, 700, 9000], seed=seed)
        q.copy_(c2["query"])
        c["key_cache"].copy_(c2["key_cache"])
        c["value_cache"].copy_(c2["value_cache"])
        c["block_tables"].copy_(c2["block_tables"])
        g.replay()
        torch.cuda.synchronize()
        assert_close(out, oracle(c2))


def test_run_appends_then_attends(sqa):
    q_len, lens = 4, [40, 513, 2048]
    c = case(q_len, lens, seed=8)
    gen = torch.Generator().manual_seed(9)
    nk = torch.randn(3, q_len, 8, 128, generator=gen).half().cuda()
    nv = torch.randn(3, q_len, 8, 128, generator=gen).half().cuda()
    ek, ev = cache_append_reference(nk.cpu(), nv.cpu(), c["key_cache"].cpu(), c["value_cache"].cpu(),
                                    c["block_tables"].cpu(), c["seq_lens"].cpu())
    attn = _plan(sqa, c)
    out = attn.run(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                   append_keys=nk, append_values=nv, check=True)
    assert np.array_equal(c["key_cache"].cpu().numpy().view(np.uint16), ek.view(np.uint16))
    expected = dict(c, key_cache=torch.from_numpy(ek), value_cache=torch.from_numpy(ev))
    assert_close(out, oracle(expected))


def test_shape_checks(sqa):
    c = case(2, [100, 200], seed=1)
    attn = sqa.PagedMTPAttention(c["query"].device)
    with pytest.raises(RuntimeError):
        attn.run(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"])
    _plan(sqa, c)
    attn.plan(2, 4, 8, c["key_cache"].shape[0], c["block_tables"].shape[1])
    with pytest.raises(ValueError):
        attn.run(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"])
    with pytest.raises(ValueError):
        attn.plan(2, 17, 8, 10, 10)


@pytest.mark.parametrize("q_len,lens,expect", [(4, [8192], "split"), (4, [1024] * 4, "cluster")],
                         ids=["aligned-split", "cluster"])
def test_plan_with_length_bounds(sqa, q_len, lens, expect):
    """Both bounds given to plan(): the batch-1 call gets the segment-aligned split and
    the short near-uniform batch the cluster mode, as small_q_attention gives them; run
    matches the oracle eagerly and replayed from a CUDA graph."""
    c = case(q_len, lens, seed=21)
    q = c["query"]
    attn = sqa.PagedMTPAttention(q.device).plan(
        q.shape[0], q.shape[1], c["key_cache"].shape[2], c["key_cache"].shape[0], c["block_tables"].shape[1],
        max(lens), min_seq_len=min(lens))
    sel = attn.selected_kernel
    assert sel >= 10000 if expect == "split" else 100 < sel < 10000, sel
    assert sel == sqa.selected_kernel(q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16,
                                      max(lens), min_seq_len=min(lens))
    ref = oracle(c)
    out = torch.empty_like(q)
    attn.run(q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], out=out, check=True)
    assert_close(out, ref)
    out.zero_()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.Stream()):
        attn.run(q, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], out=out)
    g.replay()
    torch.cuda.synchronize()
    assert_close(out, ref)
    with pytest.raises(ValueError):
        attn.plan(1, 4, 8, 64, 8, 128, min_seq_len=-1)
