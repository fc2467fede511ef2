"""sqa_forward_timed: the measurement entry point does the work of sqa_forward, eagerly
and inside a CUDA graph, where its events are side-branch nodes of the graph.

Each captured call's "before" event fires when the previous call's last kernel ends and
its "after" event when its split-KV kernel ends, so inside one replay:
* every interval is positive and shorter than the replay;
* intervals of consecutive calls do not overlap (call k's "after" precedes call k+1's
  "before", up to when the front end takes the records: the merge kernel runs between);
* the outputs equal the oracle's, as with sqa_forward.
"""

import ctypes

import pytest
import torch

from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from small_q_attention_b200 import _native

    return _native.library()


def _prepared(lib, c, kernel):
    from small_q_attention_b200 import _native
    from small_q_attention_b200.attention import _fill_args

    a = _fill_args(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], None,
                   max(c["lens"]), 0, 0, kernel)
    out = torch.empty_like(c["query"])
    a.out = out.data_ptr()
    st = ctypes.c_int(0)
    nbytes = lib.sqa_workspace_bytes(ctypes.byref(a), torch.cuda.current_device(), ctypes.byref(st))
    _native.check(st.value, "sqa_workspace_bytes")
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    return a, out, ws


def _call(lib, a, ws, stream, e0, e1):
    from small_q_attention_b200 import _native

    code = lib.sqa_forward_timed(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
                                 ctypes.c_void_p(stream), ctypes.c_void_p(e0), ctypes.c_void_p(e1))
    _native.check(code, "sqa_forward_timed")


@pytest.mark.parametrize("kernel", [1, 2])
def test_timed_eager_matches_oracle(lib, kernel):
    c = case(4, [3000, 17, 8192], hkv=8, seed=61)
    a, out, ws = _prepared(lib, c, kernel)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    e0.record(stream)  # creates the CUDA events (torch creates them lazily, at the first record)
    e1.record(stream)
    _call(lib, a, ws, stream.cuda_stream, e0.cuda_event, e1.cuda_event)
    torch.cuda.synchronize()
    assert e0.elapsed_time(e1) > 0
    assert_close(out, oracle(c))


@pytest.mark.parametrize("kernel", [1, 2])
def test_timed_side_branch_events_in_graph(lib, kernel):
    c = case(4, [8192] * 4, hkv=8, seed=62)
    a, out, ws = _prepared(lib, c, kernel)
    K = 6
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    stream = torch.cuda.Stream()
    for e0, e1 in evs:  # creates the CUDA events
        e0.record(stream)
        e1.record(stream)
    start = torch.cuda.Event(enable_timing=True, external=True)
    end = torch.cuda.Event(enable_timing=True, external=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        start.record()
        for e0, e1 in evs:
            _call(lib, a, ws, torch.cuda.current_stream().cuda_stream, e0.cuda_event, e1.cuda_event)
        end.record()
    out.zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert_close(out, oracle(c))
    total = start.elapsed_time(end)
    spans = [e0.elapsed_time(e1) for e0, e1 in evs]
    assert all(0 < s < total for s in spans), (spans, total)
    for k in range(K - 1):  # call k's split ends before call k+1's "before" event (its merge runs between;
        # 5 us of slack for when the front end takes the two records)
        assert evs[k][1].elapsed_time(evs[k + 1][0]) >= -5e-3
    assert sum(spans[1:]) < total
    del g
