"""The torch extension's operators on the GPU: ``torch.ops.sqa_b200.*`` and the
direct entry behind ``small_q_attention`` compute the same result as the C ABI
called through ctypes, and ``torch.compile`` traces the operator without a graph
break (fullgraph, ``aot_eager``: the operator is not lowered or replaced).
"""

import ctypes

import pytest
import torch

from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sqa():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import small_q_attention_b200 as m

    return m


def _ctypes_forward(c):
    """The same call straight through the C ABI (ctypes), as a second path."""
    from small_q_attention_b200 import _native
    from small_q_attention_b200.attention import _fill_args

    lib = _native.library()
    out = torch.empty_like(c["query"])
    a = _fill_args(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], None, 0, 0, 0)
    a.out = out.data_ptr()
    st = ctypes.c_int(0)
    need = lib.sqa_workspace_bytes(ctypes.byref(a), torch.cuda.current_device(), ctypes.byref(st))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    assert lib.sqa_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(need),
                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    return out


def test_ops_equal_the_c_abi(sqa):
    c = case(4, [3000, 77, 1024], seed=41)
    args = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)
    a = torch.ops.sqa_b200.small_q_attention(*args)
    b = sqa.small_q_attention(*args)
    r = _ctypes_forward(c)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, r)
    assert_close(a, oracle(c))
    o, lse = torch.ops.sqa_b200.small_q_attention_partial(*args)
    o2, lse2 = sqa.small_q_attention_partial(*args)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    assert_close(o.half(), oracle(c))


def test_torch_compile_traces_the_operator(sqa):
    c = case(8, [2000, 500], seed=43)

    def step(q, k, v, bt, sl):
        return torch.ops.sqa_b200.small_q_attention(q * 1.0, k, v, bt, sl, 16) + 0.0

    compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
    args = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"])
    assert torch.equal(compiled(*args), step(*args))


def test_direct_entry_errors(sqa):
    c = case(2, [64], hkv=2, seed=1)
    args = [c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16]
    with pytest.raises(ValueError):
        sqa.small_q_attention("not a tensor", *args[1:])
    with pytest.raises(ValueError):
        sqa.small_q_attention(c["query"][:, :, :, :64], *args[1:])  # not contiguous / head_dim
    with pytest.raises(ValueError):
        sqa.small_q_attention(*args, out=torch.empty(1, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        sqa.small_q_attention(*args, workspace=torch.zeros(16, dtype=torch.uint8, device="cuda"))
