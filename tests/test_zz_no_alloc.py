"""sqa_forward_noalloc: the entry point for callers that cannot allocate device memory.

Callers such as a direct C-ABI binding with no CUDA allocator of its own, or a
serving engine that has handed nearly all of HBM to its KV-cache pool, cannot
provide the workspace sqa_forward needs; sqa_forward_noalloc uses a scratch
array built into the library instead.  These tests call it through the C ABI
(ctypes) and compare its output with sqa_forward's and with the CPU oracle,
within the parity tolerance of the other GPU tests, on two calls in a row with
different shapes (the second call runs on scratch that still holds the first
call's data); and they check that a call with a bad page id reports it through
sqa_noalloc_read_device_status without leaking the bit into the next call.
This file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 1e-2


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from small_q_attention_b200 import _native

    return _native.library()


def _case(q_len, lens, seed):
    from small_q_attention_b200.workloads import make_case

    return make_case(len(lens), q_len, lens, hkv=8, pool_factor=1.5, seed=seed, device="cuda",
                     gen_device="cpu")


def _args(c, out):
    from small_q_attention_b200.attention import _fill_args

    a = _fill_args(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], None,
                   0, 0, 0)
    a.out = out.data_ptr()
    return a


def _with_workspace(lib, c):
    """Output of the existing entry point, sqa_forward, with a caller workspace."""
    out = torch.empty_like(c["query"])
    a = _args(c, out)
    st = ctypes.c_int(0)
    need = lib.sqa_workspace_bytes(ctypes.byref(a), torch.cuda.current_device(), ctypes.byref(st))
    assert st.value == 0
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.sqa_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(need),
                           ctypes.c_void_p(stream)) == 0
    torch.cuda.synchronize()
    return out


def _no_alloc(lib, c):
    out = torch.empty_like(c["query"])
    a = _args(c, out)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.sqa_forward_noalloc(ctypes.byref(a), ctypes.c_void_p(stream)) == 0
    torch.cuda.synchronize()
    return out


def _assert_close(out, ref):
    o, r = out.float().cpu().numpy(), ref.float().cpu().numpy()
    assert np.isfinite(o).all()
    err = np.abs(o - r)
    assert (err <= ATOL + RTOL * np.abs(r)).all() and err.max() <= ATOL, f"max err {err.max():.3e}"


def _oracle(c):
    from oracle import paged_mtp_attention_reference

    return torch.from_numpy(paged_mtp_attention_reference(c["query"], c["key_cache"], c["value_cache"],
                                                          c["block_tables"], c["seq_lens"], 16, 8))


def _status(lib, clear=1):
    bits = ctypes.c_uint32(0)
    code = lib.sqa_noalloc_read_device_status(ctypes.byref(bits), clear,
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code in (0, 5)  # SQA_OK, or SQA_ERR_DEVICE when a bit is set
    return bits.value


def test_no_alloc_matches_workspace_entry_two_calls(lib):
    first = _case(8, [8192, 777, 33, 4000], seed=31)     # split sequences -> merge partials
    second = _case(2, [1024, 16, 5000], seed=32)          # other shape, stale scratch from the first
    for c in (first, second):
        out = _no_alloc(lib, c)
        _assert_close(out, _with_workspace(lib, c))
        _assert_close(out, _oracle(c))
        assert _status(lib) == 0


def test_no_alloc_status_of_a_bad_call_does_not_leak(lib):
    from small_q_attention_b200._native import DEV_BAD_PAGE

    c = _case(4, [300, 1000, 40], seed=33)
    bad = dict(c, block_tables=c["block_tables"].clone())
    bad["block_tables"][1, 3] = c["key_cache"].shape[0] + 7  # outside the pool: read as page 0, reported
    _no_alloc(lib, bad)
    assert _status(lib, clear=0) & DEV_BAD_PAGE
    out = _no_alloc(lib, c)  # the next call starts from a clean status word
    assert _status(lib) == 0
    _assert_close(out, _oracle(c))


def test_no_alloc_rejects_shapes_beyond_the_scratch(lib):
    from small_q_attention_b200._native import SQA_ERR_WORKSPACE_TOO_SMALL, SqaArgs

    a = SqaArgs()
    dummy = torch.zeros(1024, dtype=torch.float16, device="cuda")
    a.query = a.key_cache = a.value_cache = a.block_tables = a.seq_lens = a.out = dummy.data_ptr()
    a.batch, a.q_len, a.num_q_heads, a.num_kv_heads = 4096, 16, 32, 8
    a.head_dim, a.page_size, a.num_pages, a.max_pages = 128, 16, 1 << 20, 64
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.sqa_forward_noalloc(ctypes.byref(a), ctypes.c_void_p(stream)) == SQA_ERR_WORKSPACE_TOO_SMALL
