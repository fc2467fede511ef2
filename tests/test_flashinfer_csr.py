"""Host logic of the FlashInfer-compatible decode wrapper (no GPU): the CSR page
layout (indptr / indices / last_page_len) becomes this path's padded page table and
per-request lengths."""

import pytest
import torch

from small_q_attention_b200.flashinfer_compat import csr_to_block_table


def test_csr_to_block_table_ragged_and_empty_requests():
    indptr = torch.tensor([0, 3, 3, 7, 8], dtype=torch.int32)
    indices = torch.tensor([5, 9, 2, 11, 12, 13, 1, 40], dtype=torch.int32)
    last = torch.tensor([4, 16, 16, 1], dtype=torch.int32)
    table, lens = csr_to_block_table(indptr, indices, last)
    assert table.dtype == torch.int32 and lens.dtype == torch.int32
    assert table.tolist() == [[5, 9, 2, 0], [0, 0, 0, 0], [11, 12, 13, 1], [40, 0, 0, 0]]
    assert lens.tolist() == [36, 0, 64, 1]


def test_csr_to_block_table_rejects_bad_layouts():
    with pytest.raises(ValueError):
        csr_to_block_table(torch.tensor([0, 2, 1]), torch.tensor([1, 2]), torch.tensor([3, 3]))
    with pytest.raises(ValueError):
        csr_to_block_table(torch.tensor([0, 2]), torch.tensor([1, 2]), torch.tensor([17]))


def test_decode_wrapper_plan_records_the_length_bounds():
    """plan() reads the layout once on the host: the table, the lengths and both length
    bounds that steer the launch (run passes them to the operator)."""
    from small_q_attention_b200.flashinfer_compat import BatchDecodeWithPagedKVCacheWrapper

    w = BatchDecodeWithPagedKVCacheWrapper(torch.zeros(1 << 10, dtype=torch.uint8), "NHD", use_tensor_cores=True)
    indptr = torch.tensor([0, 3, 3, 7, 8], dtype=torch.int32)
    indices = torch.tensor([5, 9, 2, 11, 12, 13, 1, 40], dtype=torch.int32)
    last = torch.tensor([4, 16, 16, 1], dtype=torch.int32)
    w.plan(indptr, indices, last, 32, 8, 128, 16, q_data_type=torch.float16, q_len_per_req=4)
    assert (w._plan["max_seq_len"], w._plan["min_seq_len"], w._plan["q_len"]) == (64, 0, 4)
    w.plan(torch.tensor([0, 2, 4]), torch.tensor([1, 2, 3, 4]), torch.tensor([16, 9]), 32, 8, 128, 16,
           q_data_type=torch.float16, q_len_per_req=2)
    assert (w._plan["max_seq_len"], w._plan["min_seq_len"]) == (32, 25)
