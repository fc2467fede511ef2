"""The upstream's own CUDA kernels, built unmodified for sm_100a
(``oracle/build_ref_gpu.py``), checked against the CPU oracle on the same inputs.

They are the same-box GPU comparator of ``bench.py --impl reference``; this pins
that what is timed there computes the operator.  Tolerance: the operator
contract's (max-abs 2e-2, element-wise 2e-2 + 1e-2 |ref|).  Skipped when the
upstream extension was not built (no upstream tree where it was built).
"""

import pytest
import torch

from tests.test_gpu_parity import assert_close, case, oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from oracle import build_ref_gpu

    if build_ref_gpu.built_module_path() is None:
        pytest.skip("upstream extension not built")
    return build_ref_gpu.load_module()


@pytest.mark.parametrize("q_len,lens", [(2, [1024]), (4, [8192, 300, 8192, 17]), (8, [4096, 64])])
def test_upstream_v3_v4_match_the_oracle(ref, q_len, lens):
    c = case(q_len, lens, seed=90 + q_len)
    args = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16)
    expected = oracle(c)
    assert_close(ref.forward_v3(*args, 512, max(lens)), expected)  # scripts/run_gpu_matrix.py:116
    assert_close(ref.forward_v4(*args, 512, max(lens)), expected)
