"""Pin the CPU oracle against golden vectors made by the upstream reference.

The ``.npz`` files under ``tests/golden/`` were produced by
``tests/golden/make_golden.py``, which runs the upstream
``paged_mtp_attention_reference`` (``src/small_q_attention/reference.py:10-74``)
on float32 upcasts of seeded fp16 inputs.
"""

from pathlib import Path

import numpy as np
import pytest

from oracle import paged_mtp_attention_partial, paged_mtp_attention_reference

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


def load_golden(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def test_golden_set_is_present():
    assert len(GOLDEN) >= 10


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_upstream_golden(path):
    c = load_golden(path)
    out = paged_mtp_attention_reference(
        c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
        int(c["page_size"]), int(c["num_kv_heads"]))
    assert out.shape == c["expected"].shape
    np.testing.assert_allclose(out, c["expected"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_partial_form_equals_full_form(path):
    """With mask_lens == seq_lens the (O, LSE) form is the full operator."""
    c = load_golden(path)
    o, lse = paged_mtp_attention_partial(
        c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
        c["seq_lens"], int(c["page_size"]), int(c["num_kv_heads"]))
    np.testing.assert_allclose(o, c["expected"], rtol=1e-5, atol=1e-5)
    assert np.isfinite(lse).all()
