"""Known-answer and contract tests of the CPU oracle.

These restate the upstream unit tests (``tests/test_reference.py``,
``tests/test_reference_edges.py``) against the oracle.  Two upstream fixtures
are broken (``test_reference_edges.py:30`` expands head 0 over two distinct
query heads; ``:58`` reshapes ``arange(8)`` to an impossible shape); the
versions here keep their intent with valid arithmetic.
"""

import numpy as np
import pytest

from oracle import merge_partials, paged_mtp_attention_partial, paged_mtp_attention_reference


def _softmax(x):
    e = np.exp(x - x.max())
    return e / e.sum()


def test_manual_single_head_case():
    # upstream tests/test_reference.py:9-33
    rng = np.random.default_rng(0)
    query = rng.standard_normal((1, 2, 2, 4)).astype(np.float32)
    key_cache = rng.standard_normal((2, 2, 1, 4)).astype(np.float32)
    value_cache = rng.standard_normal((2, 2, 1, 4)).astype(np.float32)
    out = paged_mtp_attention_reference(
        query, key_cache, value_cache, np.array([[0, 1]], np.int32), np.array([4], np.int32), 2, 1)
    keys = key_cache.reshape(4, 4)
    values = value_cache.reshape(4, 4)
    for qi in range(2):
        valid = 4 - 2 + qi + 1
        for qh in range(2):
            p = _softmax(keys[:valid] @ query[0, qi, qh] / 2.0)
            np.testing.assert_allclose(out[0, qi, qh], p @ values[:valid], rtol=1e-5, atol=1e-6)


def test_gqa_grouping_shape_and_mapping():
    # upstream tests/test_reference.py:35-45, plus the head mapping kvh = qh // group
    rng = np.random.default_rng(1)
    query = rng.standard_normal((1, 2, 4, 8)).astype(np.float32)
    key_cache = rng.standard_normal((2, 4, 2, 8)).astype(np.float32)
    value_cache = rng.standard_normal((2, 4, 2, 8)).astype(np.float32)
    out = paged_mtp_attention_reference(
        query, key_cache, value_cache, np.array([[0, 1]], np.int32), np.array([5], np.int32), 4, 2)
    assert out.shape == query.shape
    keys = key_cache.reshape(8, 2, 8)[:5]
    values = value_cache.reshape(8, 2, 8)[:5]
    for qi in range(2):
        valid = 5 - 2 + qi + 1
        for qh in range(4):
            kvh = qh // 2
            p = _softmax(keys[:valid, kvh] @ query[0, qi, qh] / np.sqrt(8))
            np.testing.assert_allclose(out[0, qi, qh], p @ values[:valid, kvh], rtol=1e-5, atol=1e-6)


def test_physical_page_order_fixed():
    # upstream tests/test_reference_edges.py:17-38, with each query head checked on its own
    rng = np.random.default_rng(2)
    query = rng.standard_normal((1, 2, 2, 4)).astype(np.float32)
    key_cache = rng.standard_normal((3, 2, 1, 4)).astype(np.float32)
    value_cache = rng.standard_normal((3, 2, 1, 4)).astype(np.float32)
    table = np.array([[2, 0, 1]], np.int32)
    out = paged_mtp_attention_reference(query, key_cache, value_cache, table, np.array([5], np.int32), 2, 1)
    keys = key_cache[[2, 0, 1]].reshape(6, 4)[:5]
    values = value_cache[[2, 0, 1]].reshape(6, 4)[:5]
    for qi in range(2):
        valid = 5 - 2 + qi + 1
        for qh in range(2):
            p = _softmax(keys[:valid] @ query[0, qi, qh] / 2.0)
            np.testing.assert_allclose(out[0, qi, qh], p @ values[:valid], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("seq_lens", [[1], [4, 4]])
def test_rejects_invalid_metadata(seq_lens):
    # upstream tests/test_reference_edges.py:41-52
    query = np.zeros((1, 2, 2, 4), np.float32)
    cache = np.zeros((3, 2, 1, 4), np.float32)
    with pytest.raises(ValueError):
        paged_mtp_attention_reference(query, cache, cache, np.array([[2, 0, 1]], np.int32),
                                      np.array(seq_lens, np.int32), 2, 1)


def test_rejects_bad_shapes():
    q = np.zeros((1, 2, 3, 4), np.float32)
    cache = np.zeros((2, 2, 2, 4), np.float32)
    with pytest.raises(ValueError):  # 3 query heads over 2 KV heads
        paged_mtp_attention_reference(q, cache, cache, np.zeros((1, 2), np.int32), np.array([4]), 2, 2)
    with pytest.raises(ValueError):  # page size mismatch
        paged_mtp_attention_reference(np.zeros((1, 2, 2, 4), np.float32), cache, cache,
                                      np.zeros((1, 2), np.int32), np.array([4]), 4, 2)


def test_rejects_out_of_range_page_id():
    query = np.zeros((1, 1, 1, 4), np.float32)
    cache = np.zeros((2, 2, 1, 4), np.float32)
    with pytest.raises(IndexError):
        paged_mtp_attention_reference(query, cache, cache, np.array([[0, 5]], np.int32),
                                      np.array([3], np.int32), 2, 1)


def test_zero_qk_gives_uniform_average_fixed():
    # upstream tests/test_reference_edges.py:55-66 with a valid V shape [2, 2, 1, 4]
    query = np.zeros((1, 2, 2, 4), np.float32)
    key_cache = np.zeros((2, 2, 1, 4), np.float32)
    value_cache = np.arange(16, dtype=np.float32).reshape(2, 2, 1, 4)
    out = paged_mtp_attention_reference(query, key_cache, value_cache, np.array([[0, 1]], np.int32),
                                        np.array([4], np.int32), 2, 1)
    v = value_cache.reshape(4, 4)
    np.testing.assert_allclose(out[0, 0], np.broadcast_to(v[:3].mean(0), (2, 4)), rtol=1e-6)
    np.testing.assert_allclose(out[0, 1], np.broadcast_to(v[:4].mean(0), (2, 4)), rtol=1e-6)


def test_high_magnitude_stays_finite():
    # upstream tests/test_reference_edges.py:69-78
    query = np.full((1, 2, 2, 4), 100.0, np.float32)
    key_cache = np.full((2, 2, 1, 4), 100.0, np.float32)
    value_cache = np.ones_like(key_cache)
    out = paged_mtp_attention_reference(query, key_cache, value_cache, np.array([[0, 1]], np.int32),
                                        np.array([4], np.int32), 2, 1)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, np.ones_like(out))


def one_hot_case(q_len, lens, num_kv_heads=2, seed=0):
    """Q = K = 0 (uniform attention) and V[token t, d] = 16 * (d == t): output bin d
    is 16 / (visible tokens) when token d is visible to the row, else 0.  A wrong
    page or a wrong mask moves some bin by at least 16/128."""
    rng = np.random.default_rng(seed)
    page, d = 16, 128
    pages = [(n + page - 1) // page for n in lens]
    pool = 2 * sum(pages)
    ids = rng.permutation(pool).astype(np.int32)
    table = np.full((len(lens), max(pages)), 0x7FFFFFFF, np.int32)
    value_cache = np.zeros((pool, page, num_kv_heads, d), np.float16)
    cursor = 0
    for b, n in enumerate(lens):
        table[b, :pages[b]] = ids[cursor:cursor + pages[b]]
        for t in range(n):
            value_cache[table[b, t // page], t % page, :, t] = 16.0
        cursor += pages[b]
    query = np.zeros((len(lens), q_len, 4 * num_kv_heads, d), np.float16)
    key_cache = np.zeros_like(value_cache)
    expected = np.zeros(query.shape, np.float32)
    for b, n in enumerate(lens):
        for qi in range(q_len):
            visible = n - q_len + qi + 1
            expected[b, qi, :, :visible] = 16.0 / visible
    return query, key_cache, value_cache, table, np.array(lens, np.int32), expected


def test_one_hot_indexing_is_exact():
    q, k, v, table, lens, expected = one_hot_case(4, [4, 17, 33, 128])
    out = paged_mtp_attention_reference(q, k, v, table, lens, 16, 2)
    np.testing.assert_allclose(out, expected, rtol=1e-6, atol=1e-6)


def test_split_sequence_merge_equals_whole():
    """Split one sequence's pages into shards, take (O, LSE) per shard with the
    shard-relative mask length, merge: equals the unsplit operator."""
    rng = np.random.default_rng(5)
    q_len, n, hkv = 8, 150, 2
    pages = (n + 15) // 16
    query = rng.standard_normal((1, q_len, 4 * hkv, 128)).astype(np.float16)
    kc = rng.standard_normal((pages, 16, hkv, 128)).astype(np.float16)
    vc = rng.standard_normal((pages, 16, hkv, 128)).astype(np.float16)
    table = rng.permutation(pages).astype(np.int32)[None]
    whole = paged_mtp_attention_reference(query, kc, vc, table, np.array([n]), 16, hkv)
    # page-aligned cut points; the last shard is shorter than q_len, so the causal
    # tail spans two shards and row 0 sees nothing in the last shard
    cuts = [0, 3, 9, 144 // 16, pages]
    parts_o, parts_lse = [], []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        held = min(n, hi * 16) - lo * 16
        o, lse = paged_mtp_attention_partial(
            query, kc, vc, table[:, lo:hi], np.array([held]), np.array([n - lo * 16]), 16, hkv)
        parts_o.append(o)
        parts_lse.append(lse)
    merged, _ = merge_partials(parts_o, parts_lse)
    np.testing.assert_allclose(merged, whole, rtol=1e-5, atol=1e-5)
    assert np.isneginf(parts_lse[-1][0, 0]).all()  # row 0 has no visible key in the last shard
