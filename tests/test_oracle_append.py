"""Pin the cache-append oracle (``oracle/cache_append.py``) on CPU.

The upstream has no append function; it defines where token ``t`` of sequence
``b`` lives (page ``block_tables[b, t // 16]``, slot ``t % 16``,
``src/small_q_attention/reference.py:54-59``) and that ``seq_lens`` counts the
appended draft tokens (``reference.py:25``).  The append is pinned to the caches
the upstream reference itself attended when it produced the golden vectors:
blanking the q_len newest tokens of every sequence and appending them again
must restore those caches bit for bit, and the attention oracle on the restored
cache must reproduce the golden output.
"""

from pathlib import Path

import numpy as np
import pytest

from oracle import cache_append_reference, paged_mtp_attention_reference

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


def _newest_tokens(kc, table, lens, q_len, ps):
    """K or V rows of the q_len newest tokens of every sequence, [B, q_len, Hkv, D]."""
    out = np.zeros((len(lens), q_len) + kc.shape[2:], kc.dtype)
    for b, n in enumerate(lens):
        for qi in range(q_len):
            t = int(n) - q_len + qi
            out[b, qi] = kc[table[b, t // ps], t % ps]
    return out


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_append_restores_upstream_golden_caches(path):
    with np.load(path) as z:
        c = {k: z[k] for k in z.files}
    q_len, ps = c["query"].shape[1], int(c["page_size"])
    kc, vc, table, lens = c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"]
    nk = _newest_tokens(kc, table, lens, q_len, ps)
    nv = _newest_tokens(vc, table, lens, q_len, ps)
    kb, vb = kc.copy(), vc.copy()
    for b, n in enumerate(lens):  # blank the newest slots
        for qi in range(q_len):
            t = int(n) - q_len + qi
            kb[table[b, t // ps], t % ps] = -7.0
            vb[table[b, t // ps], t % ps] = -7.0
    k2, v2 = cache_append_reference(nk, nv, kb, vb, table, lens, ps)
    assert np.array_equal(k2.view(np.uint8), kc.view(np.uint8))
    assert np.array_equal(v2.view(np.uint8), vc.view(np.uint8))
    out = paged_mtp_attention_reference(c["query"], k2, v2, table, lens, ps, int(c["num_kv_heads"]))
    np.testing.assert_allclose(out, c["expected"], rtol=1e-5, atol=1e-5)


def test_known_positions():
    """Token qi of sequence b lands in page table[b, t // 16], slot t % 16, t = len - q + qi."""
    q_len, hkv = 3, 2
    lens = np.array([17, 3, 32], np.int32)
    table = np.array([[4, 1, 9], [0, 9, 9], [2, 7, 9]], np.int32)
    kc = np.zeros((10, 16, hkv, 128), np.float16)
    vc = np.zeros_like(kc)
    nk = np.zeros((3, q_len, hkv, 128), np.float16)
    for b in range(3):
        for qi in range(q_len):
            nk[b, qi] = b * 10 + qi + 1
    nv = -nk
    k2, v2 = cache_append_reference(nk, nv, kc, vc, table, lens)
    expect = {(4, 14): 1, (4, 15): 2, (1, 0): 3,        # b=0: t = 14, 15, 16
              (0, 0): 11, (0, 1): 12, (0, 2): 13,       # b=1: t = 0, 1, 2
              (7, 13): 21, (7, 14): 22, (7, 15): 23}    # b=2: t = 29, 30, 31
    for (page, slot), val in expect.items():
        assert np.all(k2[page, slot] == val) and np.all(v2[page, slot] == -val)
    written = np.zeros((10, 16), bool)
    for page, slot in expect:
        written[page, slot] = True
    assert np.all(k2[~written] == 0)


def test_errors_match_the_attention_reference():
    kc = np.zeros((4, 16, 1, 128), np.float16)
    nk = np.zeros((1, 2, 1, 128), np.float16)
    with pytest.raises(ValueError):
        cache_append_reference(nk, nk, kc, kc, np.array([[0]], np.int32), np.array([1], np.int32))
    with pytest.raises(ValueError):
        cache_append_reference(nk, nk, kc, kc, np.array([[0]], np.int32), np.array([17], np.int32))
    with pytest.raises(IndexError):
        cache_append_reference(nk, nk, kc, kc, np.array([[5]], np.int32), np.array([4], np.int32))
